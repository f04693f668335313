// peer.cu -- dbias reduce-scatter over peer memory for attention rows sharded across the GPUs
// of one node (one process per GPU).
//
// The reference runs on one device (cuda/volta_mma_attn.cu:295: grid parallelism only).  With
// the attention rows sharded, every rank holds a partial dbias [H, Sq, Sk] (its rows' sum) and
// rank r needs the full sum of its query rows [r Sq / W, (r + 1) Sq / W) of every head -- the
// rows of the pair representation it owns.  Instead of a library collective, one kernel reads
// those rows straight out of every rank's dbias over NVLink and adds them in rank order:
//
//   every rank's dbias lives in CUDA-IPC memory (cfk_ipc_alloc), followed by a 128-byte sync
//   block; each rank opens its peers' buffers (cfk_ipc_open).  A launch of
//   cfk_dbias_reduce_scatter then:
//     1. the first CTA to start (a local ticket) announces "my dbias is complete" (the kernels
//        before it on the stream wrote it) with one system-scope release store of the call
//        number into every rank's arrival slot for this rank;
//     2. every CTA waits (bounded) until all arrival slots of its own sync block hold the call;
//     3. every CTA adds its share of the W partial row blocks in rank order 0..W-1
//        (deterministic, and the same order on every rank), one warp per output row, 16-byte
//        loads of peer memory (no TMA);
//     4. the last CTA to finish (a second local ticket) announces "done reading" the same way
//        and waits (bounded) until every rank has, so no peer still reads this rank's dbias
//        when the launch completes and the next step may overwrite it.
//   So each call costs 2 W remote stores per rank, not one remote operation per CTA.  The call
//   number is kept in the sync block (device memory) and advanced by the last CTA, so a launch
//   carries no per-call host argument and may be replayed from a CUDA graph.
//
// Waits give up after the device's wait limit (cfk_set_wait_limit_ns), set kStatusTimeoutPeer
// in the status word and let the kernel finish; a rank that never arrives therefore costs its
// peers one wait limit, not a hang.
#include <cstring>

#include "host.h"
#include "sm100.cuh"

namespace cfk {
namespace {

constexpr int kPeerMaxWorld = 8;
constexpr int kRsThreads = 256;
constexpr int kRsVecPerThread = 6;     // 16-byte columns per lane per trip (768 floats: one)
constexpr int kRsMaxCtas = 296;        // 2 per SM of a B200
constexpr uint32_t kStatusTimeoutPeer = 4u; // a wait for another GPU ran past its limit

// Sync block of one rank (128 bytes after its dbias, zeroed by cfk_ipc_alloc).
struct SyncBlock {
    uint32_t arrive[kPeerMaxWorld];  // arrive[r]: the latest call whose dbias rank r finished
    uint32_t depart[kPeerMaxWorld];  // depart[r]: the latest call rank r finished reading
    uint32_t in_ticket;              // CTAs of this rank that started (all calls)
    uint32_t out_ticket;             // CTAs of this rank that finished (all calls)
    uint32_t calls;                  // calls completed on this rank
    uint32_t pad[13];
};
static_assert(sizeof(SyncBlock) == 128, "sync block layout");

struct RsParams {
    const float* src[kPeerMaxWorld]; // dbias of each rank, rank order (this rank's own included)
    SyncBlock* sync[kPeerMaxWorld];  // sync block of each rank
    float* out;                      // [H, Sq / W, Sk]
    int world, rank;
    int H, part, Sk4;                // part = Sq / W rows per rank; Sk4 = Sk / 4
    int Sq;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// A 16-byte load of memory another GPU wrote (system-scope, never a stale cached copy).
__device__ __forceinline__ float4 ld_relaxed_sys_v4(const float* p) {
    float4 v;
    asm volatile("ld.relaxed.sys.global.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}

// Bounded waits for another GPU; false (and kStatusTimeoutPeer recorded) past the limit.
__device__ bool wait_arrival(const uint32_t* slot, uint32_t call, unsigned long long limit) {
    if (static_cast<int32_t>(ld_acquire_sys(slot) - call) >= 0) {
        return true;
    }
    const unsigned long long t0 = global_ns();
    while (static_cast<int32_t>(ld_acquire_sys(slot) - call) < 0) {
        if (global_ns() - t0 > limit) {
            atomicOr(&g_status_word, kStatusTimeoutPeer);
            return false;
        }
        __nanosleep(32);
    }
    return true;
}

// Every rank's slot in `slots` holds `call` (or later); false after a timeout.
__device__ bool wait_all(const uint32_t* slots, int world, uint32_t call,
                         unsigned long long limit) {
    bool ok = true;
    for (int r = 0; r < world && ok; ++r) {
        ok = wait_arrival(slots + r, call, limit);
    }
    return ok;
}

__global__ void __launch_bounds__(kRsThreads) dbias_rs_kernel(const RsParams p) {
    __shared__ uint32_t call_s;
    __shared__ int ok_s;
    SyncBlock* mine = p.sync[p.rank];
    const unsigned long long limit = wait_limit_ns();
    if (threadIdx.x == 0) {
        // the call number: the last CTA of the previous call advanced it before that launch
        // completed, and this launch started after it on the stream
        const uint32_t call = *reinterpret_cast<volatile uint32_t*>(&mine->calls) + 1u;
        call_s = call;
        // 1. the first CTA of the call (it is running, so no CTA waits for one that may not be
        //    resident yet) announces on every rank that this rank's dbias is complete
        if (atomicAdd(&mine->in_ticket, 1u) == (call - 1u) * gridDim.x) {
            __threadfence_system();
            for (int r = 0; r < p.world; ++r) {
                st_release_sys(&p.sync[r]->arrive[p.rank], call);
            }
        }
        // 2. wait for every rank's announcement
        ok_s = wait_all(mine->arrive, p.world, call, limit);
    }
    __syncthreads();
    if (ok_s) {
        // 3. out[h, i, :] = sum over ranks r (in order) of src_r[h, rank * part + i, :]; one
        //    warp per output row (one division per row), lanes over its 16-byte columns
        const int lane = threadIdx.x & 31;
        const int warps = gridDim.x * (kRsThreads / 32);
        const int rows = p.H * p.part;
        for (int row = blockIdx.x * (kRsThreads / 32) + (threadIdx.x >> 5); row < rows;
             row += warps) {
            const int h = row / p.part;
            const int i = row - h * p.part;
            const int64_t src_row = (static_cast<int64_t>(h) * p.Sq + p.rank * p.part + i) * p.Sk4;
            float4* dst = reinterpret_cast<float4*>(p.out) + static_cast<int64_t>(row) * p.Sk4;
            for (int j0 = lane; j0 < p.Sk4; j0 += 32 * kRsVecPerThread) {
                float4 acc[kRsVecPerThread];
#pragma unroll
                for (int u = 0; u < kRsVecPerThread; ++u) {
                    const int j = j0 + 32 * u;
                    acc[u] = j < p.Sk4 ? ld_relaxed_sys_v4(p.src[0] + (src_row + j) * 4)
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int r = 1; r < kPeerMaxWorld; ++r) {
                    if (r < p.world) {
                        float4 v[kRsVecPerThread];
#pragma unroll
                        for (int u = 0; u < kRsVecPerThread; ++u) {
                            const int j = j0 + 32 * u;
                            v[u] = j < p.Sk4 ? ld_relaxed_sys_v4(p.src[r] + (src_row + j) * 4)
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
                        }
#pragma unroll
                        for (int u = 0; u < kRsVecPerThread; ++u) {
                            acc[u].x += v[u].x;
                            acc[u].y += v[u].y;
                            acc[u].z += v[u].z;
                            acc[u].w += v[u].w;
                        }
                    }
                }
#pragma unroll
                for (int u = 0; u < kRsVecPerThread; ++u) {
                    if (j0 + 32 * u < p.Sk4) {
                        dst[j0 + 32 * u] = acc[u];
                    }
                }
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        // 4. this CTA's reads are done (also after a timeout, so that no peer waits for it);
        //    the last CTA of the call announces on every rank that this rank has finished
        //    reading, and waits until every rank has, before the launch may complete
        const uint32_t call = call_s;
        __threadfence();
        if (atomicAdd(&mine->out_ticket, 1u) + 1u == call * gridDim.x) {
            __threadfence_system();
            for (int r = 0; r < p.world; ++r) {
                st_release_sys(&p.sync[r]->depart[p.rank], call);
            }
            wait_all(mine->depart, p.world, call, limit);
            __threadfence();
            *reinterpret_cast<volatile uint32_t*>(&mine->calls) = call;
        }
    }
}

// CTAs of a launch: one warp per output row up to kRsMaxCtas CTAs (a function of the shape
// alone, so every rank launches the same number; the done counters rely on it).
int rs_grid(int64_t rows) {
    const int64_t per_cta = kRsThreads / 32;
    const int64_t g = (rows + per_cta - 1) / per_cta;
    return static_cast<int>(g < 1 ? 1 : (g > kRsMaxCtas ? kRsMaxCtas : g));
}

} // namespace
} // namespace cfk

extern "C" size_t cfk_dbias_exchange_bytes(int64_t H, int64_t Sq, int64_t Sk) {
    if (H <= 0 || Sq <= 0 || Sk <= 0 || H > (1 << 20) || Sq > (1 << 20) || Sk > (1 << 20)) {
        return 0;
    }
    const size_t dbias = static_cast<size_t>(H) * Sq * Sk * sizeof(float);
    return ((dbias + 255) / 256) * 256 + sizeof(cfk::SyncBlock);
}

extern "C" int cfk_ipc_alloc(size_t bytes, void** dptr, void* handle) {
    cfk::clear_error();
    if (!dptr || !handle || bytes == 0) {
        return cfk::fail(CFK_ERR_INVALID_ARGUMENT, "cfk_ipc_alloc: null pointer or zero size");
    }
    cfk::DeviceInfo info;
    CFK_TRY(cfk::current_device(&info));
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        return cfk::fail(CFK_ERR_LAUNCH, "cfk_ipc_alloc: cudaMalloc(%zu): %s", bytes,
                         cudaGetErrorString(e));
    }
    e = cudaMemset(p, 0, bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) {
        e = cudaIpcGetMemHandle(&h, p);
    }
    if (e != cudaSuccess) {
        cudaFree(p);
        return cfk::fail(CFK_ERR_LAUNCH, "cfk_ipc_alloc: %s", cudaGetErrorString(e));
    }
    static_assert(sizeof(h) == CFK_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    *dptr = p;
    return CFK_OK;
}

extern "C" int cfk_ipc_open(const void* handle, void** dptr) {
    cfk::clear_error();
    if (!dptr || !handle) {
        return cfk::fail(CFK_ERR_INVALID_ARGUMENT, "cfk_ipc_open: null pointer");
    }
    cfk::DeviceInfo info;
    CFK_TRY(cfk::current_device(&info));
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        return cfk::fail(CFK_ERR_LAUNCH, "cfk_ipc_open: %s", cudaGetErrorString(e));
    }
    *dptr = p;
    return CFK_OK;
}

extern "C" int cfk_ipc_close(void* dptr) {
    cfk::clear_error();
    if (!dptr) {
        return cfk::fail(CFK_ERR_INVALID_ARGUMENT, "cfk_ipc_close: null pointer");
    }
    const cudaError_t e = cudaIpcCloseMemHandle(dptr);
    if (e != cudaSuccess) {
        return cfk::fail(CFK_ERR_LAUNCH, "cfk_ipc_close: %s", cudaGetErrorString(e));
    }
    return CFK_OK;
}

extern "C" int cfk_ipc_free(void* dptr) {
    cfk::clear_error();
    if (!dptr) {
        return cfk::fail(CFK_ERR_INVALID_ARGUMENT, "cfk_ipc_free: null pointer");
    }
    const cudaError_t e = cudaFree(dptr);
    if (e != cudaSuccess) {
        return cfk::fail(CFK_ERR_LAUNCH, "cfk_ipc_free: %s", cudaGetErrorString(e));
    }
    return CFK_OK;
}

extern "C" int cfk_dbias_reduce_scatter(cfk_stream_t stream, void* const* buffers, int world,
                                        int rank, int64_t H, int64_t Sq, int64_t Sk, float* out) {
    cfk::clear_error();
    if (!buffers || !out) {
        return cfk::fail(CFK_ERR_INVALID_ARGUMENT, "cfk_dbias_reduce_scatter: null pointer");
    }
    if (world < 2 || world > cfk::kPeerMaxWorld || rank < 0 || rank >= world) {
        return cfk::fail(CFK_ERR_INVALID_ARGUMENT,
                         "cfk_dbias_reduce_scatter: world %d / rank %d (2 <= world <= %d)",
                         world, rank, cfk::kPeerMaxWorld);
    }
    const size_t total = cfk_dbias_exchange_bytes(H, Sq, Sk);
    if (total == 0 || Sq % world != 0 || Sk % 4 != 0 || H * Sq >= (int64_t(1) << 31)) {
        return cfk::fail(CFK_ERR_INVALID_ARGUMENT,
                         "cfk_dbias_reduce_scatter: H %lld, Sq %lld, Sk %lld (each in [1, 2^20], "
                         "H * Sq < 2^31, Sq a multiple of the world size %d, Sk a multiple of "
                         "4)",
                         static_cast<long long>(H), static_cast<long long>(Sq),
                         static_cast<long long>(Sk), world);
    }
    if (reinterpret_cast<uintptr_t>(out) % 16 != 0) {
        return cfk::fail(CFK_ERR_INVALID_ARGUMENT, "cfk_dbias_reduce_scatter: out not 16-byte "
                         "aligned");
    }
    cfk::RsParams p;
    memset(&p, 0, sizeof(p));
    const size_t sync_off = total - sizeof(cfk::SyncBlock);
    for (int r = 0; r < world; ++r) {
        if (!buffers[r] || reinterpret_cast<uintptr_t>(buffers[r]) % 256 != 0) {
            return cfk::fail(CFK_ERR_INVALID_ARGUMENT,
                             "cfk_dbias_reduce_scatter: buffer of rank %d null or not 256-byte "
                             "aligned", r);
        }
        p.src[r] = static_cast<const float*>(buffers[r]);
        p.sync[r] = reinterpret_cast<cfk::SyncBlock*>(static_cast<char*>(buffers[r]) + sync_off);
    }
    p.out = out;
    p.world = world;
    p.rank = rank;
    p.H = static_cast<int>(H);
    p.part = static_cast<int>(Sq / world);
    p.Sk4 = static_cast<int>(Sk / 4);
    p.Sq = static_cast<int>(Sq);
    cfk::DeviceInfo info;
    CFK_TRY(cfk::current_device(&info));
    cfk::dbias_rs_kernel<<<cfk::rs_grid(H * (Sq / world)), cfk::kRsThreads, 0,
                           reinterpret_cast<cudaStream_t>(stream)>>>(p);
    return cfk::check_launch("dbias_reduce_scatter");
}
