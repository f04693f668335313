// linear.cu -- the plain projections around the attention of the Evoformer modules, forward and
// backward: y = x w + b (the forward is gdp_fwd_kernel without its gate, gdp.cu), and here
//   dx = sum_s dy_s w_s^T               (linear_dx_kernel)
//   dw_s = x^T dy_s, db_s = sum_m dy_s  (linear_dw_kernel + a fixed-order sum over row groups)
// for up to kLinSegs column blocks s of the output gradient, each with its own buffer, row
// stride and weight, so one launch serves a projection whose outputs were written to several
// buffers (q, k, v and the gate, say) and reads x once.
//
// The reference ships no backward at all; its forward projection with a fused epilogue is the
// gated dual projection (cuda/volta_ops.cu:143-207), whose tiling these kernels share: weights
// resident in shared memory, row tiles of 128 streamed by TMA, f32 accumulation in tensor
// memory.
#include "host.h"
#include "sm100.cuh"
#include "attention_common.cuh"

namespace cfk {
namespace gdp {
namespace {

constexpr int kLinSegs = 4;

struct LinSegs {
    int nseg;
    int n[kLinSegs];      // columns of segment s
    int atom0[kLinSegs];  // (dx) first 64-column weight atom of segment s in shared memory
    int blk0[kLinSegs];   // (dw) first 128-column block of segment s
    int col0[kLinSegs];   // (dw) first column of segment s in the partial sums
    int atoms, nblocks, ntot;
};

// ------------------------------------------------------------------------------------------
// dx [M, K] = sum_s dy_s [M, n_s] w_s^T: weights resident (64-column atoms of K rows x 128 B,
// the K-major B operand), dy streamed as [128 x 64] panels through a ring of stages (the
// K-major A operand), dx of a row tile in double-buffered tensor memory; two epilogue
// warpgroups (64 columns each) stage 16-bit rows for TMA stores.
// ------------------------------------------------------------------------------------------
struct LinDxLayout {
    int w, stg, dy, ns, bar, total;
};

__host__ __device__ inline LinDxLayout lin_dx_layout(int K, int atoms) {
    LinDxLayout L;
    L.w = 0;
    L.stg = atoms * K * 128;
    L.dy = L.stg + 2 * 16384;
    for (L.ns = 4; L.ns >= 2; --L.ns) {
        L.bar = L.dy + L.ns * 16384;
        L.total = L.bar + 32 * 8 + 16 + 1024;
        if (L.total <= 227 * 1024) {
            break;
        }
    }
    return L;
}

constexpr int kLinDxThreads = 320; // 8 epilogue warps, producer (8), MMA (9)
constexpr int kLinDxProducer = 8;
constexpr int kLinDxMma = 9;

template <typename T>
__global__ void __launch_bounds__(kLinDxThreads, 1)
    linear_dx_kernel(const __grid_constant__ CUtensorMap tm_dy0,
                     const __grid_constant__ CUtensorMap tm_dy1,
                     const __grid_constant__ CUtensorMap tm_dy2,
                     const __grid_constant__ CUtensorMap tm_dy3,
                     const __grid_constant__ CUtensorMap tm_w0,
                     const __grid_constant__ CUtensorMap tm_w1,
                     const __grid_constant__ CUtensorMap tm_w2,
                     const __grid_constant__ CUtensorMap tm_w3,
                     const __grid_constant__ CUtensorMap tm_dx, const LinSegs sg, int M, int K) {
    using E = Elem<T>;
    const LinDxLayout L = lin_dx_layout(K, sg.atoms);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar);
    uint64_t* w_full = bars;
    uint64_t* dy_full = bars + 1;     // [ns]
    uint64_t* dy_empty = bars + 5;    // [ns]
    uint64_t* acc_full = bars + 9;    // [2]
    uint64_t* acc_empty = bars + 11;  // [2] count 8
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.bar + 32 * 8);
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n_mt = (M + 127) / 128;
    const int n_mine = (n_mt - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                       static_cast<int>(gridDim.x);
    const CUtensorMap* tm_dy[kLinSegs] = {&tm_dy0, &tm_dy1, &tm_dy2, &tm_dy3};
    const CUtensorMap* tm_w[kLinSegs] = {&tm_w0, &tm_w1, &tm_w2, &tm_w3};

    if (threadIdx.x == 0) {
        mbar_init(w_full, 1);
        for (int i = 0; i < L.ns; ++i) {
            mbar_init(&dy_full[i], 1);
            mbar_init(&dy_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 8);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == kLinDxMma) {
        tmem_alloc(tmem_slot, 256);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == kLinDxProducer) {
        if (lane == 0) {
            mbar_arrive_expect_tx(w_full, sg.atoms * K * 128);
            for (int s = 0; s < sg.nseg; ++s) {
                for (int a = 0; a < (sg.n[s] + 63) / 64; ++a) {
                    tma_load_3d(smem + L.w + (sg.atom0[s] + a) * K * 128, tm_w[s], w_full, a * 64,
                                0, 0);
                }
            }
            uint32_t g = 0;
            for (int i = 0; i < n_mine; ++i) {
                const int mt = blockIdx.x + i * gridDim.x;
                // the dy rows of the tile after next into L2
                if (i + 2 < n_mine) {
                    for (int s = 0; s < sg.nseg; ++s) {
                        for (int pn = 0; pn < (sg.n[s] + 63) / 64; ++pn) {
                            tma_prefetch_l2_3d(tm_dy[s], pn * 64, (mt + 2 * gridDim.x) * 128, 0);
                        }
                    }
                }
                for (int s = 0; s < sg.nseg; ++s) {
                    for (int pn = 0; pn < (sg.n[s] + 63) / 64; ++pn, ++g) {
                        const int st = g % L.ns;
                        if (g >= static_cast<uint32_t>(L.ns) &&
                            !mbar_wait(&dy_empty[st], ((g / L.ns) - 1) & 1, abort_flag)) {
                            goto done;
                        }
                        mbar_arrive_expect_tx(&dy_full[st], 16384);
                        tma_load_3d(smem + L.dy + st * 16384, tm_dy[s], &dy_full[st], pn * 64,
                                    mt * 128, 0);
                    }
                }
            }
        }
    } else if (warp == kLinDxMma) {
        // whole warp, converged: MMAs and commits are elect.sync-issued
        const uint32_t kId = idesc_f16(128, K, false, false, E::kBf16);
        if (!mbar_wait_w(w_full, 0, abort_flag)) {
            goto done;
        }
        uint32_t g = 0;
        for (int i = 0; i < n_mine; ++i) {
            const int buf = i & 1;
            if (i >= 2 && !mbar_wait_w(&acc_empty[buf], ((i >> 1) - 1) & 1, abort_flag)) {
                goto done;
            }
            tc_fence_after();
            const uint32_t acc = tmem + buf * 128;
            uint32_t accumulate = 0;
            for (int s = 0; s < sg.nseg; ++s) {
                for (int pn = 0; pn < (sg.n[s] + 63) / 64; ++pn, ++g) {
                    const int st = g % L.ns;
                    if (!mbar_wait_w(&dy_full[st], (g / L.ns) & 1, abort_flag)) {
                        goto done;
                    }
                    tc_fence_after();
                    const int ksn = min(4, (sg.n[s] - 64 * pn) / 16);
                    const uint32_t a0 = sbase + L.dy + st * 16384;
                    const uint32_t b0 = sbase + L.w + (sg.atom0[s] + pn) * K * 128;
                    for (int ks = 0; ks < ksn; ++ks) {
                        umma_ss_w(acc, smem_desc(a0 + ks * 32, 16, 1024, kSwizzle128),
                                  smem_desc(b0 + ks * 32, 16, 1024, kSwizzle128), kId,
                                  accumulate);
                        accumulate = 1;
                    }
                    umma_commit_w(&dy_empty[st]);
                }
            }
            umma_commit_w(&acc_full[buf]);
        }
    } else {
        // epilogue: warpgroup w owns dx columns [64 w, 64 w + 64), thread = row; 16-bit rows
        // staged in a 128-byte-swizzled [128 x 64] box for one TMA store
        const int w = warp >> 2;
        const int r = static_cast<int>(attn::warp_lane_base()) + lane;
        const uint32_t lane_off = attn::warp_lane_base() << 16;
        const uint32_t stg = sbase + L.stg + w * 16384;
        const bool leader = (threadIdx.x == 128 * w);
        const int ncol = max(0, min(64, K - 64 * w));
        for (int i = 0; i < n_mine; ++i) {
            const int mt = blockIdx.x + i * gridDim.x;
            const int buf = i & 1;
            const bool ok = mbar_wait(&acc_full[buf], (i >> 1) & 1, abort_flag);
            if (leader) {
                bulk_wait_read<0>(); // the previous store has read the staging box
            }
            if (!named_bar_and(1 + w, 128, ok && !*abort_flag)) {
                goto done;
            }
            __syncwarp();
            tc_fence_after();
            for (int q = 0; q < ncol / 16; ++q) {
                uint32_t v[16];
                tmem_ld16(tmem + lane_off + buf * 128 + 64 * w + 16 * q, v);
                tmem_ld_wait();
                uint32_t o[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    o[e] = E::pack(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1]));
                }
                attn::sts128(stg + r * 128 + ((((2 * q) ^ (r & 7))) << 4),
                             make_uint4(o[0], o[1], o[2], o[3]));
                attn::sts128(stg + r * 128 + ((((2 * q + 1) ^ (r & 7))) << 4),
                             make_uint4(o[4], o[5], o[6], o[7]));
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&acc_empty[buf]);
            }
            fence_proxy_async_smem();
            named_bar_sync(1 + w, 128);
            if (leader && ncol > 0) {
                tma_store_3d(&tm_dx, stg, 64 * w, mt * 128, 0);
                bulk_commit();
            }
        }
    }
done:
    __syncwarp();
    if (warp < 8 && (threadIdx.x & 127) == 0) {
        bulk_wait<0>(); // no store may still read the staging boxes (also on the abort path)
    }
    if (*abort_flag) {
        const unsigned long long t0 = global_ns();
        while (global_ns() - t0 < 200000ull) {
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kLinDxMma) {
        tmem_dealloc(tmem, 256);
    }
}

// ------------------------------------------------------------------------------------------
// dw_s = x^T dy_s and db_s = sum over rows of dy_s, per 128-column block of a segment: a group
// of CTAs per block, each over a strided set of row tiles, accumulating [K x 128] (x^T as the
// MN-major A operand, dy as the MN-major B operand) and the column sums (an all-ones A
// operand against the same dy tile) in tensor memory; each CTA writes its f32 partial sums and
// lin_dw_sum_kernel adds the groups in a fixed order, so the result does not depend on timing.
// ------------------------------------------------------------------------------------------
struct LinDwLayout {
    int stage, x, dy, ones, bar, total, ns;
};

__host__ __device__ inline LinDwLayout lin_dw_layout() {
    LinDwLayout L;
    L.stage = 65536; // x tile (two 64-column panels) + dy block (two 64-column atoms)
    L.ns = 3;
    L.x = 0;
    L.dy = 32768;
    L.ones = L.ns * L.stage;
    L.bar = L.ones + 4096;
    L.total = L.bar + 16 * 8 + 16 + 1024;
    return L;
}

constexpr int kLinDwThreads = 192; // 4 epilogue warps, producer (4), MMA (5)
constexpr int kLinDwProducer = 4;
constexpr int kLinDwMma = 5;
constexpr int kLinDwPrefetch = 4; // row tiles prefetched into L2 ahead of the loads

template <typename T>
__global__ void __launch_bounds__(kLinDwThreads, 1)
    linear_dw_kernel(const __grid_constant__ CUtensorMap tm_x,
                     const __grid_constant__ CUtensorMap tm_dy0,
                     const __grid_constant__ CUtensorMap tm_dy1,
                     const __grid_constant__ CUtensorMap tm_dy2,
                     const __grid_constant__ CUtensorMap tm_dy3, const LinSegs sg,
                     const uint32_t db_mask, float* __restrict__ part, int M, int K,
                     int n_groups) {
    using E = Elem<T>;
    const LinDwLayout L = lin_dw_layout();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar);
    uint64_t* in_full = bars;       // [ns]
    uint64_t* in_empty = bars + 4;  // [ns]
    uint64_t* dw_done = bars + 8;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.bar + 16 * 8);
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n_mt = (M + 127) / 128;
    const int blk = blockIdx.x % sg.nblocks;
    const int group = blockIdx.x / sg.nblocks;
    int seg = 0;
    while (seg + 1 < sg.nseg && blk >= sg.blk0[seg + 1]) {
        ++seg;
    }
    const int c0 = 128 * (blk - sg.blk0[seg]);       // first column of the block in its segment
    const int ncols = min(128, sg.n[seg] - c0);        // columns of the block
    const bool with_db = (db_mask >> seg) & 1u;
    const int n_mine = (n_mt - group + n_groups - 1) / n_groups;
    const CUtensorMap* tm_dy[kLinSegs] = {&tm_dy0, &tm_dy1, &tm_dy2, &tm_dy3};
    const int xpanels = (K + 63) / 64;
    const int dyatoms = (ncols + 63) / 64;

    if (threadIdx.x == 0) {
        for (int i = 0; i < L.ns; ++i) {
            mbar_init(&in_full[i], 1);
            mbar_init(&in_empty[i], 1);
        }
        mbar_init(dw_done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    {
        // all-ones [128 x 16] operand (interleave layout) for the column sums; the panels and
        // atoms no load writes (K <= 64, a block of <= 64 columns) are zero in every stage
        const uint32_t one = E::kBf16 ? 0x3F80u : 0x3C00u;
        uint32_t* ones = reinterpret_cast<uint32_t*>(smem + L.ones);
        for (int i = threadIdx.x; i < 1024; i += blockDim.x) {
            ones[i] = one | (one << 16);
        }
        for (int st = 0; st < L.ns; ++st) {
            if (xpanels < 2) {
                uint32_t* z = reinterpret_cast<uint32_t*>(smem + st * L.stage + L.x + 16384);
                for (int i = threadIdx.x; i < 4096; i += blockDim.x) {
                    z[i] = 0u;
                }
            }
            if (dyatoms < 2) {
                uint32_t* z = reinterpret_cast<uint32_t*>(smem + st * L.stage + L.dy + 16384);
                for (int i = threadIdx.x; i < 4096; i += blockDim.x) {
                    z[i] = 0u;
                }
            }
        }
        fence_proxy_async_smem();
    }
    if (warp == kLinDwMma) {
        tmem_alloc(tmem_slot, 256);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot; // dw at columns [0, 128), column sums at [128, 256)

    if (warp == kLinDwProducer) {
        if (lane == 0) {
            for (int i = 0; i < n_mine; ++i) {
                const int mt = group + i * n_groups;
                const int st = i % L.ns;
                for (int ip = (i == 0 ? 1 : i + kLinDwPrefetch);
                     ip <= i + kLinDwPrefetch && ip < n_mine; ++ip) {
                    const int mp = group + ip * n_groups;
                    for (int pn = 0; pn < xpanels; ++pn) {
                        tma_prefetch_l2_3d(&tm_x, pn * 64, mp * 128, 0);
                    }
                    for (int a = 0; a < dyatoms; ++a) {
                        tma_prefetch_l2_3d(tm_dy[seg], c0 + 64 * a, mp * 128, 0);
                    }
                }
                if (i >= L.ns && !mbar_wait(&in_empty[st], ((i / L.ns) - 1) & 1, abort_flag)) {
                    goto done;
                }
                mbar_arrive_expect_tx(&in_full[st], (xpanels + dyatoms) * 16384);
                uint8_t* sp = smem + st * L.stage;
                for (int pn = 0; pn < xpanels; ++pn) {
                    tma_load_3d(sp + L.x + pn * 16384, &tm_x, &in_full[st], pn * 64, mt * 128, 0);
                }
                for (int a = 0; a < dyatoms; ++a) {
                    tma_load_3d(sp + L.dy + a * 16384, tm_dy[seg], &in_full[st], c0 + 64 * a,
                                mt * 128, 0);
                }
            }
        }
    } else if (warp == kLinDwMma) {
        // whole warp, converged: MMAs and commits are elect.sync-issued
        constexpr uint32_t kIdDw = idesc_f16(128, 128, true, true, E::kBf16);
        constexpr uint32_t kIdDb = idesc_f16(128, 128, false, true, E::kBf16);
        const uint64_t ones = attn::interleave16_kmajor(sbase + L.ones);
        for (int i = 0; i < n_mine; ++i) {
            const int st = i % L.ns;
            if (!mbar_wait_w(&in_full[st], (i / L.ns) & 1, abort_flag)) {
                goto done;
            }
            tc_fence_after();
            const uint32_t xs = sbase + st * L.stage + L.x;
            const uint32_t dys = sbase + st * L.stage + L.dy;
#pragma unroll 1
            for (int ks = 0; ks < 8; ++ks) {
                // rows [16 ks, 16 ks + 16) of the tile: dw[k, n] += x[m, k] dy[m, n]
                const uint64_t b = smem_desc(dys + ks * 2048, 16384, 1024, kSwizzle128);
                const uint32_t acc = (i > 0 || ks > 0) ? 1u : 0u;
                umma_ss_w(tmem, smem_desc(xs + ks * 2048, 16384, 1024, kSwizzle128), b, kIdDw,
                          acc);
                if (with_db) {
                    umma_ss_w(tmem + 128, ones, b, kIdDb, acc);
                }
            }
            umma_commit_w(&in_empty[st]);
        }
        umma_commit_w(dw_done);
    } else if (warp < 4) {
        // epilogue: thread = row k of dw; partial sums of this group into part
        // [group][K + 1][ntot] (row K: the column sums)
        const int k = 32 * warp + lane;
        const uint32_t lane_off = static_cast<uint32_t>(32 * warp) << 16;
        float* prow = part + (static_cast<int64_t>(group) * (K + 1) + k) * sg.ntot +
                      sg.col0[seg] + c0;
        float* pdb = part + (static_cast<int64_t>(group) * (K + 1) + K) * sg.ntot +
                     sg.col0[seg] + c0;
        if (n_mine > 0) {
            if (!mbar_wait(dw_done, 0, abort_flag)) {
                goto done;
            }
            tc_fence_after();
        }
        for (int q = 0; q < 8; ++q) {
            uint32_t v[16], d[16];
            if (n_mine > 0) {
                tmem_ld16(tmem + lane_off + 16 * q, v);
                tmem_ld16(tmem + lane_off + 128 + 16 * q, d);
                tmem_ld_wait();
            } else {
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    v[e] = 0u;
                    d[e] = 0u;
                }
            }
            if (k < K) {
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    if (16 * q + e < ncols) {
                        prow[16 * q + e] = __uint_as_float(v[e]);
                    }
                }
            }
            if (k == 0) {
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    if (16 * q + e < ncols) {
                        pdb[16 * q + e] = with_db ? __uint_as_float(d[e]) : 0.f;
                    }
                }
            }
        }
    }
done:
    __syncwarp();
    if (*abort_flag) {
        const unsigned long long t0 = global_ns();
        while (global_ns() - t0 < 200000ull) {
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kLinDwMma) {
        tmem_dealloc(tmem, 256);
    }
}

// dw_s [K, n_s] and db_s [n_s] (db_s may be null): the groups' partial sums added in order.
__global__ void lin_dw_sum_kernel(const float* __restrict__ part, int n_groups, int K,
                                  LinSegs sg, float* dw0, float* dw1, float* dw2, float* dw3,
                                  float* db0, float* db1, float* db2, float* db3) {
    const int64_t total = static_cast<int64_t>(K + 1) * sg.ntot;
    float* dws[kLinSegs] = {dw0, dw1, dw2, dw3};
    float* dbs[kLinSegs] = {db0, db1, db2, db3};
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int k = static_cast<int>(i / sg.ntot);
        const int c = static_cast<int>(i % sg.ntot);
        int s = 0;
        while (s + 1 < sg.nseg && c >= sg.col0[s + 1]) {
            ++s;
        }
        const int n = c - sg.col0[s];
        float acc = 0.f;
        for (int g = 0; g < n_groups; ++g) {
            acc += part[(static_cast<int64_t>(g) * (K + 1) + k) * sg.ntot + c];
        }
        if (k < K) {
            dws[s][static_cast<int64_t>(k) * sg.n[s] + n] = acc;
        } else if (dbs[s]) {
            dbs[s][n] = acc;
        }
    }
}

// ------------------------------------------------------------------------------------------
// CUDA-core fallbacks (shapes or alignments the tcgen05 kernels do not take)
// ------------------------------------------------------------------------------------------
struct LinPtrs {
    const uint16_t* dy[kLinSegs];
    int64_t ld[kLinSegs];
    const uint16_t* w[kLinSegs];
    float* dw[kLinSegs];
    float* db[kLinSegs];
};

template <typename T>
__global__ void linear_dx_generic_kernel(LinPtrs p, LinSegs sg, uint16_t* __restrict__ dx, int M,
                                         int K) {
    using E = Elem<T>;
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    const int m = blockIdx.y * blockDim.y + threadIdx.y;
    if (m >= M || k >= K) {
        return;
    }
    float a = 0.f;
    for (int s = 0; s < sg.nseg; ++s) {
        for (int n = 0; n < sg.n[s]; ++n) {
            a = fmaf(E::to_float(p.dy[s][m * p.ld[s] + n]),
                     E::to_float(p.w[s][static_cast<int64_t>(k) * sg.n[s] + n]), a);
        }
    }
    dx[static_cast<int64_t>(m) * K + k] = E::from_float(a);
}

// one thread per (k, column): k = K is the column sum
template <typename T>
__global__ void linear_dw_generic_kernel(const uint16_t* __restrict__ x, LinPtrs p, LinSegs sg,
                                         int M, int K) {
    using E = Elem<T>;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    const int k = blockIdx.y;
    if (c >= sg.ntot) {
        return;
    }
    int s = 0;
    while (s + 1 < sg.nseg && c >= sg.col0[s + 1]) {
        ++s;
    }
    const int n = c - sg.col0[s];
    if (k == K && !p.db[s]) {
        return;
    }
    float a = 0.f;
    for (int m = 0; m < M; ++m) {
        const float xv = k < K ? E::to_float(x[static_cast<int64_t>(m) * K + k]) : 1.f;
        a = fmaf(xv, E::to_float(p.dy[s][m * p.ld[s] + n]), a);
    }
    if (k < K) {
        p.dw[s][static_cast<int64_t>(k) * sg.n[s] + n] = a;
    } else {
        p.db[s][n] = a;
    }
}

// ------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------
constexpr int kLinDxWeightBudget = 144 * 1024;

int lin_segs(const char* fn, const cfk_linear_seg* segs, int nseg, int64_t M, int64_t K,
             bool dx, LinSegs* sg, LinPtrs* p) {
    if (!segs || nseg < 1 || nseg > kLinSegs) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: 1..%d segments", fn, kLinSegs);
    }
    if (M < 0 || M > (1ll << 31) - 1 || K <= 0 || K > 65535) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: M in [0, 2^31), K in [1, 65535]", fn);
    }
    *sg = LinSegs{};
    *p = LinPtrs{};
    sg->nseg = nseg;
    for (int s = 0; s < nseg; ++s) {
        const cfk_linear_seg& g = segs[s];
        if (g.n <= 0 || g.n % 8 || g.n > 65535 || g.ld < g.n) {
            return fail(CFK_ERR_INVALID_ARGUMENT,
                        "%s: segment %d needs n > 0, n %% 8 == 0 and ld >= n", fn, s);
        }
        if ((M > 0 && !g.dy) || (dx && !g.w) || (!dx && !g.dw)) {
            return fail(CFK_ERR_INVALID_ARGUMENT, "%s: segment %d: null buffer", fn, s);
        }
        sg->n[s] = static_cast<int>(g.n);
        sg->atom0[s] = sg->atoms;
        sg->atoms += static_cast<int>((g.n + 63) / 64);
        sg->blk0[s] = sg->nblocks;
        sg->nblocks += static_cast<int>((g.n + 127) / 128);
        sg->col0[s] = sg->ntot;
        sg->ntot += static_cast<int>(g.n);
        p->dy[s] = static_cast<const uint16_t*>(g.dy);
        p->ld[s] = g.ld;
        p->w[s] = static_cast<const uint16_t*>(g.w);
        p->dw[s] = g.dw;
        p->db[s] = g.db;
    }
    return CFK_OK;
}

// dy blocks the TMA loads take (16-byte aligned rows); the dx kernel also steps through each
// block 16 columns at a time (n % 16 == 0)
bool lin_dy_fast(const cfk_linear_seg* segs, int nseg, int n_mult) {
    for (int s = 0; s < nseg; ++s) {
        if (segs[s].n % n_mult || segs[s].ld % 8 || !aligned16(segs[s].dy)) {
            return false;
        }
    }
    return true;
}

template <typename T>
int linear_dx_impl(cudaStream_t st, const DeviceInfo& dev, const cfk_linear_seg* segs,
                   const LinSegs& sg, const LinPtrs& p, void* dx, int M, int K) {
    bool fast = K % 16 == 0 && K >= 16 && K <= 128 && aligned16(dx) &&
                lin_dy_fast(segs, sg.nseg, 16) &&
                sg.atoms * K * 128 <= kLinDxWeightBudget;
    for (int s = 0; s < sg.nseg && fast; ++s) {
        fast = aligned16(segs[s].w);
    }
    if (fast) {
        fast = lin_dx_layout(K, sg.atoms).total <= 227 * 1024;
    }
    if (!fast) {
        dim3 block(16, 16), grid((K + 15) / 16, (M + 15) / 16);
        linear_dx_generic_kernel<T><<<grid, block, 0, st>>>(p, sg, static_cast<uint16_t*>(dx), M,
                                                            K);
        return check_launch("linear_dx_generic");
    }
    CUtensorMap tdy[kLinSegs], tw[kLinSegs], tdx;
    for (int s = 0; s < sg.nseg; ++s) {
        CFK_TRY(make_tmap_3d(&tdy[s], segs[s].dy, segs[s].n, M, 1, 2ull * segs[s].ld,
                             2ull * segs[s].ld * M, 64, 128, 1, 128, "linear dy"));
        CFK_TRY(make_tmap_3d(&tw[s], segs[s].w, segs[s].n, K, 1, 2ull * segs[s].n,
                             2ull * segs[s].n * K, 64, K, 1, 128, "linear w"));
    }
    for (int s = sg.nseg; s < kLinSegs; ++s) {
        tdy[s] = tdy[0];
        tw[s] = tw[0];
    }
    CFK_TRY(make_tmap_3d(&tdx, dx, K, M, 1, 2ull * K, 2ull * K * M, 64, 128, 1, 128,
                         "linear dx"));
    const LinDxLayout L = lin_dx_layout(K, sg.atoms);
    auto kern = linear_dx_kernel<T>;
    CFK_TRY(ensure_smem_attr(reinterpret_cast<const void*>(kern), dev.device, 227 * 1024,
                             "linear_dx"));
    const int grid = std::min((M + 127) / 128, dev.num_sms);
    kern<<<grid, kLinDxThreads, L.total, st>>>(tdy[0], tdy[1], tdy[2], tdy[3], tw[0], tw[1], tw[2],
                                               tw[3], tdx, sg, M, K);
    return check_launch("linear_dx");
}

bool lin_dw_fast(const cfk_linear_seg* segs, int nseg, const void* x, int K) {
    return K % 16 == 0 && K >= 16 && K <= 128 && aligned16(x) && lin_dy_fast(segs, nseg, 8);
}

int lin_dw_groups(const LinSegs& sg, int M, int num_sms) {
    const int n_mt = (M + 127) / 128;
    return std::max(1, std::min(n_mt, num_sms / sg.nblocks));
}

template <typename T>
int linear_dw_impl(cudaStream_t st, const DeviceInfo& dev, const void* x,
                   const cfk_linear_seg* segs, const LinSegs& sg, const LinPtrs& p, int M, int K,
                   void* ws, size_t ws_bytes) {
    if (!lin_dw_fast(segs, sg.nseg, x, K)) {
        dim3 block(128), grid((sg.ntot + 127) / 128, K + 1);
        linear_dw_generic_kernel<T><<<grid, block, 0, st>>>(static_cast<const uint16_t*>(x), p,
                                                            sg, M, K);
        return check_launch("linear_dw_generic");
    }
    const int groups = lin_dw_groups(sg, M, dev.num_sms);
    const size_t need = static_cast<size_t>(groups) * (K + 1) * sg.ntot * 4;
    if (!ws || ws_bytes < need) {
        return fail(CFK_ERR_INVALID_ARGUMENT,
                    "cfk_linear_bwd_dw: needs a %zu-byte workspace (got %zu)", need, ws_bytes);
    }
    CUtensorMap tx, tdy[kLinSegs];
    CFK_TRY(make_tmap_3d(&tx, x, K, M, 1, 2ull * K, 2ull * K * M, 64, 128, 1, 128, "linear x"));
    for (int s = 0; s < sg.nseg; ++s) {
        CFK_TRY(make_tmap_3d(&tdy[s], segs[s].dy, segs[s].n, M, 1, 2ull * segs[s].ld,
                             2ull * segs[s].ld * M, 64, 128, 1, 128, "linear dy"));
    }
    for (int s = sg.nseg; s < kLinSegs; ++s) {
        tdy[s] = tdy[0];
    }
    uint32_t db_mask = 0;
    for (int s = 0; s < sg.nseg; ++s) {
        db_mask |= (segs[s].db ? 1u : 0u) << s;
    }
    const LinDwLayout L = lin_dw_layout();
    auto kern = linear_dw_kernel<T>;
    CFK_TRY(ensure_smem_attr(reinterpret_cast<const void*>(kern), dev.device, L.total,
                             "linear_dw"));
    float* part = static_cast<float*>(ws);
    kern<<<sg.nblocks * groups, kLinDwThreads, L.total, st>>>(tx, tdy[0], tdy[1], tdy[2], tdy[3],
                                                              sg, db_mask, part, M, K, groups);
    CFK_TRY(check_launch("linear_dw"));
    const int64_t total = static_cast<int64_t>(K + 1) * sg.ntot;
    const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 4 * dev.num_sms));
    lin_dw_sum_kernel<<<blocks, 256, 0, st>>>(part, groups, K, sg, p.dw[0], p.dw[1], p.dw[2],
                                              p.dw[3], p.db[0], p.db[1], p.db[2], p.db[3]);
    return check_launch("linear_dw_sum");
}

} // namespace
} // namespace gdp
} // namespace cfk

using namespace cfk;

extern "C" int cfk_linear_fwd(cfk_stream_t stream, cfk_dtype dtype, const void* x, const void* w,
                              const void* b, void* y0, int64_t ld0, void* y1, int64_t ld1,
                              int64_t n_split, int64_t M, int64_t K, int64_t N) {
    clear_error();
    if (dtype != CFK_F16 && dtype != CFK_BF16) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_linear_fwd: dtype must be CFK_F16 or CFK_BF16");
    }
    if (M < 0 || M > (1ll << 31) - 1 || K <= 0 || K > 65535 || N <= 0 || N > 65535 || N % 8) {
        return fail(CFK_ERR_INVALID_ARGUMENT,
                    "cfk_linear_fwd: M in [0, 2^31), K in [1, 65535], N in [8, 65535] with "
                    "N %% 8 == 0");
    }
    if (!(n_split == N || (n_split > 0 && n_split < N && n_split % 128 == 0))) {
        return fail(CFK_ERR_INVALID_ARGUMENT,
                    "cfk_linear_fwd: n_split must be N or a multiple of 128 in (0, N)");
    }
    if (ld0 < n_split || (n_split < N && ld1 < N - n_split)) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_linear_fwd: row stride below the row width");
    }
    if (M == 0) {
        return CFK_OK;
    }
    if (!x || !w || !y0 || (n_split < N && !y1)) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_linear_fwd: null buffer");
    }
    DeviceInfo dev;
    CFK_TRY(current_device(&dev));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int m = static_cast<int>(M), k = static_cast<int>(K), n = static_cast<int>(N);
    const int ns = static_cast<int>(n_split);
    return dtype == CFK_BF16
               ? gdp::linear_fwd_impl<__nv_bfloat16>(st, dev, x, w, b, y0, ld0, y1, ld1, ns, m,
                                                     k, n)
               : gdp::linear_fwd_impl<__half>(st, dev, x, w, b, y0, ld0, y1, ld1, ns, m, k, n);
}

extern "C" int cfk_linear_bwd_dx(cfk_stream_t stream, cfk_dtype dtype, const cfk_linear_seg* segs,
                                 int n_segs, void* dx, int64_t M, int64_t K) {
    clear_error();
    if (dtype != CFK_F16 && dtype != CFK_BF16) {
        return fail(CFK_ERR_INVALID_ARGUMENT,
                    "cfk_linear_bwd_dx: dtype must be CFK_F16 or CFK_BF16");
    }
    gdp::LinSegs sg;
    gdp::LinPtrs p;
    CFK_TRY(gdp::lin_segs("cfk_linear_bwd_dx", segs, n_segs, M, K, true, &sg, &p));
    if (M == 0) {
        return CFK_OK;
    }
    if (!dx) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_linear_bwd_dx: null dx");
    }
    DeviceInfo dev;
    CFK_TRY(current_device(&dev));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int m = static_cast<int>(M), k = static_cast<int>(K);
    return dtype == CFK_BF16
               ? gdp::linear_dx_impl<__nv_bfloat16>(st, dev, segs, sg, p, dx, m, k)
               : gdp::linear_dx_impl<__half>(st, dev, segs, sg, p, dx, m, k);
}

extern "C" int cfk_linear_bwd_dw_workspace_size(const cfk_linear_seg* segs, int n_segs,
                                                int64_t M, int64_t K, size_t* bytes) {
    clear_error();
    gdp::LinSegs sg;
    gdp::LinPtrs p;
    CFK_TRY(gdp::lin_segs("cfk_linear_bwd_dw_workspace_size", segs, n_segs, M, K, false, &sg,
                          &p));
    if (!bytes) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_linear_bwd_dw_workspace_size: null pointer");
    }
    DeviceInfo dev;
    CFK_TRY(current_device(&dev));
    const int groups = gdp::lin_dw_groups(sg, static_cast<int>(M), dev.num_sms);
    *bytes = static_cast<size_t>(groups) * (K + 1) * sg.ntot * 4;
    return CFK_OK;
}

extern "C" int cfk_linear_bwd_dw(cfk_stream_t stream, cfk_dtype dtype, const void* x,
                                 const cfk_linear_seg* segs, int n_segs, int64_t M, int64_t K,
                                 void* workspace, size_t workspace_bytes) {
    clear_error();
    if (dtype != CFK_F16 && dtype != CFK_BF16) {
        return fail(CFK_ERR_INVALID_ARGUMENT,
                    "cfk_linear_bwd_dw: dtype must be CFK_F16 or CFK_BF16");
    }
    gdp::LinSegs sg;
    gdp::LinPtrs p;
    CFK_TRY(gdp::lin_segs("cfk_linear_bwd_dw", segs, n_segs, M, K, false, &sg, &p));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (M == 0) {
        // no rows: zero gradients
        for (int s = 0; s < n_segs; ++s) {
            if (cudaMemsetAsync(segs[s].dw, 0, static_cast<size_t>(K) * segs[s].n * 4, st) !=
                    cudaSuccess ||
                (segs[s].db &&
                 cudaMemsetAsync(segs[s].db, 0, static_cast<size_t>(segs[s].n) * 4, st) !=
                     cudaSuccess)) {
                return fail(CFK_ERR_LAUNCH, "cfk_linear_bwd_dw: memset failed");
            }
        }
        return CFK_OK;
    }
    if (!x) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_linear_bwd_dw: null x");
    }
    DeviceInfo dev;
    CFK_TRY(current_device(&dev));
    const int m = static_cast<int>(M), k = static_cast<int>(K);
    return dtype == CFK_BF16 ? gdp::linear_dw_impl<__nv_bfloat16>(st, dev, x, segs, sg, p, m, k,
                                                                  workspace, workspace_bytes)
                             : gdp::linear_dw_impl<__half>(st, dev, x, segs, sg, p, m, k,
                                                           workspace, workspace_bytes);
}
