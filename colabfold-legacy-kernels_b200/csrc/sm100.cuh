// sm100.cuh -- thin wrappers around the Blackwell (sm_100a) instructions the kernels use:
// mbarriers with bounded waits, TMA tile loads, tcgen05 MMA / tensor-memory traffic and the
// shared-memory matrix descriptors.  Every wrapper is hand-written inline PTX.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ != 1000)
#error "this library is built for sm_100a only"
#endif

namespace cfk {

// ---------------------------------------------------------------------------------------------
// Device status: a wait that gives up records why here, and the kernel returns early.
// ---------------------------------------------------------------------------------------------
enum : uint32_t {
    kStatusOk = 0,
    kStatusTimeoutBarrier = 1u, // an mbarrier wait ran past its limit
    kStatusAborted = 2u,        // another thread of the CTA gave up first
};

// How long a wait may take before it gives up, per device (cfk_set_wait_limit_ns); one second
// unless changed.
constexpr unsigned long long kDefaultWaitLimitNs = 1000000000ull;

// The device status word (one per process and device; read through cfk_device_status()) and
// the wait limit.  The kernels are compiled as one translation unit (all_kernels.cu) without
// relocatable device code, which lets ptxas honour setmaxnreg; the variables are defined here,
// once, in that unit.
__device__ uint32_t g_status_word = 0;
__device__ unsigned long long g_wait_limit_ns = kDefaultWaitLimitNs;

__device__ __forceinline__ unsigned long long wait_limit_ns() {
    return *reinterpret_cast<volatile unsigned long long*>(&g_wait_limit_ns);
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok)
                 : "r"(smem_u32(bar)), "r"(parity)
                 : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete.  Gives up after the device's wait
// limit (wait_limit_ns()), or as soon as another thread of the CTA has given up
// (*abort != 0).  Returns false on giving up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile uint32_t* abort) {
    if (mbar_try_wait(bar, parity)) {
        return true;
    }
    const unsigned long long t0 = global_ns();
    const unsigned long long limit = wait_limit_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) {
            return true;
        }
        if (*abort) {
            return false;
        }
        if (global_ns() - t0 > limit) {
            *abort = 1;
            atomicOr(&g_status_word, kStatusTimeoutBarrier);
            return false;
        }
    }
}

// mbar_wait by every lane of a converged warp, with a warp-uniform result (a lane that gave up
// makes the whole warp give up), so the warp stays converged for elect.sync issue.
__device__ __forceinline__ bool mbar_wait_w(uint64_t* bar, uint32_t parity,
                                            volatile uint32_t* abort) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort));
}

// The same operations on a 32-bit shared-memory address (one register instead of a 64-bit
// generic pointer; used where register pressure matters).
__device__ __forceinline__ void mbar_arrive_s(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_s(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok)
                 : "r"(bar), "r"(parity)
                 : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint32_t ld_shared_u32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}

// The waiting loop with an explicit limit (ns): gives up when the limit has passed or the
// CTA's abort word (shared-memory address) is set; giving up sets the abort word and records
// kStatusTimeoutBarrier in the status word.  Inlined: an out-of-line call would save and restore
// the caller's live registers through local memory on every wait that does not complete at
// once, which in a pipelined kernel is most of them.
__device__ __forceinline__ bool mbar_wait_limit_s(uint32_t bar, uint32_t parity, uint32_t abort,
                                                  unsigned long long limit) {
    const unsigned long long t0 = global_ns();
    while (true) {
        if (mbar_try_wait_s(bar, parity)) {
            return true;
        }
        if (ld_shared_u32(abort)) {
            return false;
        }
        if (global_ns() - t0 > limit) {
            asm volatile("st.shared.u32 [%0], 1;" ::"r"(abort) : "memory");
            atomicOr(&g_status_word, kStatusTimeoutBarrier);
            return false;
        }
    }
}

// Waits for the phase with the given parity; gives up like mbar_wait (abort = address of the
// CTA's abort word).
__device__ __forceinline__ bool mbar_wait_s(uint32_t bar, uint32_t parity, uint32_t abort) {
    if (mbar_try_wait_s(bar, parity)) {
        return true;
    }
    return mbar_wait_limit_s(bar, parity, abort, wait_limit_ns());
}

// mbar_wait_s by every lane of a converged warp, with a warp-uniform result.
__device__ __forceinline__ bool mbar_wait_s_w(uint32_t bar, uint32_t parity, uint32_t abort) {
    return __all_sync(0xffffffffu, mbar_wait_s(bar, parity, abort));
}

// ---------------------------------------------------------------------------------------------
// Proxy fences
// ---------------------------------------------------------------------------------------------
// Makes this thread's generic-proxy shared-memory writes visible to the async proxy (TMA,
// tcgen05.mma operand reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor) tile loads into this CTA's shared memory
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Prefetches the box at (c0, c1, c2) of a tensor map into L2 (no shared memory, no completion).
__device__ __forceinline__ void tma_prefetch_l2_3d(const CUtensorMap* map, int32_t c0, int32_t c1,
                                                   int32_t c2) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2) {
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
                 "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1),
                 "r"(c2)
                 : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2, int32_t c3) {
    asm volatile("cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
                 "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1),
                 "r"(c2), "r"(c3)
                 : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
                 "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
                 : "memory");
}

// Untiled bulk copy of `bytes` from global into this CTA's shared memory, completing as
// transaction bytes on the mbarrier.  Both addresses 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
                 "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// Tiled add-reduction of a shared-memory box into global memory through a tensor map (f32 map:
// element-wise f32 add, performed at L2).  Completes through the issuing thread's bulk group.
// Out-of-range parts of the box are skipped.  Coordinates must not be negative.
// Tiled store of a shared-memory box into global memory through a tensor map, completed through
// the issuing thread's bulk group.  Out-of-range parts of the box are skipped; coordinates must
// not be negative and the innermost one times the element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int32_t c0,
                                             int32_t c1, int32_t c2) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group"
                 " [%0, {%2, %3, %4}], [%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
                 "r"(src), "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}

__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* map, const void* src,
                                                  int32_t c0, int32_t c1, int32_t c2) {
    asm volatile("cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group"
                 " [%0, {%2, %3, %4}], [%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}

// Rank-4 tiled add-reduction (element type from the map: f32, or f16/bf16 rounded per add).
__device__ __forceinline__ void tma_reduce_add_4d(const CUtensorMap* map, const void* src,
                                                  int32_t c0, int32_t c1, int32_t c2,
                                                  int32_t c3) {
    asm volatile("cp.reduce.async.bulk.tensor.4d.global.shared::cta.add.tile.bulk_group"
                 " [%0, {%2, %3, %4, %5}], [%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
                 : "memory");
}

// Bulk (untiled) add-reduction of f32 data from shared into global memory, completed through
// the bulk async-group of the issuing thread.  Both addresses 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_reduce_add_f32(float* gdst, const void* ssrc,
                                                    uint32_t bytes) {
    asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::
                     "l"(gdst),
                 "r"(smem_u32(ssrc)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Waits until at most N bulk groups of this thread are still reading their shared source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Waits until at most N bulk groups of this thread are incomplete (writes performed).
template <int N>
__device__ __forceinline__ void bulk_wait() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------------------------------------
// Shared-memory matrix descriptors for tcgen05.mma
//
// Bits: [0,14) start >> 4 | [16,30) leading-dim byte offset >> 4 | [32,46) stride-dim byte
// offset >> 4 | [46,48) version = 1 | [61,64) layout (0 none, 2 128B, 4 64B, 6 32B swizzle).
// ---------------------------------------------------------------------------------------------
enum SmemLayout : uint32_t {
    kInterleave = 0,
    kSwizzle128 = 2,
    kSwizzle64 = 4,
    kSwizzle32 = 6,
};

__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes,
                                              uint32_t sbo_bytes, uint32_t layout) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= 1ull << 46;
    d |= static_cast<uint64_t>(layout & 7u) << 61;
    return d;
}

// Instruction descriptor of tcgen05.mma.kind::f16 with an f32 accumulator.
// Bits: [4,6) D format (1 = f32) | [7,10) A format | [10,13) B format (0 f16, 1 bf16) |
// 15 A MN-major | 16 B MN-major | [17,23) N >> 3 | [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool a_mn_major, bool b_mn_major,
                                                 bool bf16) {
    return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
           ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
           (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// ---------------------------------------------------------------------------------------------
// tcgen05: tensor memory allocation, MMA, commit, loads / stores, fences
// ---------------------------------------------------------------------------------------------
// Whole warp.  Writes the allocated tensor-memory address into *slot (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

// Whole warp.
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]   (one thread issues)
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
                 "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
                 : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]   (one thread issues)
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
                 "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
                 : "memory");
}

// Arrives once on the mbarrier when every tcgen05.mma issued so far by this thread completes.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// Warp-converged forms: called by all 32 lanes of a converged warp; one lane, chosen by
// elect.sync, issues.  A stream of tcgen05.mma issued this way runs at the tensor pipe's rate
// (an N = 128 MMA every 64 cycles on B200); the same stream issued by one lane of a diverged
// warp measured 140-220 cycles per instruction.  The elected lane is the same on every call
// of a converged warp, so commits track the MMAs of the issuing lane.
__device__ __forceinline__ void umma_ss_w(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred e, p;\n\t"
                 "elect.sync _|e, 0xffffffff;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
                 "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
                 : "memory");
}

__device__ __forceinline__ void umma_ts_w(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred e, p;\n\t"
                 "elect.sync _|e, 0xffffffff;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
                 "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
                 : "memory");
}

__device__ __forceinline__ void umma_commit_w(uint64_t* bar) {
    asm volatile("{\n\t.reg .pred e;\n\t"
                 "elect.sync _|e, 0xffffffff;\n\t"
                 "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 "\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}

// True on one lane of a converged warp (elect.sync).
__device__ __forceinline__ bool elect_one() {
    uint32_t e;
    asm volatile("{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(e));
    return e != 0;
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Tensor-memory address: lane in bits [16,32), column in [0,16).
__device__ __forceinline__ uint32_t tmem_addr(uint32_t base, uint32_t lane, uint32_t col) {
    return base + (lane << 16) + col;
}

// 32 lanes x 32 bit, 8 / 16 / 32 consecutive columns per thread (lane = thread of the warp).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                   "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                   "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]),
                   "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
                   "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
                   "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
}

__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint32_t (&r)[4]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3])
                 : "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
        : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
                 "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
                 "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]),
                 "r"(r[13]), "r"(r[14]), "r"(r[15])
                 : "memory");
}

// Moves registers between the warpgroups of a CTA (all threads of a warpgroup execute it).  The
// per-thread counts of all warpgroups must add up to the CTA's allocation at launch.
template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// ---------------------------------------------------------------------------------------------
// Small helpers
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 1 / x by the rcp.approx.ftz instruction (at most 1 ulp from the rounded quotient).
__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t elect_lane0() {
    return (threadIdx.x & 31u) == 0u;
}

// Named barrier over `count` threads (a multiple of 32), id 1..15.
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Named barrier that also returns the AND of `v` over the participating threads: every thread
// gets the same answer, so a group can decide together whether to go on.
__device__ __forceinline__ bool named_bar_and(uint32_t id, uint32_t count, bool v) {
    uint32_t r;
    asm volatile("{\n\t.reg .pred p, q;\n\t"
                 "setp.ne.u32 p, %1, 0;\n\t"
                 "bar.red.and.pred q, %2, %3, p;\n\t"
                 "selp.u32 %0, 1, 0, q;\n\t}"
                 : "=r"(r)
                 : "r"(v ? 1u : 0u), "r"(id), "r"(count)
                 : "memory");
    return r != 0;
}

} // namespace cfk
