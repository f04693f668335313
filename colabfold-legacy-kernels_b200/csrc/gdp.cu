// gdp.cu -- gated dual projection, forward and backward.
//
//   out[m, n] = mask[m] * (x @ wp + bp)[m, n] * sigmoid((x @ wg + bg)[m, n])
//
// after volta_gdp_kernel (cuda/volta_ops.cu:109-208) and volta_gdp_wmma_kernel
// (cuda/volta_gdp_wmma.cu:16-97): both products share the x tile and the epilogue is fused.
//
// Forward (tcgen05): a persistent CTA keeps both weight matrices in shared memory (loaded once)
// and streams 128-row tiles of x through TMA.  Per 128-column chunk the MMA warp computes
// p = x wp and g = x wg into tensor memory (double-buffered, so the epilogue of one chunk
// overlaps the MMAs of the next); the biases enter as one extra K=16 MMA step, ones[128 x 16]
// times a bias row, so the epilogue only evaluates mask * p * sigmoid(g) and stores.
//
// Backward (tcgen05, two kernels, both recompute p and g from x):
//   gdp_bwd_dxr: both weight matrices resident in shared memory; per 64-column chunk one
//               N = 128 MMA chain gives [p | g], the epilogue writes dp = dout*mask*s and
//               dg = dout*mask*p*s*(1-s) back into tensor memory as 16-bit pairs, and
//               dx += dp wp^T + dg wg^T runs with A in tensor memory.  Shapes whose weights do
//               not fit take gdp_bwd_dx, which streams 128-column weight chunks and stages
//               dp, dg in shared memory.
//   gdp_bwd_dw: per 64-column chunk (a group of CTAs per chunk), dp and dg split into
//               bf16 hi + lo parts so that dwp = x^T dp, dwg = x^T dg keep f32 accuracy; the
//               bias gradients are f32 column sums; per-CTA sums are added at the end.
//
// Shapes outside the fast paths (K not a multiple of 16 or above 128, weights larger than the
// shared-memory budget, unaligned pointers) take plain CUDA-core kernels.
#include "attention_common.cuh"
#include "host.h"

namespace cfk {
namespace gdp {
namespace {

constexpr int kThreads = 320; // 2 epilogue warpgroups + producer warp + MMA warp
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;

// Forward: warps 0-15 are four epilogue warpgroups (32 output columns each per 128-column
// chunk), then the producer and the MMA warp.  With the fused LayerNorm, warpgroups 4 and 5
// (warps 16-23, 16 rows of a tile each) normalise the x rows and warpgroup 6 holds the
// producer, the MMA warp and two idle warps; setmaxnreg moves registers from warpgroup 6 to
// the LayerNorm warps while the epilogue keeps the launch share:
// 4 x 128 x kEpiRegs + 2 x 128 x kLnRegs + 128 x kMiscRegs = 896 x 72, what the launch gives
// the block (65536 / 896, in units of 8).
template <bool kLn>
struct FwdWarps {
    static constexpr int kEpiWg = 4;
    static constexpr int kCols = 128 / kEpiWg;      // output columns per warpgroup and chunk
    static constexpr int kLnWarp0 = 16;             // (kLn) first LayerNorm warp
    static constexpr int kLnWarps = 8;              // (kLn)
    static constexpr int kLnRows = 128 / kLnWarps;  // rows of a tile per LayerNorm warp
    static constexpr int kProducer = kLn ? kLnWarp0 + kLnWarps : 16;
    static constexpr int kMma = kProducer + 1;
    static constexpr int kThreads = kLn ? 32 * (kProducer + 4) : 576;
    static constexpr int kLaunchRegs = 72;
    static constexpr int kEpiRegs = 72, kLnRegs = 88, kMiscRegs = 40; // (kLn)
    static_assert(!kLn || 4 * kEpiRegs + (kLnWarps / 4) * kLnRegs + kMiscRegs ==
                              (kThreads / 128) * kLaunchRegs, "register split");
};
constexpr int kMaxK = 128;
constexpr int kWeightBudget = 128 * 1024; // both weight matrices, resident

__device__ __forceinline__ float sigmoid_fast(float x) {
    // sigmoid(x) = 0.5 * tanh(x / 2) + 0.5
    float t;
    asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * x));
    return fmaf(0.5f, t, 0.5f);
}

// sigmoid through exp2: f32-accurate (used by the backward, whose f32 outputs need it).
__device__ __forceinline__ float sigmoid_accurate(float x) {
    return rcp_approx(1.0f + ex2(-x * kLog2e));
}

// Offsets of the forward kernel's shared memory (bytes from a 1024-aligned base).
struct FwdLayout {
    int kb;        // K (multiple of 16, <= 128)
    int npad;      // N rounded up to 128
    int x_stage;   // one x tile: ceil(K/64) panels of 128 rows x 128 B
    int xs;        // x stages (2 when they fit beside the weights, else 1)
    int off_x, off_w, off_b, off_ones, off_stg, off_ln, off_bar, total;
};

// gate = false: the plain projection (one weight matrix, one bias operand).
__host__ __device__ inline FwdLayout fwd_layout(int K, int N, bool gate = true) {
    FwdLayout L;
    L.kb = K;
    L.npad = (N + 127) / 128 * 128;
    L.x_stage = ((K + 63) / 64) * 16384;
    for (L.xs = 2; L.xs >= 1; --L.xs) {
        L.off_x = 0;
        // weights per 128-column chunk c: the 64-column atoms wp 2c, wp 2c+1, wg 2c, wg 2c+1
        // (kb rows x 128 B each), so one N = 256 MMA per k-step makes [p | g] of the chunk
        L.off_w = L.xs * L.x_stage;
        // bias operand, per chunk: the 16 column groups of bp, then those of bg
        L.off_b = L.off_w + (gate ? 2 : 1) * L.kb * L.npad * 2;
        L.off_ones = L.off_b + (gate ? 2 : 1) * (L.npad / 8) * 256;
        L.off_stg = L.off_ones + 4096; // output staging: one [128 x 64] box per warpgroup
        L.off_ln = L.off_stg + 2 * 16384; // LayerNorm gamma, beta (f32 [K] each), fused form
        L.off_bar = L.off_ln + 2 * kMaxK * 4;
        L.total = L.off_bar + 16 * 8 + 16 + 1024;
        if (L.total <= 227 * 1024) {
            break;
        }
    }
    return L;
}

// Shared-memory descriptors (see attention_common.cuh for the layouts).
// x tile, K-major, k-step s: panel s/4 of 64 columns, 32 B per 16 columns.
__device__ __forceinline__ uint64_t x_desc(uint32_t x, int s) {
    return smem_desc(x + (s >> 2) * 16384 + (s & 3) * 32, 16, 1024, kSwizzle128);
}
// weight [K rows x n] stored as 64-column atoms of kb rows x 128 B, MN-major, from atom 2c
// on (as many atoms as the MMA's N spans), k-step s.
__device__ __forceinline__ uint64_t w_desc(uint32_t w, int kb, int c, int s) {
    return smem_desc(w + 2 * c * (kb * 128) + s * 2048, kb * 128, 1024, kSwizzle128);
}
// bias row operand [16 x n] (row 0 = bias), MN-major interleave: (kk, n) at
// (n/8)*256 + kk*16 + (n%8)*2; from column 128c on.
__device__ __forceinline__ uint64_t brow_desc(uint32_t b, int c) {
    return smem_desc(b + c * 16 * 256, 128, 256, kInterleave);
}

// LayerNorm prologue of the fused form: z, gamma, beta, eps; optional row statistics.
struct LnIn {
    const uint16_t* z;
    const float* gamma;
    const float* beta;
    float* mean;
    float* rstd;
    float eps;
};

// kLn: x = LayerNorm(z) is never written to memory.  A LayerNorm warpgroup reads the z rows of
// the next tile from global memory while the MMAs of the current one run, normalises them in
// f32 and writes the 16-bit result straight into the x stage in the swizzled layout the MMA
// reads; the producer then loads only the weights.
//
// kGate = false: the plain projection y = x wp + bp (bp may be null), columns [0, n_split) to
// tm_out and [n_split, N) to tm_out2 (n_split a multiple of 128); wg, bg and mask are unused.
template <typename T, bool kLn, bool kGate>
__global__ void __launch_bounds__(FwdWarps<kLn>::kThreads, 1)
    gdp_fwd_kernel(const __grid_constant__ CUtensorMap tm_x,
                   const __grid_constant__ CUtensorMap tm_wp,
                   const __grid_constant__ CUtensorMap tm_wg,
                   const __grid_constant__ CUtensorMap tm_out,
                   const __grid_constant__ CUtensorMap tm_out2, int n_split,
                   const uint16_t* __restrict__ bp, const uint16_t* __restrict__ bg,
                   const uint16_t* __restrict__ mask, int M, int K, int N, const LnIn ln) {
    using E = Elem<T>;
    using FW = FwdWarps<kLn>;
    constexpr int kProducerWarp = FW::kProducer;
    constexpr int kMmaWarp = FW::kMma;
    const FwdLayout L = fwd_layout(K, N, kGate);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.off_bar);
    uint64_t* x_full = bars;        // [2]
    uint64_t* x_empty = bars + 2;   // [2]
    uint64_t* w_full = bars + 4;
    uint64_t* acc_full = bars + 5;  // [2]
    uint64_t* acc_empty = bars + 7; // [2]
    uint64_t* x_ready = bars + 9;   // [2] (kLn) x of the stage normalised by the LN warpgroup
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.off_bar + 16 * 8);
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n_mt = (M + 127) / 128;
    const int n_chunks = L.npad / 128;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&x_full[i], 1);
            mbar_init(&x_empty[i], 1);
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 4 * FW::kEpiWg);
            mbar_init(&x_ready[i], FW::kLnWarps);
        }
        mbar_init(w_full, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    // bias rows (row 0 = bias, rows 1..15 = 0) and ones[128 x 16] (column 0 = 1), in T
    {
        uint16_t* sb = reinterpret_cast<uint16_t*>(smem + L.off_b);
        const int nel = (kGate ? 2 : 1) * (L.npad / 8) * 128; // 16-bit elements of the operand
        for (int i = threadIdx.x; i < nel; i += blockDim.x) {
            const int grp = i / 128, within = i % 128, kk = within / 8, e = within % 8;
            int n = grp * 8 + e, t = 0;
            if constexpr (kGate) {
                const int c = grp / 32; // chunk; t: 0 = bp, 1 = bg
                t = (grp / 16) & 1;
                n = c * 128 + (grp & 15) * 8 + e;
            }
            const bool on = (kk == 0 && n < N && bp != nullptr);
            sb[i] = on ? (t ? bg[n] : bp[n]) : uint16_t(0);
        }
        const uint32_t one = E::kBf16 ? 0x3F80u : 0x3C00u;
        uint32_t* ones = reinterpret_cast<uint32_t*>(smem + L.off_ones);
        for (int i = threadIdx.x; i < 1024; i += blockDim.x) {
            ones[i] = ((i < 512) && ((i & 3) == 0)) ? one : 0u;
        }
        if constexpr (kLn) {
            float* gb = reinterpret_cast<float*>(smem + L.off_ln);
            for (int i = threadIdx.x; i < K; i += blockDim.x) {
                gb[i] = ln.gamma[i];
                gb[kMaxK + i] = ln.beta[i];
            }
        }
        fence_proxy_async_smem();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, 512);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int n_mine = (n_mt - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                       static_cast<int>(gridDim.x);

    if (warp >= kProducerWarp) {
        // producer and MMA warp (with kLn warpgroup 5, whose registers go to the LayerNorm one)
        if constexpr (kLn) {
            setmaxnreg_dec<FW::kMiscRegs>();
        }
      if (warp == kProducerWarp) {
        if (lane == 0) {
            // weights once: 64-column atoms of all K rows
            const int atoms = L.npad / 64;
            mbar_arrive_expect_tx(w_full, (kGate ? 2 : 1) * atoms * L.kb * 128);
            for (int a = 0; a < atoms; ++a) {
                if constexpr (kGate) {
                    const int slot = 4 * (a >> 1) + (a & 1); // wp atom a; wg atom a two further
                    tma_load_3d(smem + L.off_w + slot * L.kb * 128, &tm_wp, w_full, a * 64, 0,
                                0);
                    tma_load_3d(smem + L.off_w + (slot + 2) * L.kb * 128, &tm_wg, w_full,
                                a * 64, 0, 0);
                } else {
                    tma_load_3d(smem + L.off_w + a * L.kb * 128, &tm_wp, w_full, a * 64, 0, 0);
                }
            }
            const int panels = (K + 63) / 64;
            for (int i = 0; i < (kLn ? 0 : n_mine); ++i) {
                const int mt = blockIdx.x + i * gridDim.x;
                const int s = i % L.xs;
                // the x tiles two and three ahead into L2: with one x stage beside the weights,
                // each load is issued only once the previous tile's MMAs are done
                for (int ip = (i == 0 ? 1 : i + 3); ip <= i + 3 && ip < n_mine; ++ip) {
                    for (int pn = 0; pn < panels; ++pn) {
                        tma_prefetch_l2_3d(&tm_x, pn * 64, (blockIdx.x + ip * gridDim.x) * 128, 0);
                    }
                }
                if (i >= L.xs && !mbar_wait(&x_empty[s], ((i / L.xs) - 1) & 1, abort_flag)) {
                    goto done;
                }
                mbar_arrive_expect_tx(&x_full[s], panels * 16384);
                for (int pn = 0; pn < panels; ++pn) {
                    tma_load_3d(smem + L.off_x + s * L.x_stage + pn * 16384, &tm_x, &x_full[s],
                                pn * 64, mt * 128, 0);
                }
            }
        }
    } else if (warp == kMmaWarp) {
        // whole warp, converged: MMAs and commits are elect.sync-issued
        {
            constexpr uint32_t kId = idesc_f16(128, kGate ? 256 : 128, false, true, E::kBf16);
            constexpr int kAtomStep = kGate ? 2 : 1; // 128-column groups per chunk operand
            const uint64_t ones = attn::interleave16_kmajor(sbase + L.off_ones);
            const int ksteps = K / 16;
            if (!mbar_wait_w(w_full, 0, abort_flag)) {
                goto done;
            }
            uint32_t chunk_ctr = 0;
            for (int i = 0; i < n_mine; ++i) {
                const int s = i % L.xs;
                if (!mbar_wait_w(kLn ? &x_ready[s] : &x_full[s], (i / L.xs) & 1, abort_flag)) {
                    goto done;
                }
                tc_fence_after();
                const uint32_t x = sbase + L.off_x + s * L.x_stage;
                for (int c = 0; c < n_chunks; ++c, ++chunk_ctr) {
                    const int bf = chunk_ctr & 1;
                    if (chunk_ctr >= 2 &&
                        !mbar_wait_w(&acc_empty[bf], ((chunk_ctr >> 1) - 1) & 1, abort_flag)) {
                        goto done;
                    }
                    tc_fence_after();
                    // [p | g] of chunk c: columns [0, 128) p, [128, 256) g (the plain
                    // projection: columns [0, 128))
                    const uint32_t acc = tmem + bf * 256;
                    for (int ks = 0; ks < ksteps; ++ks) {
                        umma_ss_w(acc, x_desc(x, ks),
                                  w_desc(sbase + L.off_w, L.kb, kAtomStep * c, ks), kId, ks > 0);
                    }
                    umma_ss_w(acc, ones, brow_desc(sbase + L.off_b, kAtomStep * c), kId, 1);
                    umma_commit_w(&acc_full[bf]);
                }
                umma_commit_w(&x_empty[s]);
            }
        }
      }
    } else if (kLn && warp >= FW::kLnWarp0) {
        // LayerNorm warps.  Warp lw normalises rows [R lw, R lw + R) of each tile (R = kLnRows),
        // two rows at a time: half h = lane / 16 takes row R lw + 2 j + h of row pair j, lane
        // cl = lane % 16 its columns [8 cl, 8 cl + 8) (16 bytes: the warp's loads of a row pair
        // are 512 contiguous bytes).  Row sums go across the 16 lanes by shuffles; gamma and
        // beta of the lane's columns stay in registers.  The z rows of the next tile are loaded
        // while the MMAs of the current one run.
        if constexpr (kLn) {
            setmaxnreg_inc<FW::kLnRegs>();
        }
        const int lw = warp - FW::kLnWarp0;
        const int h = lane >> 4;
        const int cl = lane & 15;
        const int nchk = K / 8; // 16-byte chunks of a row
        const bool col_ok = cl < nchk;
        const float inv_k = 1.0f / static_cast<float>(K);
        float2 gam[4], bet[4];
        {
            const float* gs = reinterpret_cast<const float*>(smem + L.off_ln);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int k0 = col_ok ? 8 * cl + 2 * e : 0;
                gam[e] = make_float2(gs[k0], gs[k0 + 1]);
                bet[e] = make_float2(gs[kMaxK + k0], gs[kMaxK + k0 + 1]);
            }
        }
        constexpr int kPairs = FW::kLnRows / 2;
        uint4 zr[kPairs];
        auto tile_row = [&](int i, int j) {
            return (static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x)) * 128 +
                   FW::kLnRows * lw + 2 * j + h;
        };
        auto load_tile = [&](int i) {
#pragma unroll
            for (int j = 0; j < kPairs; ++j) {
                const int row = tile_row(i, j);
                zr[j] = (col_ok && row < M)
                            ? ld_global_stream_v4(ln.z + static_cast<int64_t>(row) * K + 8 * cl)
                            : make_uint4(0u, 0u, 0u, 0u);
            }
        };
        if (n_mine > 0) {
            load_tile(0);
        }
        for (int i = 0; i < n_mine; ++i) {
            const int s = i % L.xs;
            // the warp's rows of the tile after next into L2 (its loads are then L2 hits), one
            // 128-byte line per lane and step
            if (i + 2 < n_mine) {
                const int row0 = tile_row(i + 2, 0) - h;
                const int lines = (FW::kLnRows * K * 2) / 128;
                for (int ln_i = lane; ln_i < lines; ln_i += 32) {
                    if (row0 + (ln_i * 64) / K < M) {
                        asm volatile("prefetch.global.L2 [%0];" ::"l"(
                            ln.z + static_cast<int64_t>(row0) * K + 64 * ln_i));
                    }
                }
            }
            // two passes in quarters of 4 row pairs (registers): mean, then the centred sum of
            // squares; each sum is 4 packed adds per lane, then 4 shuffle steps over 16 lanes
#pragma unroll
            for (int half = 0; half < kPairs / 4; ++half) {
                float mean[4], rstd[4];
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    const uint4 v = zr[4 * half + jj];
                    const float2 a = fadd2(E::to_float2(v.x), E::to_float2(v.y));
                    const float2 b = fadd2(E::to_float2(v.z), E::to_float2(v.w));
                    const float2 c = fadd2(a, b);
                    mean[jj] = c.x + c.y;
                }
#pragma unroll
                for (int o = 1; o < 16; o <<= 1) {
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) {
                        mean[jj] += __shfl_xor_sync(0xffffffffu, mean[jj], o);
                    }
                }
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    mean[jj] *= inv_k;
                    const uint4 v = zr[4 * half + jj];
                    const float2 nm = make_float2(-mean[jj], -mean[jj]);
                    const float2 d0 = fadd2(E::to_float2(v.x), nm);
                    const float2 d1 = fadd2(E::to_float2(v.y), nm);
                    const float2 d2 = fadd2(E::to_float2(v.z), nm);
                    const float2 d3 = fadd2(E::to_float2(v.w), nm);
                    float2 q = ffma2(d0, d0, fmul2(d1, d1));
                    q = ffma2(d2, d2, ffma2(d3, d3, q));
                    rstd[jj] = col_ok ? q.x + q.y : 0.f; // padding columns are not elements
                }
#pragma unroll
                for (int o = 1; o < 16; o <<= 1) {
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) {
                        rstd[jj] += __shfl_xor_sync(0xffffffffu, rstd[jj], o);
                    }
                }
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    const int j = 4 * half + jj;
                    rstd[jj] = rsqrtf(rstd[jj] * inv_k + ln.eps);
                    // y = (x - mean) rstd gamma + beta = t gamma + beta, t = x rstd - mean rstd
                    const float2 r2 = make_float2(rstd[jj], rstd[jj]);
                    const float2 mr2 = make_float2(-mean[jj] * rstd[jj], -mean[jj] * rstd[jj]);
                    const uint32_t w4[4] = {zr[j].x, zr[j].y, zr[j].z, zr[j].w};
                    uint32_t o4[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 t = ffma2(E::to_float2(w4[e]), r2, mr2);
                        const float2 yv = ffma2(t, gam[e], bet[e]);
                        o4[e] = E::pack(yv.x, yv.y);
                    }
                    zr[j] = make_uint4(o4[0], o4[1], o4[2], o4[3]);
                    const int row = tile_row(i, j);
                    if (cl == 0 && row < M) {
                        if (ln.mean) {
                            ln.mean[row] = mean[jj];
                        }
                        if (ln.rstd) {
                            ln.rstd[row] = rstd[jj];
                        }
                    }
                }
            }
            // the MMAs of the tile that used this stage last are done
            if (i >= L.xs && !mbar_wait(&x_empty[s], ((i / L.xs) - 1) & 1, abort_flag)) {
                goto done;
            }
            if (col_ok) {
                const uint32_t xs0 = sbase + L.off_x + s * L.x_stage;
#pragma unroll
                for (int j = 0; j < kPairs; ++j) {
                    // row r, 16-byte chunk cl: panel cl / 8, chunk cl % 8 (128-byte swizzle)
                    const int r = FW::kLnRows * lw + 2 * j + h;
                    attn::sts128(xs0 + r * 128 + (cl >> 3) * 16384 + (((cl & 7) ^ (r & 7)) << 4),
                                 zr[j]);
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&x_ready[s]);
            }
            if (i + 1 < n_mine) {
                load_tile(i + 1); // in flight while the MMAs of this tile run
            }
        }
    } else {
        // epilogue: thread (w, r) owns row r and columns [kCols w, +kCols) of each chunk; the
        // warpgroup stages its [128 x kCols] box (2 kCols-byte swizzle) in shared memory and
        // one thread writes it with a TMA store (rows >= M and columns >= N are clipped by the
        // map)
        constexpr int kCols = FW::kCols;
        constexpr int kRowB = 2 * kCols;                 // bytes per staged row
        constexpr int kSwz = kRowB / 16 - 1;             // 16-byte chunks per row - 1
        const int w = warp >> 2;
        const int r = static_cast<int>(attn::warp_lane_base()) + lane;
        const uint32_t lane_off = attn::warp_lane_base() << 16;
        const uint32_t stg_row = sbase + L.off_stg + w * 128 * kRowB + r * kRowB;
        const int swz = ((r * kRowB) >> 7) & kSwz;
        const bool leader = (threadIdx.x == 128 * w);
        uint32_t chunk_ctr = 0;
        for (int i = 0; i < n_mine; ++i) {
            const int mt = blockIdx.x + i * gridDim.x;
            const int row = mt * 128 + r;
            const bool row_ok = row < M;
            const float hm = (kGate && row_ok) ? 0.5f * E::to_float(mask[row]) : 0.f;
            for (int c = 0; c < n_chunks; ++c, ++chunk_ctr) {
                const int bf = chunk_ctr & 1;
                const bool ok = mbar_wait(&acc_full[bf], (chunk_ctr >> 1) & 1, abort_flag);
                if (leader) {
                    bulk_wait_read<0>(); // the previous store has read the staging box
                }
                // every thread arrives, also after a failed wait, and all take one decision
                if (!named_bar_and(1 + w, 128, ok && !*abort_flag)) {
                    goto done;
                }
                __syncwarp();
                tc_fence_after();
                const uint32_t accp = tmem + lane_off + bf * 256 + kCols * w;
                const uint32_t accg = accp + 128;
#pragma unroll
                for (int q = 0; q < kCols / 16; ++q) {
                    uint32_t pv[16], gv[16];
                    tmem_ld16(accp + 16 * q, pv);
                    if constexpr (kGate) {
                        tmem_ld16(accg + 16 * q, gv);
                    }
                    tmem_ld_wait();
                    uint32_t o[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        float y[2];
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const float p = __uint_as_float(pv[2 * e + h]);
                            if constexpr (kGate) {
                                const float g = __uint_as_float(gv[2 * e + h]);
                                float t;
                                asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * g));
                                y[h] = p * fmaf(hm, t, hm); // mask * p * (0.5 tanh(g/2) + 0.5)
                            } else {
                                y[h] = p;
                            }
                        }
                        o[e] = E::pack(y[0], y[1]);
                    }
                    // columns 16q..16q+15 of the box row = 16-byte chunks 2q, 2q+1
                    attn::sts128(stg_row + (((2 * q) ^ swz) << 4),
                                 make_uint4(o[0], o[1], o[2], o[3]));
                    attn::sts128(stg_row + (((2 * q + 1) ^ swz) << 4),
                                 make_uint4(o[4], o[5], o[6], o[7]));
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&acc_empty[bf]);
                }
                fence_proxy_async_smem();
                named_bar_sync(1 + w, 128);
                if (leader) {
                    const int col = c * 128 + kCols * w;
                    // (columns past N, in the last chunk's padding, are clipped by tm_out)
                    if (kGate || n_split >= N || col < n_split) {
                        tma_store_3d(&tm_out, sbase + L.off_stg + w * 128 * kRowB, col, mt * 128,
                                     0);
                    } else {
                        tma_store_3d(&tm_out2, sbase + L.off_stg + w * 128 * kRowB,
                                     col - n_split, mt * 128, 0);
                    }
                    bulk_commit();
                }
            }
        }
        if (leader) {
            bulk_wait<0>(); // stores complete before the CTA retires
        }
    }
done:
    __syncwarp();
    if (warp < 4 * FW::kEpiWg && (threadIdx.x & 127) == 0) {
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
    if (warp == kMmaWarp) {
        tmem_dealloc(tmem, 512);
    }
}

// ------------------------------------------------------------------------------------------
// CUDA-core kernels for shapes outside the tcgen05 paths.  16 x 16 output tiles, K in steps
// of 16 through shared memory, f32 accumulation.
// ------------------------------------------------------------------------------------------
template <typename T>
__global__ void gdp_fwd_generic_kernel(const uint16_t* __restrict__ x,
                                       const uint16_t* __restrict__ wp,
                                       const uint16_t* __restrict__ bp,
                                       const uint16_t* __restrict__ wg,
                                       const uint16_t* __restrict__ bg,
                                       const uint16_t* __restrict__ mask,
                                       uint16_t* __restrict__ out, int M, int K, int N) {
    using E = Elem<T>;
    __shared__ float xs[16][17], ps[16][17], gs[16][17];
    const int tx = threadIdx.x, ty = threadIdx.y;
    const int m = blockIdx.y * 16 + ty, n = blockIdx.x * 16 + tx;
    float ap = 0.f, ag = 0.f;
    for (int k0 = 0; k0 < K; k0 += 16) {
        const int mx = blockIdx.y * 16 + ty, kx = k0 + tx;
        xs[ty][tx] = (mx < M && kx < K) ? E::to_float(x[static_cast<int64_t>(mx) * K + kx]) : 0.f;
        const int kw = k0 + ty;
        ps[ty][tx] = (kw < K && n < N) ? E::to_float(wp[static_cast<int64_t>(kw) * N + n]) : 0.f;
        gs[ty][tx] = (kw < K && n < N) ? E::to_float(wg[static_cast<int64_t>(kw) * N + n]) : 0.f;
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
            ap = fmaf(xs[ty][kk], ps[kk][tx], ap);
            ag = fmaf(xs[ty][kk], gs[kk][tx], ag);
        }
        __syncthreads();
    }
    if (m < M && n < N) {
        const float p = ap + E::to_float(bp[n]);
        const float g = ag + E::to_float(bg[n]);
        out[static_cast<int64_t>(m) * N + n] = E::from_float(E::to_float(mask[m]) * p * sigmoid_accurate(g));
    }
}

bool fwd_fast_shape(int K, int N, bool gate = true) {
    const FwdLayout L = fwd_layout(K, N, gate);
    return (K % 16 == 0) && K >= 16 && K <= kMaxK &&
           (gate ? 2 : 1) * L.kb * L.npad * 2 <= kWeightBudget && L.total <= 227 * 1024;
}

// ln != nullptr: x is LayerNorm(ln->z) and only the fused tcgen05 kernel may be used (the
// caller takes the two-kernel route for other shapes).
template <typename T>
int gdp_fwd_impl(cudaStream_t st, const DeviceInfo& dev, const void* x, const void* wp,
                 const void* bp, const void* wg, const void* bg, const void* mask, void* out,
                 int M, int K, int N, const LnIn* ln = nullptr) {
    const FwdLayout L = fwd_layout(K, N);
    const bool fast = fwd_fast_shape(K, N) && aligned16(ln ? ln->z : x) && aligned16(wp) &&
                      aligned16(wg) && aligned16(out);
    if (ln && !fast) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "gdp_fwd: fused LayerNorm needs the tcgen05 shape");
    }
    if (!fast) {
        dim3 block(16, 16), grid((N + 15) / 16, (M + 15) / 16);
        gdp_fwd_generic_kernel<T><<<grid, block, 0, st>>>(
            static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(wp),
            static_cast<const uint16_t*>(bp), static_cast<const uint16_t*>(wg),
            static_cast<const uint16_t*>(bg), static_cast<const uint16_t*>(mask),
            static_cast<uint16_t*>(out), M, K, N);
        return check_launch("gdp_fwd_generic");
    }
    CUtensorMap tx, twp, twg, tout;
    // x [M, K]: dims (K, M, 1), box 64 x 128; weights [K, N]: dims (N, K, 1), box 64 x K;
    // out [M, N]: dims (N, M, 1), box 32 x 128 (stores)
    CFK_TRY(make_tmap_3d(&tx, ln ? ln->z : x, K, M, 1, 2ull * K, 2ull * K * M, 64, 128, 1, 128,
                         "gdp x"));
    CFK_TRY(make_tmap_3d(&twp, wp, N, K, 1, 2ull * N, 2ull * N * K, 64, K, 1, 128, "gdp wp"));
    CFK_TRY(make_tmap_3d(&twg, wg, N, K, 1, 2ull * N, 2ull * N * K, 64, K, 1, 128, "gdp wg"));
    constexpr int out_cols = FwdWarps<true>::kCols;
    static_assert(FwdWarps<true>::kCols == FwdWarps<false>::kCols, "one store box width");
    CFK_TRY(make_tmap_3d(&tout, out, N, M, 1, 2ull * N, 2ull * N * M, out_cols, 128, 1,
                         2 * out_cols, "gdp out"));
    auto kern = ln ? gdp_fwd_kernel<T, true, true> : gdp_fwd_kernel<T, false, true>;
    CFK_TRY(ensure_smem_attr(reinterpret_cast<const void*>(kern), dev.device, 227 * 1024,
                             ln ? "gdp_fwd_ln" : "gdp_fwd",
                             ln ? FwdWarps<true>::kLaunchRegs : 0));
    const int n_mt = (M + 127) / 128;
    const int grid = std::min(n_mt, dev.num_sms);
    const LnIn none{};
    kern<<<grid, ln ? FwdWarps<true>::kThreads : FwdWarps<false>::kThreads, L.total, st>>>(
        tx, twp, twg, tout, tout, N, static_cast<const uint16_t*>(bp),
        static_cast<const uint16_t*>(bg), static_cast<const uint16_t*>(mask), M, K, N,
        ln ? *ln : none);
    return check_launch(ln ? "gdp_fwd_ln" : "gdp_fwd");
}

// y = x w + b on CUDA cores (shapes or alignments the tcgen05 kernel does not take); columns
// [0, n_split) to y0 (row stride ld0), [n_split, N) to y1 (row stride ld1).
template <typename T>
__global__ void linear_fwd_generic_kernel(const uint16_t* __restrict__ x,
                                          const uint16_t* __restrict__ w,
                                          const uint16_t* __restrict__ b, uint16_t* y0,
                                          int64_t ld0, uint16_t* y1, int64_t ld1, int n_split,
                                          int M, int K, int N) {
    using E = Elem<T>;
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    const int m = blockIdx.y * blockDim.y + threadIdx.y;
    if (m >= M || n >= N) {
        return;
    }
    float a = b ? E::to_float(b[n]) : 0.f;
    for (int k = 0; k < K; ++k) {
        a = fmaf(E::to_float(x[static_cast<int64_t>(m) * K + k]),
                 E::to_float(w[static_cast<int64_t>(k) * N + n]), a);
    }
    if (n < n_split) {
        y0[m * ld0 + n] = E::from_float(a);
    } else {
        y1[m * ld1 + (n - n_split)] = E::from_float(a);
    }
}

// The plain projection: y = x w + b (b may be null), columns [0, n_split) into y0 with row
// stride ld0 elements and [n_split, N) into y1 with row stride ld1.
template <typename T>
int linear_fwd_impl(cudaStream_t st, const DeviceInfo& dev, const void* x, const void* w,
                    const void* b, void* y0, int64_t ld0, void* y1, int64_t ld1, int n_split,
                    int M, int K, int N) {
    const FwdLayout L = fwd_layout(K, N, false);
    const bool fast = fwd_fast_shape(K, N, false) && (n_split == N || n_split % 128 == 0) &&
                      aligned16(x) &&
                      aligned16(w) && aligned16(y0) && ld0 % 8 == 0 &&
                      (n_split == N || (aligned16(y1) && ld1 % 8 == 0));
    if (!fast) {
        dim3 block(16, 16), grid((N + 15) / 16, (M + 15) / 16);
        linear_fwd_generic_kernel<T><<<grid, block, 0, st>>>(
            static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(w),
            static_cast<const uint16_t*>(b), static_cast<uint16_t*>(y0), ld0,
            static_cast<uint16_t*>(y1), ld1, n_split, M, K, N);
        return check_launch("linear_fwd_generic");
    }
    CUtensorMap tx, tw, ty0, ty1;
    constexpr int out_cols = FwdWarps<false>::kCols;
    CFK_TRY(make_tmap_3d(&tx, x, K, M, 1, 2ull * K, 2ull * K * M, 64, 128, 1, 128, "linear x"));
    CFK_TRY(make_tmap_3d(&tw, w, N, K, 1, 2ull * N, 2ull * N * K, 64, K, 1, 128, "linear w"));
    CFK_TRY(make_tmap_3d(&ty0, y0, n_split, M, 1, 2ull * ld0, 2ull * ld0 * M, out_cols, 128, 1,
                         2 * out_cols, "linear y0"));
    if (n_split < N) {
        CFK_TRY(make_tmap_3d(&ty1, y1, N - n_split, M, 1, 2ull * ld1, 2ull * ld1 * M, out_cols,
                             128, 1, 2 * out_cols, "linear y1"));
    } else {
        ty1 = ty0;
    }
    auto kern = gdp_fwd_kernel<T, false, false>;
    CFK_TRY(ensure_smem_attr(reinterpret_cast<const void*>(kern), dev.device, 227 * 1024,
                             "linear_fwd"));
    const int n_mt = (M + 127) / 128;
    const int grid = std::min(n_mt, dev.num_sms);
    const LnIn none{};
    kern<<<grid, FwdWarps<false>::kThreads, L.total, st>>>(
        tx, tw, tw, ty0, ty1, n_split, static_cast<const uint16_t*>(b), nullptr, nullptr, M, K,
        N, none);
    return check_launch("linear_fwd");
}

// ==========================================================================================
// Backward
// ==========================================================================================
// dp = dout * mask * s and dg = dout * mask * p * s * (1 - s), s = sigmoid(g), in f32.
__device__ __forceinline__ void gate_grads(float p, float g, float dout, float m, float& dp,
                                           float& dg) {
    const float s = sigmoid_accurate(g);
    const float dm = dout * m;
    dp = dm * s;
    dg = dm * p * s * (1.f - s);
}

// gate_grads for two adjacent columns of a row, in f32x2 arithmetic (dg = dp * p * (1 - s)).
__device__ __forceinline__ void gate_grads2(float2 p, float2 g, float2 dout, float m, float2& dp,
                                            float2& dg) {
    const float2 t = fmul2(g, make_float2(-kLog2e, -kLog2e));
    const float2 e = fadd2(make_float2(ex2(t.x), ex2(t.y)), make_float2(1.f, 1.f));
    const float2 sg = make_float2(rcp_approx(e.x), rcp_approx(e.y));
    dp = fmul2(fmul2(dout, make_float2(m, m)), sg);
    const float2 oms = ffma2(sg, make_float2(-1.f, -1.f), make_float2(1.f, 1.f));
    dg = fmul2(fmul2(dp, p), oms);
}

// gate_grads2 with the sigmoid from one tanh.approx (0.5 tanh(g/2) + 0.5: one MUFU operation
// instead of an exponential and a reciprocal), for results that are rounded to 16 bits next
// (the dx pass's dp, dg operands); the weight gradients keep gate_grads2.
__device__ __forceinline__ void gate_grads2_fast(float2 p, float2 g, float2 dout, float m,
                                                 float2& dp, float2& dg) {
    const float2 sg = make_float2(sigmoid_fast(g.x), sigmoid_fast(g.y));
    dp = fmul2(fmul2(dout, make_float2(m, m)), sg);
    const float2 oms = ffma2(sg, make_float2(-1.f, -1.f), make_float2(1.f, 1.f));
    dg = fmul2(fmul2(dp, p), oms);
}

// bias-row operand of one 128- or 64-column chunk, built in shared memory by one warp:
// MN-major interleave [16 x cols], row 0 = bias[n0 + n] (0 beyond N), rows 1..15 = 0.
__device__ __forceinline__ void build_brow(uint16_t* dst, const uint16_t* bias, int n0, int cols,
                                           int N, int lane) {
    for (int i = lane; i < cols * 16; i += 32) {
        const int chunk = i / 128, within = i % 128, kk = within / 8, e = within % 8;
        const int n = n0 + chunk * 8 + e;
        dst[i] = (kk == 0 && n < N) ? bias[n] : uint16_t(0);
    }
}

// ------------------------------------------------------------------------------------------
// dx = dp wp^T + dg wg^T, per 128-row tile of x; p and g recomputed per 128-column chunk.
// ------------------------------------------------------------------------------------------
struct DxLayout {
    int x, wp, wg, dout, dp, dg, bp, bg, ones, bar, total;
};

__host__ __device__ inline DxLayout dx_layout(int K) {
    DxLayout L;
    const int wchunk = K * 256; // [K rows x 128 n] = 2 atoms of K x 128 B
    L.x = 0;                    // 2 panels (zero-filled beyond K)
    L.wp = 32768;
    L.wg = L.wp + wchunk;
    L.dout = L.wg + wchunk;     // [128 x 128] 2 panels
    L.dp = L.dout + 32768;
    L.dg = L.dp + 32768;
    L.bp = L.dg + 32768;        // [16 x 128] interleave, 4 KB
    L.bg = L.bp + 4096;
    L.ones = L.bg + 4096;
    L.bar = L.ones + 4096;
    L.total = L.bar + 16 * 8 + 16 + 1024;
    return L;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    gdp_bwd_dx_kernel(const __grid_constant__ CUtensorMap tm_x,
                      const __grid_constant__ CUtensorMap tm_wp,
                      const __grid_constant__ CUtensorMap tm_wg,
                      const __grid_constant__ CUtensorMap tm_dout,
                      const uint16_t* __restrict__ bp, const uint16_t* __restrict__ bg,
                      const uint16_t* __restrict__ mask, uint16_t* __restrict__ dx, int M, int K,
                      int N) {
    using E = Elem<T>;
    const DxLayout L = dx_layout(K);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar);
    uint64_t* x_full = bars + 0;
    uint64_t* tile_done = bars + 1;   // all MMAs of a row tile done (x free)
    uint64_t* chunk_full = bars + 2;  // w chunk, dout chunk, bias rows loaded
    uint64_t* rec_full = bars + 3;    // p, g of the chunk in tensor memory
    uint64_t* ds_full = bars + 4;     // dp, dg written (count 8)
    uint64_t* dx_done = bars + 5;     // dx MMAs of the chunk done (chunk buffers free)
    uint64_t* dx_full = bars + 6;     // dx of the tile complete
    uint64_t* dx_drained = bars + 7;  // dx read out of tensor memory (count 8)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.bar + 16 * 8);
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n_mt = (M + 127) / 128;
    const int n_chunks = (N + 127) / 128;
    const int n_mine = (n_mt - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                       static_cast<int>(gridDim.x);

    if (threadIdx.x == 0) {
        mbar_init(x_full, 1);
        mbar_init(tile_done, 1);
        mbar_init(chunk_full, 1);
        mbar_init(rec_full, 1);
        mbar_init(ds_full, 8);
        mbar_init(dx_done, 1);
        mbar_init(dx_full, 1);
        mbar_init(dx_drained, 8);
        *abort_flag = 0;
        fence_mbar_init();
    }
    {
        const uint32_t one = E::kBf16 ? 0x3F80u : 0x3C00u;
        uint32_t* ones = reinterpret_cast<uint32_t*>(smem + L.ones);
        for (int i = threadIdx.x; i < 1024; i += blockDim.x) {
            ones[i] = ((i < 512) && ((i & 3) == 0)) ? one : 0u;
        }
        if (K <= 64) { // the second x panel stays zero
            uint32_t* z = reinterpret_cast<uint32_t*>(smem + L.x + 16384);
            for (int i = threadIdx.x; i < 4096; i += blockDim.x) {
                z[i] = 0u;
            }
        }
        fence_proxy_async_smem();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, 512);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // tensor memory: p at 0, g at 128, dx at 256 (K columns)

    if (warp == kProducerWarp) {
        uint32_t cc = 0; // chunk counter
        for (int i = 0; i < n_mine; ++i) {
            const int mt = blockIdx.x + i * gridDim.x;
            if (i > 0 && !mbar_wait(tile_done, (i - 1) & 1, abort_flag)) {
                goto done;
            }
            if (lane == 0) {
                const int panels = (K + 63) / 64;
                mbar_arrive_expect_tx(x_full, panels * 16384);
                for (int pn = 0; pn < panels; ++pn) {
                    tma_load_3d(smem + L.x + pn * 16384, &tm_x, x_full, pn * 64, mt * 128, 0);
                }
            }
            for (int c = 0; c < n_chunks; ++c, ++cc) {
                if (cc > 0 && !mbar_wait(dx_done, (cc - 1) & 1, abort_flag)) {
                    goto done;
                }
                build_brow(reinterpret_cast<uint16_t*>(smem + L.bp), bp, c * 128, 128, N, lane);
                build_brow(reinterpret_cast<uint16_t*>(smem + L.bg), bg, c * 128, 128, N, lane);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive_expect_tx(chunk_full, 2 * 2 * K * 128 + 32768);
                    for (int a = 0; a < 2; ++a) {
                        tma_load_3d(smem + L.wp + a * K * 128, &tm_wp, chunk_full,
                                    c * 128 + a * 64, 0, 0);
                        tma_load_3d(smem + L.wg + a * K * 128, &tm_wg, chunk_full,
                                    c * 128 + a * 64, 0, 0);
                        tma_load_3d(smem + L.dout + a * 16384, &tm_dout, chunk_full,
                                    c * 128 + a * 64, mt * 128, 0);
                    }
                }
                __syncwarp();
            }
        }
    } else if (warp == kMmaWarp) {
        // whole warp, converged: MMAs and commits are elect.sync-issued
        {
            constexpr uint32_t kIdRec = idesc_f16(128, 128, false, true, E::kBf16);
            const uint32_t kIdDx = idesc_f16(128, K, false, false, E::kBf16);
            const uint64_t ones = attn::interleave16_kmajor(sbase + L.ones);
            const int ksteps = K / 16;
            uint32_t cc = 0;
            for (int i = 0; i < n_mine; ++i) {
                if (!mbar_wait_w(x_full, i & 1, abort_flag)) {
                    goto done;
                }
                for (int c = 0; c < n_chunks; ++c, ++cc) {
                    if (!mbar_wait_w(chunk_full, cc & 1, abort_flag)) {
                        goto done;
                    }
                    tc_fence_after();
                    for (int ks = 0; ks < ksteps; ++ks) {
                        umma_ss_w(tmem, x_desc(sbase + L.x, ks), w_desc(sbase + L.wp, K, 0, ks),
                                kIdRec, ks > 0);
                    }
                    umma_ss_w(tmem, ones, brow_desc(sbase + L.bp, 0), kIdRec, 1);
                    for (int ks = 0; ks < ksteps; ++ks) {
                        umma_ss_w(tmem + 128, x_desc(sbase + L.x, ks),
                                w_desc(sbase + L.wg, K, 0, ks), kIdRec, ks > 0);
                    }
                    umma_ss_w(tmem + 128, ones, brow_desc(sbase + L.bg, 0), kIdRec, 1);
                    umma_commit_w(rec_full);
                    if (!mbar_wait_w(ds_full, cc & 1, abort_flag)) {
                        goto done;
                    }
                    if (c == 0 && i > 0 && !mbar_wait_w(dx_drained, (i - 1) & 1, abort_flag)) {
                        goto done;
                    }
                    tc_fence_after();
                    // dx[m, k] += sum_n dp[m, n] wp[k, n]: A = dp K-major, B = w chunk K-major
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks) {
                        const uint32_t boff = (ks >> 2) * (K * 128) + (ks & 3) * 32;
                        umma_ss_w(tmem + 256, x_desc(sbase + L.dp, ks),
                                smem_desc(sbase + L.wp + boff, 16, 1024, kSwizzle128), kIdDx,
                                (c > 0 || ks > 0) ? 1u : 0u);
                        umma_ss_w(tmem + 256, x_desc(sbase + L.dg, ks),
                                smem_desc(sbase + L.wg + boff, 16, 1024, kSwizzle128), kIdDx, 1);
                    }
                    umma_commit_w(dx_done);
                }
                umma_commit_w(tile_done);
                umma_commit_w(dx_full);
            }
        }
    } else {
        const int w = warp >> 2;
        const int r = static_cast<int>(attn::warp_lane_base()) + lane;
        const uint32_t lane_off = attn::warp_lane_base() << 16;
        const uint32_t dp_row = sbase + L.dp + w * 16384 + r * 128;
        const uint32_t dg_row = sbase + L.dg + w * 16384 + r * 128;
        const uint32_t do_row = sbase + L.dout + w * 16384 + r * 128;
        uint32_t cc = 0;
        for (int i = 0; i < n_mine; ++i) {
            const int mt = blockIdx.x + i * gridDim.x;
            const int row = mt * 128 + r;
            const bool row_ok = row < M;
            const float mk = row_ok ? E::to_float(mask[row]) : 0.f;
            for (int c = 0; c < n_chunks; ++c, ++cc) {
                if (!mbar_wait(rec_full, cc & 1, abort_flag) ||
                    !mbar_wait(chunk_full, cc & 1, abort_flag)) {
                    goto done;
                }
                // dp / dg shared buffers are free once the previous chunk's dx MMAs are done
                if (cc > 0 && !mbar_wait(dx_done, (cc - 1) & 1, abort_flag)) {
                    goto done;
                }
                __syncwarp();
                tc_fence_after();
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    uint32_t pv[16], gv[16];
                    tmem_ld16(tmem + lane_off + 64 * w + 16 * q, pv);
                    tmem_ld16(tmem + lane_off + 128 + 64 * w + 16 * q, gv);
                    tmem_ld_wait();
                    uint32_t op[8], og[8];
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint4 dw = attn::lds128(do_row + (((2 * q + h) ^ (r & 7)) << 4));
                        const uint32_t dww[4] = {dw.x, dw.y, dw.z, dw.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 d2 = E::to_float2(dww[e]);
                            float dp0, dg0, dp1, dg1;
                            gate_grads(__uint_as_float(pv[8 * h + 2 * e]),
                                       __uint_as_float(gv[8 * h + 2 * e]), d2.x, mk, dp0, dg0);
                            gate_grads(__uint_as_float(pv[8 * h + 2 * e + 1]),
                                       __uint_as_float(gv[8 * h + 2 * e + 1]), d2.y, mk, dp1, dg1);
                            op[4 * h + e] = E::pack(dp0, dp1);
                            og[4 * h + e] = E::pack(dg0, dg1);
                        }
                    }
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t off = ((2 * q + h) ^ (r & 7)) << 4;
                        attn::sts128(dp_row + off, make_uint4(op[4 * h], op[4 * h + 1], op[4 * h + 2], op[4 * h + 3]));
                        attn::sts128(dg_row + off, make_uint4(og[4 * h], og[4 * h + 1], og[4 * h + 2], og[4 * h + 3]));
                    }
                }
                tc_fence_before();
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(ds_full);
                }
            }
            // dx of the tile: thread (w, r) stores columns [w*K/2, (w+1)*K/2)
            if (!mbar_wait(dx_full, i & 1, abort_flag)) {
                goto done;
            }
            __syncwarp();
            tc_fence_after();
            const int half = K / 2;
            for (int q = 0; q < half; q += 8) {
                uint32_t v[8];
                tmem_ld8(tmem + lane_off + 256 + w * half + q, v);
                tmem_ld_wait();
                if (row_ok) {
                    uint4 o = make_uint4(E::pack(__uint_as_float(v[0]), __uint_as_float(v[1])),
                                         E::pack(__uint_as_float(v[2]), __uint_as_float(v[3])),
                                         E::pack(__uint_as_float(v[4]), __uint_as_float(v[5])),
                                         E::pack(__uint_as_float(v[6]), __uint_as_float(v[7])));
                    st_global_v4(dx + static_cast<int64_t>(row) * K + w * half + q, o);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(dx_drained);
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
    if (warp == kMmaWarp) {
        tmem_dealloc(tmem, 512);
    }
}

// ------------------------------------------------------------------------------------------
// dx with both weight matrices resident in shared memory (the shapes whose weights fit beside
// two x stages).  Per 128-row tile of x and per 64-column chunk j:
//   [p | g] = x [wp_j | wg_j] + [bp_j | bg_j]   one N = 128 MMA chain: the 64-column atoms
//                                               j of wp and of wg form the B operand
//   dp, dg  -> the same tensor-memory columns, as packed 16-bit pairs (tcgen05.st)
//   dx     += dp wp_j^T + dg wg_j^T             A read from tensor memory (TS form)
// The epilogue reads dout straight from global memory (one chunk ahead in registers, the next
// tile's lines prefetched into L2), which leaves the shared memory to the weights and x.
// Tensor memory: [p | g] buffers at 0 and 128 (chunk counter & 1), dx buffers at 256 and 384
// (tile counter & 1).  The chunk buffer of chunk c is rewritten by the recompute of chunk
// c + 2, which the MMA warp issues after the dx MMAs of chunk c (tcgen05.mma runs in issue
// order, so the dx MMAs read dp / dg before the recompute overwrites them).
// ------------------------------------------------------------------------------------------
struct DxrLayout {
    int nch;    // 64-column chunks of N
    int xpan;   // 64-column panels of an x tile
    int xs;     // x stages
    int w, brow, ones, x, bar, total;
};

__host__ __device__ inline DxrLayout dxr_layout(int K, int N) {
    DxrLayout L;
    L.nch = (N + 63) / 64;
    L.xpan = (K + 63) / 64;
    L.w = 0;                                   // wp atoms, then wg atoms: K x 128 B each
    L.brow = L.w + 2 * L.nch * K * 128;        // per chunk [16 x 128] interleave: bp_j | bg_j
    L.ones = L.brow + L.nch * 4096;
    L.x = L.ones + 4096;
    for (L.xs = 2; L.xs >= 1; --L.xs) {
        L.bar = L.x + L.xs * L.xpan * 16384;
        L.total = L.bar + 16 * 8 + 16 + 1024;
        if (L.total <= 227 * 1024) {
            break;
        }
    }
    return L;
}

constexpr int kDxrThreads = 320; // 8 epilogue warps (2 per lane quarter), producer, MMA
constexpr int kDxrProducer = 8;
constexpr int kDxrMma = 9;
constexpr int kDxrCols = 32;     // columns of a 64-column chunk per epilogue warp

template <typename T>
__global__ void __launch_bounds__(kDxrThreads, 1)
    gdp_bwd_dxr_kernel(const __grid_constant__ CUtensorMap tm_x,
                       const __grid_constant__ CUtensorMap tm_wp,
                       const __grid_constant__ CUtensorMap tm_wg,
                       const uint16_t* __restrict__ bp, const uint16_t* __restrict__ bg,
                       const uint16_t* __restrict__ mask, const uint16_t* __restrict__ dout,
                       uint16_t* __restrict__ dx, int M, int K, int N) {
    using E = Elem<T>;
    const DxrLayout L = dxr_layout(K, N);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar);
    uint64_t* w_full = bars + 0;     // weights loaded
    uint64_t* x_full = bars + 1;     // [2]
    uint64_t* x_empty = bars + 3;    // [2] recompute MMAs of the tile done
    uint64_t* pg_full = bars + 5;    // [2] p, g of a chunk in tensor memory
    uint64_t* ds_full = bars + 7;    // [2] dp, dg of a chunk in tensor memory (count 8)
    uint64_t* dx_full = bars + 9;    // [2] dx of a tile complete
    uint64_t* dx_empty = bars + 11;  // [2] dx of a tile read out (count 8)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.bar + 16 * 8);
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n_mt = (M + 127) / 128;
    const int nch = L.nch;
    const int n_mine = (n_mt - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                       static_cast<int>(gridDim.x);

    if (threadIdx.x == 0) {
        mbar_init(w_full, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&x_full[s], 1);
            mbar_init(&x_empty[s], 1);
            mbar_init(&pg_full[s], 1);
            mbar_init(&ds_full[s], 8);
            mbar_init(&dx_full[s], 1);
            mbar_init(&dx_empty[s], 8);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    {
        const uint32_t one = E::kBf16 ? 0x3F80u : 0x3C00u;
        uint32_t* ones = reinterpret_cast<uint32_t*>(smem + L.ones);
        for (int i = threadIdx.x; i < 1024; i += blockDim.x) {
            ones[i] = ((i < 512) && ((i & 3) == 0)) ? one : 0u;
        }
        // bias rows: chunk j holds bp[64j, 64j + 64) in columns 0..63, bg in 64..127
        for (int j = warp; j < nch; j += kDxrThreads / 32) {
            uint16_t* b = reinterpret_cast<uint16_t*>(smem + L.brow + j * 4096);
            build_brow(b, bp, 64 * j, 64, N, lane);
            build_brow(b + 1024, bg, 64 * j, 64, N, lane);
        }
        fence_proxy_async_smem();
    }
    if (warp == kDxrMma) {
        tmem_alloc(tmem_slot, 512);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == kDxrProducer) {
        if (lane == 0) {
            mbar_arrive_expect_tx(w_full, 2 * nch * K * 128);
            for (int j = 0; j < nch; ++j) {
                tma_load_3d(smem + L.w + j * K * 128, &tm_wp, w_full, 64 * j, 0, 0);
                tma_load_3d(smem + L.w + (nch + j) * K * 128, &tm_wg, w_full, 64 * j, 0, 0);
            }
            for (int t = 0; t < n_mine; ++t) {
                const int s = t % L.xs;
                if (t >= L.xs && !mbar_wait(&x_empty[s], (t / L.xs - 1) & 1, abort_flag)) {
                    break;
                }
                const int mt = blockIdx.x + t * gridDim.x;
                mbar_arrive_expect_tx(&x_full[s], L.xpan * 16384);
                for (int pn = 0; pn < L.xpan; ++pn) {
                    tma_load_3d(smem + L.x + (s * L.xpan + pn) * 16384, &tm_x, &x_full[s],
                                pn * 64, mt * 128, 0);
                }
            }
        }
        __syncwarp();
    } else if (warp == kDxrMma) {
        // whole warp, converged: MMAs and commits are elect.sync-issued
        const uint32_t kIdRec = idesc_f16(128, 128, false, true, E::kBf16);
        const uint32_t kIdDx = idesc_f16(128, K, false, false, E::kBf16);
        const uint64_t ones = attn::interleave16_kmajor(sbase + L.ones);
        const int ksteps = K / 16;
        const uint32_t pair_lbo = static_cast<uint32_t>(nch * K * 128); // wp_j -> wg_j
        // dx MMAs of chunk h (tile h / nch, chunk h % nch)
        auto issue_dx = [&](int h) -> bool {
            const int th = h / nch, jh = h - th * nch;
            if (!mbar_wait_w(&ds_full[h & 1], (h >> 1) & 1, abort_flag)) {
                return false;
            }
            if (jh == 0 && th >= 2 &&
                !mbar_wait_w(&dx_empty[th & 1], ((th >> 1) + 1) & 1, abort_flag)) {
                return false;
            }
            tc_fence_after();
            const uint32_t pg = tmem + (h & 1) * 128;
            const uint32_t d = tmem + 256 + (th & 1) * 128;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                // dp of columns [16 ks, 16 ks + 16) sits in the columns of epilogue warp
                // 16 ks / kDxrCols, packed: dp in its first half, dg in its second
                const uint32_t a = pg + kDxrCols * ((16 * ks) / kDxrCols) + ((16 * ks) % kDxrCols) / 2;
                const uint32_t boff = jh * K * 128 + ks * 32;
                umma_ts_w(d, a, smem_desc(sbase + L.w + boff, 16, 1024, kSwizzle128), kIdDx,
                          (jh > 0 || ks > 0) ? 1u : 0u);
                umma_ts_w(d, a + kDxrCols / 2,
                          smem_desc(sbase + L.w + nch * K * 128 + boff, 16, 1024, kSwizzle128),
                          kIdDx, 1u);
            }
            if (jh == nch - 1) {
                umma_commit_w(&dx_full[th & 1]);
            }
            return true;
        };
        if (!mbar_wait_w(w_full, 0, abort_flag)) {
            goto done;
        }
        int g = 0;
        for (int t = 0; t < n_mine; ++t) {
            const int s = t % L.xs;
            if (!mbar_wait_w(&x_full[s], (t / L.xs) & 1, abort_flag)) {
                goto done;
            }
            tc_fence_after();
            const uint32_t xb = sbase + L.x + s * L.xpan * 16384;
            for (int j = 0; j < nch; ++j, ++g) {
                const uint32_t pg = tmem + (g & 1) * 128;
                const uint32_t wj = sbase + L.w + j * K * 128;
                for (int ks = 0; ks < ksteps; ++ks) {
                    umma_ss_w(pg, x_desc(xb, ks),
                              smem_desc(wj + ks * 2048, pair_lbo, 1024, kSwizzle128), kIdRec,
                              ks > 0 ? 1u : 0u);
                }
                umma_ss_w(pg, ones, brow_desc(sbase + L.brow + j * 4096, 0), kIdRec, 1u);
                umma_commit_w(&pg_full[g & 1]);
                if (j == nch - 1) {
                    umma_commit_w(&x_empty[s]);
                }
                if (g >= 1 && !issue_dx(g - 1)) {
                    goto done;
                }
            }
        }
        if (g >= 1 && !issue_dx(g - 1)) {
            goto done;
        }
    } else {
        const int sl = warp >> 2; // column slice of the chunk: [32 sl, 32 sl + 32)
        const int r = static_cast<int>(attn::warp_lane_base()) + lane;
        const uint32_t lane_off = attn::warp_lane_base() << 16;
        const int total = n_mine * nch;
        const bool wide = (N % 16 == 0) && (reinterpret_cast<uintptr_t>(dout) & 31) == 0;
        const bool dx32 = (reinterpret_cast<uintptr_t>(dx) & 31) == 0;
        // dout of chunk h for this thread: row of tile h / nch, 32 columns
        // (32-byte loads when the rows allow them: fewer, fully used sectors per instruction)
        auto load_dout = [&](int h, uint32_t (&v)[16]) {
            const int th = h / nch, jh = h - th * nch;
            const int row = (static_cast<int>(blockIdx.x) + th * static_cast<int>(gridDim.x)) * 128 + r;
            const int c0 = 64 * jh + kDxrCols * sl;
            const uint16_t* src = dout + static_cast<int64_t>(row) * N + c0;
            if (wide) {
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    uint32_t (&w8)[8] = *reinterpret_cast<uint32_t (*)[8]>(&v[8 * q]);
                    if (row < M && c0 + 16 * q < N) {
                        ld_global_nc_v8(src + 16 * q, w8);
                    } else {
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            w8[e] = 0u;
                        }
                    }
                }
            } else {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint4 u = (row < M && c0 + 8 * q < N) ? ld_global_nc_v4(src + 8 * q)
                                                                : make_uint4(0u, 0u, 0u, 0u);
                    v[4 * q] = u.x;
                    v[4 * q + 1] = u.y;
                    v[4 * q + 2] = u.z;
                    v[4 * q + 3] = u.w;
                }
            }
        };
        // dx of tile t: this warp stores columns [K/2 sl, K/2 sl + K/2) of row r
        auto drain = [&](int t) -> bool {
            if (!mbar_wait(&dx_full[t & 1], (t >> 1) & 1, abort_flag)) {
                return false;
            }
            __syncwarp();
            tc_fence_after();
            const int row = (static_cast<int>(blockIdx.x) + t * static_cast<int>(gridDim.x)) * 128 + r;
            const int half = K / 2;
            const uint32_t src = tmem + lane_off + 256 + (t & 1) * 128 + sl * half;
            uint16_t* dst = dx + static_cast<int64_t>(row) * K + sl * half;
            if (half % 32 == 0 && dx32) {
                // 32 columns per tensor-memory load, 32-byte stores
                for (int q = 0; q < half; q += 32) {
                    uint32_t v[32];
                    tmem_ld32(src + q, v);
                    tmem_ld_wait();
                    if (row < M) {
#pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            uint32_t o[8];
#pragma unroll
                            for (int e = 0; e < 8; ++e) {
                                o[e] = E::pack(__uint_as_float(v[16 * u + 2 * e]),
                                               __uint_as_float(v[16 * u + 2 * e + 1]));
                            }
                            st_global_v8(dst + q + 16 * u, o);
                        }
                    }
                }
            } else {
                for (int q = 0; q < half; q += 8) {
                    uint32_t v[8];
                    tmem_ld8(src + q, v);
                    tmem_ld_wait();
                    if (row < M) {
                        st_global_v4(dst + q,
                                     make_uint4(E::pack(__uint_as_float(v[0]), __uint_as_float(v[1])),
                                                E::pack(__uint_as_float(v[2]), __uint_as_float(v[3])),
                                                E::pack(__uint_as_float(v[4]), __uint_as_float(v[5])),
                                                E::pack(__uint_as_float(v[6]), __uint_as_float(v[7]))));
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&dx_empty[t & 1]);
            }
            return true;
        };
        // dout of the next two chunks in flight
        uint32_t dn[16], dn2[16];
        if (total > 0) {
            load_dout(0, dn);
        }
        if (total > 1) {
            load_dout(1, dn2);
        }
        float mk = 0.f;
        for (int h = 0; h < total; ++h) {
            const int th = h / nch, jh = h - th * nch;
            if (jh == 0) {
                const int row = (static_cast<int>(blockIdx.x) + th * static_cast<int>(gridDim.x)) * 128 + r;
                mk = row < M ? E::to_float(mask[row]) : 0.f;
                // the next tile's dout lines of this row, into L2
                const int nrow = row + static_cast<int>(gridDim.x) * 128;
                if (th + 1 < n_mine && nrow < M) {
                    for (int c = 64 * sl; c < N; c += 128) {
                        asm volatile("prefetch.global.L2 [%0];" ::"l"(dout + static_cast<int64_t>(nrow) * N + c));
                    }
                }
            }
            uint32_t dc[16];
#pragma unroll
            for (int q = 0; q < 16; ++q) {
                dc[q] = dn[q];
                dn[q] = dn2[q];
            }
            if (h + 2 < total) {
                load_dout(h + 2, dn2);
            }
            if (!mbar_wait(&pg_full[h & 1], (h >> 1) & 1, abort_flag)) {
                goto done;
            }
            __syncwarp();
            tc_fence_after();
            const uint32_t pg = tmem + lane_off + (h & 1) * 128 + kDxrCols * sl;
            uint32_t pv[32], gv[32];
            tmem_ld32(pg, pv);
            tmem_ld32(pg + 64, gv);
            tmem_ld_wait();
            uint32_t op[16], og[16];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t* dw = dc + 4 * q;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int c = 8 * q + 2 * e;
                    float2 dp2, dg2;
                    gate_grads2_fast(
                        make_float2(__uint_as_float(pv[c]), __uint_as_float(pv[c + 1])),
                        make_float2(__uint_as_float(gv[c]), __uint_as_float(gv[c + 1])),
                        E::to_float2(dw[e]), mk, dp2, dg2);
                    op[4 * q + e] = E::pack(dp2.x, dp2.y);
                    og[4 * q + e] = E::pack(dg2.x, dg2.y);
                }
            }
            tmem_st16(pg, op);
            tmem_st16(pg + kDxrCols / 2, og);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&ds_full[h & 1]);
            }
            if (jh == 0 && th >= 1 && !drain(th - 1)) {
                goto done;
            }
        }
        if (n_mine > 0 && !drain(n_mine - 1)) {
            goto done;
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
    if (warp == kDxrMma) {
        tmem_dealloc(tmem, 512);
    }
}

// ------------------------------------------------------------------------------------------
// dwp, dwg, dbp, dbg for one 64-column chunk per CTA (a group of CTAs per chunk, each over a
// strided set of row tiles); per-CTA sums are added into the zeroed f32 outputs at the end.
// ------------------------------------------------------------------------------------------
struct DwLayout {
    int x, dout, hi_p, lo_p, hi_g, lo_g, wp, wg, bp, bg, ones, red, bar, total;
};

__host__ __device__ inline DwLayout dw_layout(int K) {
    DwLayout L;
    L.x = 0;                  // 2 stages x 2 panels x 16 KB
    L.dout = 65536;           // 2 stages x [128 x 64] (one 16 KB panel)
    L.hi_p = L.dout + 32768;  // four [128 x 64] bf16 tiles; hi_p | hi_g and lo_p | lo_g are
    L.hi_g = L.hi_p + 16384;  // the two 64-column atoms of one N = 128 MMA operand
    L.lo_p = L.hi_g + 16384;
    L.lo_g = L.lo_p + 16384;
    L.wp = L.lo_g + 16384;    // [K rows x 64 n] = K x 128 B
    L.wg = L.wp + K * 128;
    L.bp = L.wg + K * 128;    // [16 x 64] interleave, 2 KB
    L.bg = L.bp + 2048;
    L.ones = L.bg + 2048;
    L.red = L.ones + 4096;    // f32 [8 warps][64] bias-gradient partials
    L.bar = L.red + 8 * 64 * 4;
    L.total = L.bar + 16 * 8 + 16 + 1024;
    return L;
}

// Warp roles of the dW kernel: 4*EQ epilogue warps (EQ per tensor-memory lane quarter, each
// with 64/EQ columns of the chunk), then the producer and the MMA warp.
template <int EQ>
struct DwWarps {
    static constexpr int kEpi = 4 * EQ;
    static constexpr int kProducer = kEpi;
    static constexpr int kMma = kEpi + 1;
    static constexpr int kThreads = (kEpi + 2) * 32;
    static constexpr int kCols = 64 / EQ;
};
constexpr int kDwEq = 4;
constexpr int kDwPrefetch = 4; // row tiles prefetched into L2 ahead of the loads

template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[N]) {
    if constexpr (N == 32) {
        tmem_ld32(taddr, r);
    } else {
        static_assert(N == 16, "16 or 32 columns");
        tmem_ld16(taddr, r);
    }
}

// Column sums of v[0..31] over the 32 lanes: afterwards lane l holds the sum of column l.
__device__ __forceinline__ float warp_column_sum32(float (&v)[32], int lane) {
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) {
        const bool up = (lane & s) != 0;
#pragma unroll
        for (int i = 0; i < s; ++i) {
            const float send = up ? v[i] : v[i + s];
            const float keep = up ? v[i + s] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, s);
        }
    }
    return v[0];
}

// Column sums of v[0..N) over the 32 lanes: afterwards lane l (l < N) holds the sum of column l.
template <int N>
__device__ __forceinline__ float warp_column_sum(float (&v)[N], int lane) {
    if constexpr (N == 32) {
        return warp_column_sum32(v, lane);
    } else {
        static_assert(N == 16, "16 or 32 columns");
#pragma unroll
        for (int s = 8; s >= 1; s >>= 1) {
            const bool up = (lane & s) != 0;
#pragma unroll
            for (int i = 0; i < s; ++i) {
                const float send = up ? v[i] : v[i + s];
                const float keep = up ? v[i + s] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, s);
            }
        }
        // lanes l and l ^ 16 hold the two half-warp sums of column l & 15
        return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 16);
    }
}

template <typename T, int EQ>
__global__ void __launch_bounds__(DwWarps<EQ>::kThreads, 1)
    gdp_bwd_dw_kernel(const __grid_constant__ CUtensorMap tm_x,
                      const __grid_constant__ CUtensorMap tm_wp,
                      const __grid_constant__ CUtensorMap tm_wg,
                      const __grid_constant__ CUtensorMap tm_dout,
                      const uint16_t* __restrict__ bp, const uint16_t* __restrict__ bg,
                      const uint16_t* __restrict__ mask, float* __restrict__ dwp,
                      float* __restrict__ dwg, float* __restrict__ dbp, float* __restrict__ dbg,
                      int M, int K, int N, int n_groups) {
    using E = Elem<T>;
    using WR = DwWarps<EQ>;
    constexpr int kMmaWarp = WR::kMma;
    constexpr int kProducerWarp = WR::kProducer;
    constexpr int CW = WR::kCols;   // columns of the 64-column chunk per epilogue warp
    constexpr int NJ = CW / 2;      // column pairs
    constexpr int NH = CW / 8;      // 16-byte chunks
    const DwLayout L = dw_layout(K);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar);
    uint64_t* w_full = bars + 0;
    uint64_t* in_full = bars + 1;    // [2] x tile + dout chunk
    uint64_t* in_empty = bars + 3;   // [2]
    uint64_t* rec_full = bars + 5;   // [2] p, g of a tile in tensor-memory buffer i & 1
    uint64_t* ds_full = bars + 7;    // count 8
    uint64_t* dw_done = bars + 8;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.bar + 16 * 8);
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(tmem_slot + 1);
    float* red = reinterpret_cast<float*>(smem + L.red);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n_mt = (M + 127) / 128;
    const int chunk = blockIdx.x % ((N + 63) / 64);
    const int group = blockIdx.x / ((N + 63) / 64);
    const int n0 = chunk * 64;
    const int n_mine = (n_mt - group + n_groups - 1) / n_groups;

    if (threadIdx.x == 0) {
        mbar_init(w_full, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&in_full[s], 1);
            mbar_init(&in_empty[s], 1);
            mbar_init(&rec_full[s], 1);
        }
        mbar_init(ds_full, WR::kEpi);
        mbar_init(dw_done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    {
        const uint32_t one = E::kBf16 ? 0x3F80u : 0x3C00u;
        uint32_t* ones = reinterpret_cast<uint32_t*>(smem + L.ones);
        for (int i = threadIdx.x; i < 1024; i += blockDim.x) {
            ones[i] = ((i < 512) && ((i & 3) == 0)) ? one : 0u;
        }
        if (K <= 64) {
            for (int s = 0; s < 2; ++s) {
                uint32_t* z = reinterpret_cast<uint32_t*>(smem + L.x + s * 32768 + 16384);
                for (int i = threadIdx.x; i < 4096; i += blockDim.x) {
                    z[i] = 0u;
                }
            }
        }
        for (int i = threadIdx.x; i < 8 * 64; i += blockDim.x) {
            red[i] = 0.f;
        }
        if (warp == 0) {
            build_brow(reinterpret_cast<uint16_t*>(smem + L.bp), bp, n0, 64, N, lane);
            build_brow(reinterpret_cast<uint16_t*>(smem + L.bg), bg, n0, 64, N, lane);
        }
        fence_proxy_async_smem();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, 512);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // tensor memory: p, g of tile i at (i & 1) * 128 + {0, 64}; dwp at 256, dwg at 320.  The
    // two p/g buffers let the recompute of tile i+1 run while the epilogue works on tile i.

    if (warp == kProducerWarp) {
        if (lane == 0) {
            mbar_arrive_expect_tx(w_full, 2 * K * 128);
            tma_load_3d(smem + L.wp, &tm_wp, w_full, n0, 0, 0);
            tma_load_3d(smem + L.wg, &tm_wg, w_full, n0, 0, 0);
            const int panels = (K + 63) / 64;
            for (int i = 0; i < n_mine; ++i) {
                const int mt = group + i * n_groups;
                const int s = i & 1;
                // the tiles kDwPrefetch ahead into L2: the two stages alone cannot cover the
                // load latency of a streaming GPU
                for (int ip = (i == 0 ? 1 : i + kDwPrefetch); ip <= i + kDwPrefetch && ip < n_mine; ++ip) {
                    const int mp = group + ip * n_groups;
                    for (int pn = 0; pn < panels; ++pn) {
                        tma_prefetch_l2_3d(&tm_x, pn * 64, mp * 128, 0);
                    }
                    tma_prefetch_l2_3d(&tm_dout, n0, mp * 128, 0);
                }
                if (i >= 2 && !mbar_wait(&in_empty[s], ((i >> 1) - 1) & 1, abort_flag)) {
                    goto done;
                }
                mbar_arrive_expect_tx(&in_full[s], panels * 16384 + 16384);
                for (int pn = 0; pn < panels; ++pn) {
                    tma_load_3d(smem + L.x + s * 32768 + pn * 16384, &tm_x, &in_full[s],
                                pn * 64, mt * 128, 0);
                }
                tma_load_3d(smem + L.dout + s * 16384, &tm_dout, &in_full[s], n0, mt * 128, 0);
            }
        }
    } else if (warp == kMmaWarp) {
        // whole warp, converged: MMAs and commits are elect.sync-issued
        {
            // [p | g] and [dwp | dwg] as one N = 128 MMA each: wp | wg, bp | bg, hi_p | hi_g and
            // lo_p | lo_g are 64-column atoms at a fixed distance in shared memory
            constexpr uint32_t kIdRec = idesc_f16(128, 128, false, true, E::kBf16);
            constexpr uint32_t kIdDw = idesc_f16(128, 128, true, true, E::kBf16);
            const uint64_t ones = attn::interleave16_kmajor(sbase + L.ones);
            const int ksteps = K / 16;
            if (!mbar_wait_w(w_full, 0, abort_flag)) {
                goto done;
            }
            auto issue_dw = [&](int i) {
                // dw[k, n] += sum_m x[m, k] (hi + lo)[m, n]: A = x^T (MN-major), B MN-major
                const uint32_t xs = sbase + L.x + (i & 1) * 32768;
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {
                    const uint64_t a = smem_desc(xs + ks * 2048, 16384, 1024, kSwizzle128);
                    const uint32_t acc = (i > 0 || ks > 0) ? 1u : 0u;
                    umma_ss_w(tmem + 256, a, smem_desc(sbase + L.hi_p + ks * 2048, 16384, 1024, kSwizzle128), kIdDw, acc);
                    umma_ss_w(tmem + 256, a, smem_desc(sbase + L.lo_p + ks * 2048, 16384, 1024, kSwizzle128), kIdDw, 1);
                }
                umma_commit_w(dw_done);
                umma_commit_w(&in_empty[i & 1]);
            };
            for (int i = 0; i < n_mine; ++i) {
                const int s = i & 1;
                if (!mbar_wait_w(&in_full[s], (i >> 1) & 1, abort_flag)) {
                    goto done;
                }
                // p, g of tile i into buffer i & 1: its previous user, tile i-2, was read by
                // the epilogue before ds_full(i-2), which this loop waited for already
                const uint32_t xs = sbase + L.x + s * 32768;
                const uint32_t pg = tmem + s * 128;
                for (int ks = 0; ks < ksteps; ++ks) {
                    umma_ss_w(pg, x_desc(xs, ks), smem_desc(sbase + L.wp + ks * 2048, K * 128, 1024, kSwizzle128), kIdRec, ks > 0);
                }
                umma_ss_w(pg, ones, smem_desc(sbase + L.bp, 128, 256, kInterleave), kIdRec, 1);
                umma_commit_w(&rec_full[s]);
                if (i > 0) {
                    // dW of tile i-1 once its epilogue has written the hi / lo tiles
                    if (!mbar_wait_w(ds_full, (i - 1) & 1, abort_flag)) {
                        goto done;
                    }
                    tc_fence_after();
                    issue_dw(i - 1);
                }
            }
            if (n_mine > 0) {
                if (!mbar_wait_w(ds_full, (n_mine - 1) & 1, abort_flag)) {
                    goto done;
                }
                tc_fence_after();
                issue_dw(n_mine - 1);
            }
        }
    } else {
        const int w = warp >> 2;
        const int r = static_cast<int>(attn::warp_lane_base()) + lane;
        const uint32_t lane_off = attn::warp_lane_base() << 16;
        // bias gradients: this thread's row summed over its tiles, per column (pairs)
        float2 accp[NJ], accg[NJ];
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            accp[j] = make_float2(0.f, 0.f);
            accg[j] = make_float2(0.f, 0.f);
        }
        bool failed = false; // a wait gave up: leave together at the barrier after the loop
        for (int i = 0; i < n_mine; ++i) {
            const int mt = group + i * n_groups;
            const int row = mt * 128 + r;
            const bool row_ok = row < M;
            const float mk = row_ok ? E::to_float(mask[row]) : 0.f;
            if (!mbar_wait(&rec_full[i & 1], (i >> 1) & 1, abort_flag) ||
                !mbar_wait(&in_full[i & 1], (i >> 1) & 1, abort_flag)) {
                failed = true;
                break;
            }
            __syncwarp();
            tc_fence_after();
            float2 vp[NJ], vg[NJ]; // dp, dg of columns (2j, 2j + 1) of this warp's slice
            {
                uint32_t pv[CW], gv[CW];
                const uint32_t pg = tmem + lane_off + (i & 1) * 128 + CW * w;
                tmem_ld_cols(pg, pv);
                tmem_ld_cols(pg + 64, gv);
                tmem_ld_wait();
                const uint32_t do_row = sbase + L.dout + (i & 1) * 16384 + r * 128;
#pragma unroll
                for (int h = 0; h < NH; ++h) {
                    const uint4 dw4 = attn::lds128(do_row + (((NH * w + h) ^ (r & 7)) << 4));
                    const uint32_t dww[4] = {dw4.x, dw4.y, dw4.z, dw4.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int j = 4 * h + e;
                        gate_grads2(make_float2(__uint_as_float(pv[2 * j]), __uint_as_float(pv[2 * j + 1])),
                                    make_float2(__uint_as_float(gv[2 * j]), __uint_as_float(gv[2 * j + 1])),
                                    E::to_float2(dww[e]), mk, vp[j], vg[j]);
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                accp[j] = fadd2(accp[j], vp[j]);
                accg[j] = fadd2(accg[j], vg[j]);
            }
            // hi / lo tiles are free once the dw MMAs of tile i-1 are done (the gate gradients
            // above overlap them)
            if (i > 0 && !mbar_wait(dw_done, (i - 1) & 1, abort_flag)) {
                failed = true;
                break;
            }
            // hi + lo split (16-bit each) into the four MMA operand tiles
            const uint32_t rowoff = r * 128;
#pragma unroll
            for (int h = 0; h < NH; ++h) {
                uint32_t hp[4], lp[4], hg[4], lg[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int j = 4 * h + e;
                    hp[e] = E::pack(vp[j].x, vp[j].y);
                    hg[e] = E::pack(vg[j].x, vg[j].y);
                    const float2 rp = ffma2(E::to_float2(hp[e]), make_float2(-1.f, -1.f), vp[j]);
                    const float2 rg = ffma2(E::to_float2(hg[e]), make_float2(-1.f, -1.f), vg[j]);
                    lp[e] = E::pack(rp.x, rp.y);
                    lg[e] = E::pack(rg.x, rg.y);
                }
                const uint32_t off = rowoff + (((NH * w + h) ^ (r & 7)) << 4);
                attn::sts128(sbase + L.hi_p + off, make_uint4(hp[0], hp[1], hp[2], hp[3]));
                attn::sts128(sbase + L.lo_p + off, make_uint4(lp[0], lp[1], lp[2], lp[3]));
                attn::sts128(sbase + L.hi_g + off, make_uint4(hg[0], hg[1], hg[2], hg[3]));
                attn::sts128(sbase + L.lo_g + off, make_uint4(lg[0], lg[1], lg[2], lg[3]));
            }
            tc_fence_before();
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(ds_full);
            }
        }
        {
            // column sums over this warp's 32 rows, then over the 4 row quarters of each slice
            float cp[CW], cg[CW];
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                cp[2 * j] = accp[j].x;
                cp[2 * j + 1] = accp[j].y;
                cg[2 * j] = accg[j].x;
                cg[2 * j + 1] = accg[j].y;
            }
            const float sp = warp_column_sum<CW>(cp, lane);
            const float sg = warp_column_sum<CW>(cg, lane);
            if (lane < CW) {
                red[warp * 2 * CW + lane] = sp;
                red[warp * 2 * CW + CW + lane] = sg;
            }
        }
        if (!named_bar_and(1, WR::kEpi * 32, !failed && !*abort_flag)) {
            goto done;
        }
        if (threadIdx.x < 64) {
            const int ww = threadIdx.x / CW, col = threadIdx.x % CW;
            float sp = 0.f, sg = 0.f;
            for (int q = 0; q < 4; ++q) {
                sp += red[(4 * ww + q) * 2 * CW + col];
                sg += red[(4 * ww + q) * 2 * CW + CW + col];
            }
            const int n = n0 + CW * ww + col;
            if (n < N && n_mine > 0) {
                atomicAdd(dbp + n, sp);
                atomicAdd(dbg + n, sg);
            }
        }
        // weight gradients: thread (w, r) owns row k = r, columns [CW w, CW w + CW)
        if (n_mine > 0) {
            if (!mbar_wait(dw_done, (n_mine - 1) & 1, abort_flag)) {
                goto done;
            }
            __syncwarp();
            tc_fence_after();
            uint32_t a[CW], b[CW];
            tmem_ld_cols(tmem + lane_off + 256 + CW * w, a);
            tmem_ld_cols(tmem + lane_off + 320 + CW * w, b);
            tmem_ld_wait();
            if (r < K) {
#pragma unroll
                for (int j = 0; j < CW; ++j) {
                    const int n = n0 + CW * w + j;
                    if (n < N) {
                        atomicAdd(dwp + static_cast<int64_t>(r) * N + n, __uint_as_float(a[j]));
                        atomicAdd(dwg + static_cast<int64_t>(r) * N + n, __uint_as_float(b[j]));
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
    if (warp == kMmaWarp) {
        tmem_dealloc(tmem, 512);
    }
}

// ------------------------------------------------------------------------------------------
// CUDA-core backward for shapes outside the tcgen05 paths (workspace: f32 dp, dg [M, N]).
// ------------------------------------------------------------------------------------------
template <typename T>
__global__ void gdp_bwd_generic_grads_kernel(const uint16_t* __restrict__ x,
                                             const uint16_t* __restrict__ wp,
                                             const uint16_t* __restrict__ bp,
                                             const uint16_t* __restrict__ wg,
                                             const uint16_t* __restrict__ bg,
                                             const uint16_t* __restrict__ mask,
                                             const uint16_t* __restrict__ dout,
                                             float* __restrict__ dpw, float* __restrict__ dgw,
                                             int M, int K, int N) {
    using E = Elem<T>;
    __shared__ float xs[16][17], ps[16][17], gs[16][17];
    const int tx = threadIdx.x, ty = threadIdx.y;
    const int m = blockIdx.y * 16 + ty, n = blockIdx.x * 16 + tx;
    float ap = 0.f, ag = 0.f;
    for (int k0 = 0; k0 < K; k0 += 16) {
        const int kx = k0 + tx, kw = k0 + ty;
        xs[ty][tx] = (m < M && kx < K) ? E::to_float(x[static_cast<int64_t>(m) * K + kx]) : 0.f;
        ps[ty][tx] = (kw < K && n < N) ? E::to_float(wp[static_cast<int64_t>(kw) * N + n]) : 0.f;
        gs[ty][tx] = (kw < K && n < N) ? E::to_float(wg[static_cast<int64_t>(kw) * N + n]) : 0.f;
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
            ap = fmaf(xs[ty][kk], ps[kk][tx], ap);
            ag = fmaf(xs[ty][kk], gs[kk][tx], ag);
        }
        __syncthreads();
    }
    if (m < M && n < N) {
        float dp, dg;
        gate_grads(ap + E::to_float(bp[n]), ag + E::to_float(bg[n]),
                   E::to_float(dout[static_cast<int64_t>(m) * N + n]), E::to_float(mask[m]), dp,
                   dg);
        dpw[static_cast<int64_t>(m) * N + n] = dp;
        dgw[static_cast<int64_t>(m) * N + n] = dg;
    }
}

// dx[m, k] = sum_n dp[m, n] wp[k, n] + dg[m, n] wg[k, n]
template <typename T>
__global__ void gdp_bwd_generic_dx_kernel(const float* __restrict__ dpw,
                                          const float* __restrict__ dgw,
                                          const uint16_t* __restrict__ wp,
                                          const uint16_t* __restrict__ wg,
                                          uint16_t* __restrict__ dx, int M, int K, int N) {
    using E = Elem<T>;
    __shared__ float a[16][17], b[16][17], c[16][17], d[16][17];
    const int tx = threadIdx.x, ty = threadIdx.y;
    const int m = blockIdx.y * 16 + ty, k = blockIdx.x * 16 + tx;
    float acc = 0.f;
    for (int n0 = 0; n0 < N; n0 += 16) {
        const int na = n0 + tx;
        a[ty][tx] = (m < M && na < N) ? dpw[static_cast<int64_t>(m) * N + na] : 0.f;
        b[ty][tx] = (m < M && na < N) ? dgw[static_cast<int64_t>(m) * N + na] : 0.f;
        const int kb = blockIdx.x * 16 + ty; // weight row for column tx of the n tile
        c[ty][tx] = (kb < K && na < N) ? E::to_float(wp[static_cast<int64_t>(kb) * N + na]) : 0.f;
        d[ty][tx] = (kb < K && na < N) ? E::to_float(wg[static_cast<int64_t>(kb) * N + na]) : 0.f;
        __syncthreads();
#pragma unroll
        for (int nn = 0; nn < 16; ++nn) {
            acc = fmaf(a[ty][nn], c[tx][nn], acc);
            acc = fmaf(b[ty][nn], d[tx][nn], acc);
        }
        __syncthreads();
    }
    if (m < M && k < K) {
        dx[static_cast<int64_t>(m) * K + k] = E::from_float(acc);
    }
}

// dwp[k, n] = sum_m x[m, k] dp[m, n] (same for g); dbp[n] = sum_m dp[m, n]
template <typename T>
__global__ void gdp_bwd_generic_dw_kernel(const uint16_t* __restrict__ x,
                                          const float* __restrict__ dpw,
                                          const float* __restrict__ dgw, float* __restrict__ dwp,
                                          float* __restrict__ dwg, float* __restrict__ dbp,
                                          float* __restrict__ dbg, int M, int K, int N) {
    using E = Elem<T>;
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    const int k = blockIdx.y; // k == K computes the bias gradients
    if (n >= N) {
        return;
    }
    float sp = 0.f, sg = 0.f;
    for (int m = 0; m < M; ++m) {
        const float xv = (k < K) ? E::to_float(x[static_cast<int64_t>(m) * K + k]) : 1.f;
        sp = fmaf(xv, dpw[static_cast<int64_t>(m) * N + n], sp);
        sg = fmaf(xv, dgw[static_cast<int64_t>(m) * N + n], sg);
    }
    if (k < K) {
        dwp[static_cast<int64_t>(k) * N + n] = sp;
        dwg[static_cast<int64_t>(k) * N + n] = sg;
    } else {
        dbp[n] = sp;
        dbg[n] = sg;
    }
}

bool bwd_fast_shape(int64_t K, int64_t N) {
    return K % 16 == 0 && K >= 16 && K <= kMaxK && N % 8 == 0;
}

template <typename T>
int gdp_bwd_impl(cudaStream_t st, const DeviceInfo& dev, const void* x, const void* wp,
                 const void* bp, const void* wg, const void* bg, const void* mask,
                 const void* dout, void* dx, float* dwp, float* dbp, float* dwg, float* dbg,
                 void* ws, size_t ws_bytes, int M, int K, int N) {
    const uint16_t* xs = static_cast<const uint16_t*>(x);
    const uint16_t* wps = static_cast<const uint16_t*>(wp);
    const uint16_t* wgs = static_cast<const uint16_t*>(wg);
    const uint16_t* bps = static_cast<const uint16_t*>(bp);
    const uint16_t* bgs = static_cast<const uint16_t*>(bg);
    const uint16_t* ms = static_cast<const uint16_t*>(mask);
    const uint16_t* dos = static_cast<const uint16_t*>(dout);
    const bool fast = bwd_fast_shape(K, N) && aligned16(x) && aligned16(wp) && aligned16(wg) &&
                      aligned16(dout) && aligned16(dx);
    if (!fast) {
        const size_t need = static_cast<size_t>(M) * N * 8;
        if (!ws || ws_bytes < need) {
            return fail(CFK_ERR_INVALID_ARGUMENT,
                        "cfk_gdp_bwd: this shape or alignment needs a %zu-byte workspace", need);
        }
        float* dpw = static_cast<float*>(ws);
        float* dgw = dpw + static_cast<size_t>(M) * N;
        dim3 block(16, 16);
        gdp_bwd_generic_grads_kernel<T><<<dim3((N + 15) / 16, (M + 15) / 16), block, 0, st>>>(
            xs, wps, bps, wgs, bgs, ms, dos, dpw, dgw, M, K, N);
        gdp_bwd_generic_dx_kernel<T><<<dim3((K + 15) / 16, (M + 15) / 16), block, 0, st>>>(
            dpw, dgw, wps, wgs, static_cast<uint16_t*>(dx), M, K, N);
        gdp_bwd_generic_dw_kernel<T><<<dim3((N + 127) / 128, K + 1), 128, 0, st>>>(
            xs, dpw, dgw, dwp, dwg, dbp, dbg, M, K, N);
        return check_launch("gdp_bwd_generic");
    }
    if (cudaMemsetAsync(dwp, 0, static_cast<size_t>(K) * N * 4, st) != cudaSuccess ||
        cudaMemsetAsync(dwg, 0, static_cast<size_t>(K) * N * 4, st) != cudaSuccess ||
        cudaMemsetAsync(dbp, 0, static_cast<size_t>(N) * 4, st) != cudaSuccess ||
        cudaMemsetAsync(dbg, 0, static_cast<size_t>(N) * 4, st) != cudaSuccess) {
        return fail(CFK_ERR_LAUNCH, "cfk_gdp_bwd: memset failed");
    }
    CUtensorMap tx, twp, twg, tdo, tdo64;
    CFK_TRY(make_tmap_3d(&tx, x, K, M, 1, 2ull * K, 2ull * K * M, 64, 128, 1, 128, "gdp x"));
    CFK_TRY(make_tmap_3d(&twp, wp, N, K, 1, 2ull * N, 2ull * N * K, 64, K, 1, 128, "gdp wp"));
    CFK_TRY(make_tmap_3d(&twg, wg, N, K, 1, 2ull * N, 2ull * N * K, 64, K, 1, 128, "gdp wg"));
    CFK_TRY(make_tmap_3d(&tdo, dout, N, M, 1, 2ull * N, 2ull * N * M, 64, 128, 1, 128,
                         "gdp dout"));
    tdo64 = tdo;
    const int n_mt = (M + 127) / 128;
    if (dxr_layout(K, N).total <= 227 * 1024) {
        const DxrLayout L = dxr_layout(K, N);
        auto kern = gdp_bwd_dxr_kernel<T>;
        CFK_TRY(ensure_smem_attr(reinterpret_cast<const void*>(kern), dev.device, 227 * 1024,
                                 "gdp_bwd_dxr"));
        const int grid = std::min(n_mt, dev.num_sms);
        kern<<<grid, kDxrThreads, L.total, st>>>(tx, twp, twg, bps, bgs, ms, dos,
                                                 static_cast<uint16_t*>(dx), M, K, N);
        CFK_TRY(check_launch("gdp_bwd_dxr"));
    } else {
        const DxLayout L = dx_layout(K);
        auto kern = gdp_bwd_dx_kernel<T>;
        CFK_TRY(ensure_smem_attr(reinterpret_cast<const void*>(kern), dev.device, 227 * 1024,
                                 "gdp_bwd_dx"));
        const int grid = std::min(n_mt, dev.num_sms);
        kern<<<grid, kThreads, L.total, st>>>(tx, twp, twg, tdo, bps, bgs, ms,
                                              static_cast<uint16_t*>(dx), M, K, N);
        CFK_TRY(check_launch("gdp_bwd_dx"));
    }
    {
        const DwLayout L = dw_layout(K);
        auto kern = gdp_bwd_dw_kernel<T, kDwEq>;
        CFK_TRY(ensure_smem_attr(reinterpret_cast<const void*>(kern), dev.device, 227 * 1024,
                                 "gdp_bwd_dw"));
        const int nch = (N + 63) / 64;
        const int groups = std::max(1, std::min(n_mt, dev.num_sms / nch));
        kern<<<nch * groups, DwWarps<kDwEq>::kThreads, L.total, st>>>(tx, twp, twg, tdo64, bps, bgs, ms, dwp,
                                                      dwg, dbp, dbg, M, K, N, groups);
        CFK_TRY(check_launch("gdp_bwd_dw"));
    }
    return CFK_OK;
}

} // namespace
} // namespace gdp
} // namespace cfk

using namespace cfk;

namespace {
int check_gdp_args(const char* fn, int dtype, int64_t M, int64_t K, int64_t N) {
    if (dtype != CFK_F16 && dtype != CFK_BF16) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: dtype must be CFK_F16 or CFK_BF16", fn);
    }
    if (M < 0 || K <= 0 || N <= 0) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: x must be [M,K], wp/wg [K,N] with K, N > 0",
                    fn);
    }
    // cuda/volta_ops.cu:234-236
    if (N % 8) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: N must be a multiple of 8", fn);
    }
    if (M > (1ll << 31) - 1 || K > 65535 || N > 65535) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: tensor too large", fn);
    }
    return CFK_OK;
}
} // namespace

extern "C" int cfk_gdp_fwd(cfk_stream_t stream, cfk_dtype dtype, const void* x, const void* wp,
                           const void* bp, const void* wg, const void* bg, const void* mask,
                           void* out, int64_t M, int64_t K, int64_t N) {
    clear_error();
    CFK_TRY(check_gdp_args("cfk_gdp_fwd", dtype, M, K, N));
    if (M == 0) {
        return CFK_OK;
    }
    if (!x || !wp || !bp || !wg || !bg || !mask || !out) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_gdp_fwd: null buffer");
    }
    DeviceInfo dev;
    CFK_TRY(current_device(&dev));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int m = static_cast<int>(M), k = static_cast<int>(K), n = static_cast<int>(N);
    return dtype == CFK_BF16
               ? gdp::gdp_fwd_impl<__nv_bfloat16>(st, dev, x, wp, bp, wg, bg, mask, out, m, k, n)
               : gdp::gdp_fwd_impl<__half>(st, dev, x, wp, bp, wg, bg, mask, out, m, k, n);
}

extern "C" int cfk_ln_gdp_fwd_workspace_size(int64_t M, int64_t K, int64_t N, size_t* bytes) {
    clear_error();
    CFK_TRY(check_gdp_args("cfk_ln_gdp_fwd_workspace_size", CFK_BF16, M, K, N));
    if (!bytes) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_ln_gdp_fwd_workspace_size: null pointer");
    }
    // the fused kernel needs none; other shapes stage LayerNorm(z) [M, K] in the workspace
    *bytes = gdp::fwd_fast_shape(static_cast<int>(K), static_cast<int>(N))
                 ? 0
                 : static_cast<size_t>(M) * static_cast<size_t>(K) * 2;
    return CFK_OK;
}

extern "C" int cfk_ln_gdp_fwd(cfk_stream_t stream, cfk_dtype dtype, const void* z,
                              const float* gamma, const float* beta, float eps, const void* wp,
                              const void* bp, const void* wg, const void* bg, const void* mask,
                              void* out, float* mean, float* rstd, void* workspace,
                              size_t workspace_bytes, int64_t M, int64_t K, int64_t N) {
    clear_error();
    CFK_TRY(check_gdp_args("cfk_ln_gdp_fwd", dtype, M, K, N));
    if (!(eps >= 0.f)) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_ln_gdp_fwd: eps must be >= 0");
    }
    if (M == 0) {
        return CFK_OK;
    }
    if (!z || !gamma || !beta || !wp || !bp || !wg || !bg || !mask || !out) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_ln_gdp_fwd: null buffer");
    }
    DeviceInfo dev;
    CFK_TRY(current_device(&dev));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int m = static_cast<int>(M), k = static_cast<int>(K), n = static_cast<int>(N);
    const bool fused = gdp::fwd_fast_shape(k, n) && aligned16(z) && aligned16(wp) &&
                       aligned16(wg) && aligned16(out);
    if (fused) {
        const gdp::LnIn ln{static_cast<const uint16_t*>(z), gamma, beta, mean, rstd, eps};
        return dtype == CFK_BF16 ? gdp::gdp_fwd_impl<__nv_bfloat16>(st, dev, nullptr, wp, bp, wg,
                                                                     bg, mask, out, m, k, n, &ln)
                                 : gdp::gdp_fwd_impl<__half>(st, dev, nullptr, wp, bp, wg, bg,
                                                             mask, out, m, k, n, &ln);
    }
    // two kernels through a staged LayerNorm output
    const size_t need = static_cast<size_t>(M) * static_cast<size_t>(K) * 2;
    if (!workspace || workspace_bytes < need || !aligned16(workspace)) {
        return fail(CFK_ERR_INVALID_ARGUMENT,
                    "cfk_ln_gdp_fwd: this shape or alignment needs a 16-byte aligned %zu-byte "
                    "workspace (got %zu)", need, workspace_bytes);
    }
    CFK_TRY(cfk_ln_fwd(stream, dtype, z, gamma, beta, workspace, mean, rstd, M, K, eps));
    clear_error();
    return dtype == CFK_BF16 ? gdp::gdp_fwd_impl<__nv_bfloat16>(st, dev, workspace, wp, bp, wg,
                                                                 bg, mask, out, m, k, n)
                             : gdp::gdp_fwd_impl<__half>(st, dev, workspace, wp, bp, wg, bg,
                                                         mask, out, m, k, n);
}

extern "C" int cfk_gdp_bwd_workspace_size(int64_t M, int64_t K, int64_t N, size_t* bytes) {
    clear_error();
    CFK_TRY(check_gdp_args("cfk_gdp_bwd_workspace_size", CFK_BF16, M, K, N));
    if (!bytes) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_gdp_bwd_workspace_size: null pointer");
    }
    // The tcgen05 path needs none; other shapes keep f32 dp and dg.
    *bytes = gdp::bwd_fast_shape(K, N) ? 0 : static_cast<size_t>(M * N) * 8;
    return CFK_OK;
}

extern "C" int cfk_gdp_bwd(cfk_stream_t stream, cfk_dtype dtype, const void* x, const void* wp,
                           const void* bp, const void* wg, const void* bg, const void* mask,
                           const void* dout, void* dx, float* dwp, float* dbp, float* dwg,
                           float* dbg, void* workspace, size_t workspace_bytes, int64_t M,
                           int64_t K, int64_t N) {
    clear_error();
    CFK_TRY(check_gdp_args("cfk_gdp_bwd", dtype, M, K, N));
    if (!wp || !bp || !wg || !bg || !dwp || !dbp || !dwg || !dbg) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_gdp_bwd: null buffer");
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (M == 0) {
        cudaError_t e = cudaMemsetAsync(dwp, 0, static_cast<size_t>(K * N) * 4, st);
        if (e == cudaSuccess) e = cudaMemsetAsync(dwg, 0, static_cast<size_t>(K * N) * 4, st);
        if (e == cudaSuccess) e = cudaMemsetAsync(dbp, 0, static_cast<size_t>(N) * 4, st);
        if (e == cudaSuccess) e = cudaMemsetAsync(dbg, 0, static_cast<size_t>(N) * 4, st);
        return e == cudaSuccess ? CFK_OK : fail(CFK_ERR_LAUNCH, "cfk_gdp_bwd: memset failed");
    }
    if (!x || !mask || !dout || !dx) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_gdp_bwd: null buffer");
    }
    DeviceInfo dev;
    CFK_TRY(current_device(&dev));
    const int m = static_cast<int>(M), k = static_cast<int>(K), n = static_cast<int>(N);
    return dtype == CFK_BF16
               ? gdp::gdp_bwd_impl<__nv_bfloat16>(st, dev, x, wp, bp, wg, bg, mask, dout, dx, dwp,
                                                  dbp, dwg, dbg, workspace, workspace_bytes, m, k,
                                                  n)
               : gdp::gdp_bwd_impl<__half>(st, dev, x, wp, bp, wg, bg, mask, dout, dx, dwp, dbp,
                                           dwg, dbg, workspace, workspace_bytes, m, k, n);
}
