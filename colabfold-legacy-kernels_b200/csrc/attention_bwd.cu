// attention_bwd.cu -- backward of attention with pair bias and key mask, tcgen05 + TMA.
//
// The reference is forward-only; this is the exact derivative of cuda/volta_mma_attn.cu:139-271
// (masked logits are constants -1e4, so they pass no gradient):
//
//   P = exp(logit - lse)        dV = P^T dO        dP = dO V^T        delta_i = sum_d dO O
//   dS = P * (dP - delta)       dQ = scale dS K    dK = scale dS^T Q  dbias = sum_n dS
//
// dbias sums over the batch rows n, so the work item keeps its (query tile, key tile) fixed and
// walks the batch rows: its 128 x 128 dbias tile lives in registers for the whole walk and is
// written once (no atomics when the item covers every row, a deterministic result).  dQ, dK
// and dV of one batch row are then partial sums over key tiles (dQ) or query tiles (dK, dV);
// the MMA writes those partials into tensor memory, the dS warpgroups stage them in swizzled
// shared memory and a TMA tensor reduce-add folds them into f32 accumulators in the workspace.
// A final kernel converts the accumulators to the 16-bit outputs.
//
//   warps 0-7   dS warpgroups: thread (w, r) owns query row r and key columns [64w, 64w+64).
//   warp 8      TMA producer: bias tile per item; per batch row q, dO, k, v tiles and the
//               key-mask operand (as in the forward).
//   warp 9      MMA issuer: S = q k^T (+ mask), dP = dO v^T; then dV = P^T dO, dK = dS^T q,
//               dQ = dS k from the P and dS tiles the warpgroups wrote to shared memory.
#include <type_traits>

#include "attention_common.cuh"
#include "host.h"

namespace cfk {
namespace attn {
namespace {

template <int D>
struct BwdCfg {
    using G = Geo<D>;
    static constexpr int NST = (D == 64) ? 1 : 2; // operand stages
    static constexpr int NPB = (D == 64) ? 1 : 2; // partial-sum buffers in tensor memory
    static constexpr int kThreads = 320;
    static constexpr int kProducerWarp = 8;
    static constexpr int kMmaWarp = 9;
    static constexpr uint32_t kTmemCols = 512;
    static constexpr int kSCol = 0;
    static constexpr int kDPCol = 128;
    static constexpr int kPartCol = 256; // buffer pb: dV, dK, dQ at 256 + pb*3*Dp + {0,1,2}*Dp

    static constexpr int kTile = ((G::kTileAlloc + 1023) / 1024) * 1024;
    static constexpr int kMaskOpBytes = 128 * 16 * 2;
    static constexpr int kOffSQ = 0;
    static constexpr int kOffSdO = kTile;
    static constexpr int kOffSK = 2 * kTile;
    static constexpr int kOffSV = 3 * kTile;
    static constexpr int kOffSMask = 4 * kTile;
    static constexpr int kStageBytes = 4 * kTile + kMaskOpBytes;

    // f32 staging of one [128 x D] partial for the TMA reduce: panels of kPW floats per row
    static constexpr int kPW = D < 32 ? D : 32;
    static constexpr int kRowB = kPW * 4;           // bytes of one staging row (= swizzle span)
    static constexpr int kPanelBytes = 128 * kRowB;
    static constexpr int kStgBytes = 128 * D * 4;
    static constexpr int NSTG = (D == 64) ? 1 : 3;

    static constexpr int kOffStages = 0;
    static constexpr int kOffOnes = NST * kStageBytes;
    static constexpr int kOffBias = kOffOnes + kMaskOpBytes;
    static constexpr int kOffP = kOffBias + 32768;
    static constexpr int kOffDS = kOffP + 32768;
    static constexpr int kOffStg = kOffDS + 32768;
    static constexpr int kOffKeep = kOffStg + NSTG * kStgBytes; // u8 [NST][128]
    static constexpr int kOffFlag = kOffKeep + NST * 128;       // u32 [NST]
    static constexpr int kOffBar = ((kOffFlag + NST * 4 + 7) / 8) * 8;
    // kv_full[NST], kv_empty[NST], bias_full, bias_empty, sdp_full, pds_full, pds_empty,
    // part_full[NPB], part_empty[NPB], sdp_free
    static constexpr int kNumBars = 2 * NST + 6 + 2 * NPB;
    static constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
    static constexpr int kOffAbort = kOffTmemSlot + 4;
    static constexpr int kSmemBytes = kOffAbort + 4 + 1024;
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
    static_assert(kPartCol + NPB * 3 * G::kDp <= 512, "tensor memory budget");
};

struct BwdParams {
    const uint8_t* kmask;
    const uint16_t* bias; // raw pointer (read directly when the bias tile is not loaded by TMA)
    const float* lse;
    const float* delta;
    float* dbias;
    int N, H, Sq, Sk;
    int n_it, n_jt, n_bc, bchunk;
    int64_t items;
    float scale;
    uint32_t mask_bits;
    int dbias_atomic; // several batch chunks add into a zeroed dbias
};

// Byte offset of the 16-byte chunk `c` of row `r` in a staging panel of kRowB-byte rows
// (TMA swizzle of span kRowB).
template <int kRowB>
__device__ __forceinline__ uint32_t stg_chunk(int r, int c) {
    constexpr int kMask = kRowB / 16 - 1;
    return static_cast<uint32_t>(r * kRowB + ((c ^ ((r * kRowB >> 7) & kMask)) << 4));
}

template <typename T, int D, bool kBiasTma>
__global__ void __launch_bounds__(320, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v,
                    const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_bias,
                    const __grid_constant__ CUtensorMap tm_dq_acc,
                    const __grid_constant__ CUtensorMap tm_dk_acc,
                    const __grid_constant__ CUtensorMap tm_dv_acc, const BwdParams p) {
    using C = BwdCfg<D>;
    using G = Geo<D>;
    using E = Elem<T>;
    constexpr int NST = C::NST;
    constexpr int NPB = C::NPB;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
    uint64_t* kv_full = bars;
    uint64_t* kv_empty = bars + NST;
    uint64_t* bias_full = bars + 2 * NST;
    uint64_t* bias_empty = bias_full + 1;
    uint64_t* sdp_full = bias_full + 2;
    uint64_t* pds_full = bias_full + 3;
    uint64_t* pds_empty = bias_full + 4;
    uint64_t* part_full = bias_full + 5;
    uint64_t* part_empty = part_full + NPB;
    uint64_t* sdp_free = part_empty + NPB; // S and dP of the current step read out of TMEM
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffTmemSlot);
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + C::kOffAbort);
    uint8_t* keep_all = smem + C::kOffKeep;
    uint32_t* flag_all = reinterpret_cast<uint32_t*>(smem + C::kOffFlag);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&kv_full[s], 2); // TMA transaction arrival + mask operand arrival
            mbar_init(&kv_empty[s], 1 + 8);
        }
        mbar_init(bias_full, 1);
        mbar_init(bias_empty, 8);
        mbar_init(sdp_full, 1);
        mbar_init(pds_full, 8);
        mbar_init(pds_empty, 1);
        for (int b = 0; b < NPB; ++b) {
            mbar_init(&part_full[b], 1);
            mbar_init(&part_empty[b], 8);
        }
        mbar_init(sdp_free, 8);
        *abort_flag = 0;
        fence_mbar_init();
    }
    {
        uint32_t* ones = reinterpret_cast<uint32_t*>(smem + C::kOffOnes);
        for (int i = threadIdx.x; i < C::kMaskOpBytes / 4; i += blockDim.x) {
            ones[i] = ((i < 512) && ((i & 3) == 0)) ? 0x3F80u : 0u; // column 0 = 1.0 (bf16)
        }
        for (int s = 0; s < NST; ++s) {
            uint32_t* mo = reinterpret_cast<uint32_t*>(smem + C::kOffStages + s * C::kStageBytes +
                                                       C::kOffSMask);
            for (int i = threadIdx.x; i < C::kMaskOpBytes / 4; i += blockDim.x) {
                mo[i] = 0u;
            }
            if constexpr (D == 8) {
                for (int t = 0; t < 4; ++t) {
                    uint32_t* z = reinterpret_cast<uint32_t*>(
                        smem + C::kOffStages + s * C::kStageBytes + t * C::kTile + G::kTileBytes);
                    for (int i = threadIdx.x; i < G::kTileBytes / 4; i += blockDim.x) {
                        z[i] = 0u;
                    }
                }
            }
        }
        fence_proxy_async_smem();
    }
    if (warp == C::kMmaWarp) {
        tmem_alloc(tmem_slot, C::kTmemCols);
    }
    if (warp == C::kProducerWarp && lane == 0) {
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_k);
        tma_prefetch_desc(&tm_v);
        tma_prefetch_desc(&tm_do);
        if constexpr (kBiasTma) {
            tma_prefetch_desc(&tm_bias);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int n_items_mine = static_cast<int>((p.items - blockIdx.x + gridDim.x - 1) / gridDim.x);

    if (warp == C::kProducerWarp) {
        // =============================== TMA producer ===============================
        uint32_t g = 0;
        for (int it = 0; it < n_items_mine; ++it) {
            const int64_t item = blockIdx.x + static_cast<int64_t>(it) * gridDim.x;
            const int jt = static_cast<int>(item % p.n_jt);
            int64_t rest = item / p.n_jt;
            const int itile = static_cast<int>(rest % p.n_it);
            rest /= p.n_it;
            const int h = static_cast<int>(rest % p.H);
            const int bc = static_cast<int>(rest / p.H);
            const int i0 = itile * kBM, j0 = jt * kBN;
            const int b_lo = bc * p.bchunk, b_hi = min(p.N, b_lo + p.bchunk);
            if (it > 0 && !mbar_wait(bias_empty, (it - 1) & 1, abort_flag)) {
                goto done;
            }
            if (lane == 0) {
                if constexpr (kBiasTma) {
                    mbar_arrive_expect_tx(bias_full, 32768);
                    tma_load_3d(smem + C::kOffBias, &tm_bias, bias_full, j0, i0, h);
                    tma_load_3d(smem + C::kOffBias + 16384, &tm_bias, bias_full, j0 + 64, i0, h);
                } else {
                    mbar_arrive(bias_full);
                }
            }
            for (int b = b_lo; b < b_hi; ++b, ++g) {
                const int s = g % NST;
                // key-mask codes of this batch row, read before waiting for the stage so the
                // global-load latency overlaps the wait: 2 = keep, 1 = masked, 0 = past Sk
                uint8_t codes[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int j = j0 + lane * 4 + r;
                    codes[r] = j >= p.Sk ? 0 : (p.kmask[static_cast<int64_t>(b) * p.Sk + j] ? 2 : 1);
                }
                if (g >= NST && !mbar_wait(&kv_empty[s], ((g / NST) - 1) & 1, abort_flag)) {
                    goto done;
                }
                uint8_t* stage = smem + C::kOffStages + s * C::kStageBytes;
                if (lane == 0) {
                    // operand tiles first: their latency is the longest on this path
                    mbar_arrive_expect_tx(&kv_full[s], 4 * G::kTileBytes);
                    const int bh = b * p.H + h;
                    tma_load_3d(stage + C::kOffSQ, &tm_q, &kv_full[s], 0, i0, bh);
                    tma_load_3d(stage + C::kOffSdO, &tm_do, &kv_full[s], 0, i0, bh);
                    tma_load_3d(stage + C::kOffSK, &tm_k, &kv_full[s], 0, j0, bh);
                    tma_load_3d(stage + C::kOffSV, &tm_v, &kv_full[s], 0, j0, bh);
                }
                uint16_t* mo = reinterpret_cast<uint16_t*>(stage + C::kOffSMask);
                uint8_t* keep = keep_all + s * 128;
                bool any_excluded = false;
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int jj = lane * 4 + r;
                    keep[jj] = codes[r];
                    mo[jj * 8] = (codes[r] == 2 || p.mask_bits == 0) ? uint16_t(0)
                                                                     : uint16_t(p.mask_bits);
                    any_excluded |= (codes[r] != 2);
                }
                const uint32_t anyx = __any_sync(0xffffffffu, any_excluded);
                if (lane == 0) {
                    flag_all[s] = anyx;
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&kv_full[s]); // mask operand, keep codes and flag written
                }
                __syncwarp();
            }
        }
    } else if (warp == C::kMmaWarp) {
        // =============================== MMA issuer ===============================
        if (lane == 0) {
            constexpr uint32_t kIdS = idesc_f16(128, 128, false, false, E::kBf16);
            constexpr uint32_t kIdMask = idesc_f16(128, 128, false, false, true);
            constexpr uint32_t kIdPart = idesc_f16(128, G::kDp, true, true, E::kBf16);  // P^T, dS^T
            constexpr uint32_t kIdDQ = idesc_f16(128, G::kDp, false, true, E::kBf16);   // dS
            const uint64_t ones_desc = interleave16_kmajor(sbase + C::kOffOnes);
            const uint32_t p_s = sbase + C::kOffP;
            const uint32_t ds_s = sbase + C::kOffDS;
            uint32_t g = 0;
            int total_steps = 0;
            for (int it = 0; it < n_items_mine; ++it) {
                const int64_t item = blockIdx.x + static_cast<int64_t>(it) * gridDim.x;
                const int bc = static_cast<int>(item / p.n_jt / p.n_it / p.H);
                const int b_lo = bc * p.bchunk, b_hi = min(p.N, b_lo + p.bchunk);
                total_steps += max(0, b_hi - b_lo);
            }
            // partial sums of step gp (operands in stage gp % NST) into buffer gp % NPB
            auto issue_partials = [&](uint32_t gp) -> bool {
                const int pb = gp % NPB;
                if (gp >= static_cast<uint32_t>(NPB) &&
                    !mbar_wait(&part_empty[pb], ((gp / NPB) - 1) & 1, abort_flag)) {
                    return false;
                }
                tc_fence_after();
                const uint32_t st = sbase + C::kOffStages + (gp % NST) * C::kStageBytes;
                const uint32_t dv_tm = tmem + C::kPartCol + pb * 3 * G::kDp;
                const uint32_t dk_tm = dv_tm + G::kDp;
                const uint32_t dq_tm = dv_tm + 2 * G::kDp;
#pragma unroll
                for (int ks = 0; ks < kBM / 16; ++ks) {
                    // A = P^T / dS^T: [M = key j, K = query i], MN-major (128B swizzle panels)
                    const uint64_t pa = smem_desc(p_s + ks * 2048, 16384, 1024, kSwizzle128);
                    const uint64_t da = smem_desc(ds_s + ks * 2048, 16384, 1024, kSwizzle128);
                    umma_ss(dv_tm, pa, G::mnmajor(st + C::kOffSdO, ks), kIdPart, ks > 0);
                    umma_ss(dk_tm, da, G::mnmajor(st + C::kOffSQ, ks), kIdPart, ks > 0);
                }
#pragma unroll
                for (int ks = 0; ks < kBN / 16; ++ks) {
                    // A = dS: [M = query i, K = key j], K-major
                    const uint64_t da =
                        smem_desc(ds_s + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024, kSwizzle128);
                    umma_ss(dq_tm, da, G::mnmajor(st + C::kOffSK, ks), kIdDQ, ks > 0);
                }
                umma_commit(&part_full[pb]);
                umma_commit(pds_empty);
                umma_commit(&kv_empty[gp % NST]);
                return true;
            };
            for (int step = 0; step < total_steps; ++step, ++g) {
                const int s = g % NST;
                if (NST == 1 && g > 0) {
                    // one operand stage: step g's operands overwrite step g-1's, so the
                    // partial sums of g-1 go first
                    if (!mbar_wait(pds_full, (g - 1) & 1, abort_flag) || !issue_partials(g - 1)) {
                        goto done;
                    }
                }
                if (!mbar_wait(&kv_full[s], (g / NST) & 1, abort_flag)) {
                    goto done;
                }
                if (NST > 1 && g > 0 && !mbar_wait(sdp_free, (g - 1) & 1, abort_flag)) {
                    goto done;
                }
                tc_fence_after();
                const uint32_t st = sbase + C::kOffStages + s * C::kStageBytes;
#pragma unroll
                for (int ks = 0; ks < G::kKSteps; ++ks) {
                    umma_ss(tmem + C::kSCol, G::kmajor(st + C::kOffSQ, ks),
                            G::kmajor(st + C::kOffSK, ks), kIdS, ks > 0);
                }
                umma_ss(tmem + C::kSCol, ones_desc, interleave16_kmajor(st + C::kOffSMask),
                        kIdMask, 1);
#pragma unroll
                for (int ks = 0; ks < G::kKSteps; ++ks) {
                    umma_ss(tmem + C::kDPCol, G::kmajor(st + C::kOffSdO, ks),
                            G::kmajor(st + C::kOffSV, ks), kIdS, ks > 0);
                }
                umma_commit(sdp_full);
                if (NST > 1 && g > 0 &&
                    (!mbar_wait(pds_full, (g - 1) & 1, abort_flag) || !issue_partials(g - 1))) {
                    goto done;
                }
            }
            if (g > 0) {
                if (!mbar_wait(pds_full, (g - 1) & 1, abort_flag) || !issue_partials(g - 1)) {
                    goto done;
                }
            }
        }
    } else {
        // =============================== dS warpgroups ===============================
        const int w = warp >> 2;
        const int r = static_cast<int>(warp_lane_base()) + lane;
        const uint32_t lane_off = warp_lane_base() << 16;
        const float scale = p.scale;
        const bool always_select = (p.mask_bits == 0);
        const uint32_t p_s = sbase + C::kOffP + w * 16384 + r * 128;
        const uint32_t ds_s = sbase + C::kOffDS + w * 16384 + r * 128;
        const uint32_t bias_row = sbase + C::kOffBias + w * 16384 + r * 128;
        uint32_t g = 0;
        int prev_b = 0, prev_h = 0, prev_i0 = 0, prev_j0 = 0;

        // Stages the partial sums of step gp from tensor memory and reduces them into the f32
        // accumulators (dV, dK at key rows, dQ at query rows).
        auto drain = [&](uint32_t gp, int bh, int i0, int j0) -> bool {
            const int pb = gp % NPB;
            if (!mbar_wait(&part_full[pb], (gp / NPB) & 1, abort_flag)) {
                return false;
            }
            __syncwarp();
            tc_fence_after();
            if (threadIdx.x == 0) {
                bulk_wait_read<0>(); // the previous reductions have read the staging buffers
            }
            named_bar_sync(1, 256);
            const uint32_t part = tmem + lane_off + C::kPartCol + pb * 3 * G::kDp;
#pragma unroll
            for (int t = 0; t < 3; ++t) {
                uint8_t* stg = smem + C::kOffStg + (t % C::NSTG) * C::kStgBytes;
                if (t >= C::NSTG) {
                    if (threadIdx.x == 0) {
                        bulk_wait_read<0>();
                    }
                    named_bar_sync(1, 256);
                }
                constexpr int kHalf = G::kDp / 2;
                float v[kHalf];
                {
                    uint32_t raw[kHalf];
                    if constexpr (kHalf == 8) {
                        tmem_ld8(part + t * G::kDp + w * kHalf, raw);
                    } else if constexpr (kHalf == 16) {
                        tmem_ld16(part + t * G::kDp + w * kHalf, raw);
                    } else {
                        tmem_ld32(part + t * G::kDp + w * kHalf, raw);
                    }
                    tmem_ld_wait();
#pragma unroll
                    for (int k = 0; k < kHalf; ++k) {
                        v[k] = __uint_as_float(raw[k]); // dK, dQ: dS already carries the scale
                    }
                }
                if (w * kHalf < D) {
#pragma unroll
                    for (int q = 0; q < kHalf / 4; ++q) {
                        const int col = w * kHalf + q * 4;
                        const int panel = col / C::kPW;
                        const int cc = (col % C::kPW) / 4;
                        sts128(smem_u32(stg) + panel * C::kPanelBytes + stg_chunk<C::kRowB>(r, cc),
                               make_uint4(__float_as_uint(v[4 * q]), __float_as_uint(v[4 * q + 1]),
                                          __float_as_uint(v[4 * q + 2]),
                                          __float_as_uint(v[4 * q + 3])));
                    }
                }
                if (t + 1 == 3 || (t + 1) % C::NSTG == 0) {
                    // buffers [t0, t] are complete: hand them to the TMA
                    fence_proxy_async_smem();
                    named_bar_sync(1, 256);
                    if (threadIdx.x == 0) {
                        const int t0 = (C::NSTG == 1) ? t : 0;
                        for (int u = t0; u <= t; ++u) {
                            const uint8_t* sb = smem + C::kOffStg + (u % C::NSTG) * C::kStgBytes;
                            const CUtensorMap* tm = u == 0 ? &tm_dv_acc : (u == 1 ? &tm_dk_acc : &tm_dq_acc);
                            const int row0 = (u == 2) ? i0 : j0;
#pragma unroll
                            for (int pn = 0; pn < D / C::kPW; ++pn) {
                                tma_reduce_add_3d(tm, sb + pn * C::kPanelBytes, pn * C::kPW, row0,
                                                  bh);
                            }
                        }
                        bulk_commit();
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&part_empty[pb]);
            }
            return true;
        };

        for (int it = 0; it < n_items_mine; ++it) {
            const int64_t item = blockIdx.x + static_cast<int64_t>(it) * gridDim.x;
            const int jt = static_cast<int>(item % p.n_jt);
            int64_t rest = item / p.n_jt;
            const int itile = static_cast<int>(rest % p.n_it);
            rest /= p.n_it;
            const int h = static_cast<int>(rest % p.H);
            const int bc = static_cast<int>(rest / p.H);
            const int i0 = itile * kBM, j0 = jt * kBN;
            const int b_lo = bc * p.bchunk, b_hi = min(p.N, b_lo + p.bchunk);
            const int row = i0 + r;
            const bool row_ok = row < p.Sq;
            float dbias[64];
#pragma unroll
            for (int k = 0; k < 64; ++k) {
                dbias[k] = 0.f;
            }
            if (!mbar_wait(bias_full, it & 1, abort_flag)) {
                goto done;
            }
            for (int b = b_lo; b < b_hi; ++b, ++g) {
                const int s = g % NST;
                // row statistics first: their latency overlaps the wait for S and dP
                const int64_t lrow = (static_cast<int64_t>(b) * p.H + h) * p.Sq + row;
                const float lse = row_ok ? p.lse[lrow] : 0.f;
                const float delta = row_ok ? p.delta[lrow] : 0.f;
                if (!mbar_wait(sdp_full, g & 1, abort_flag) ||
                    !mbar_wait(&kv_full[s], (g / NST) & 1, abort_flag)) {
                    goto done;
                }
                __syncwarp();
                tc_fence_after();
                const float lseL = lse * kLog2e;
                const bool select = flag_all[s] != 0 && (always_select || lse < kMaskedLogit + 104.f);
                const float p_masked = ex2((kMaskedLogit - lse) * kLog2e);
                const uint8_t* keep = keep_all + s * 128 + 64 * w;
                // dS is computed pre-multiplied by the softmax scale (both dK and dQ carry it);
                // dbias divides it out once when the tile is written.
                const float sdelta = scale * delta;
                // kSel: some row of this warp needs the exact masked-logit replacement (rows
                // whose every unmasked logit is below the mask constant, or masks with no bias
                // code); the common path carries no per-element select.
                auto ds_tile = [&](auto sel_tag) -> bool {
                constexpr bool kSel = decltype(sel_tag)::value;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int col0 = 64 * w + 16 * c; // key column within the tile
                    uint32_t sv[16], dpv[16];
                    tmem_ld16(tmem + lane_off + C::kSCol + col0, sv);
                    tmem_ld16(tmem + lane_off + C::kDPCol + col0, dpv);
                    tmem_ld_wait();
                    if (c == 3 && NST > 1) {
                        // S and dP are in registers: the MMA may overwrite them with the next
                        // batch row's tiles
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) {
                            mbar_arrive(sdp_free);
                        }
                    }
                    float bvals[16];
                    if constexpr (kBiasTma) {
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            const uint4 bw = lds128(bias_row + (((2 * c + q) ^ (r & 7)) << 4));
                            const uint32_t wv[4] = {bw.x, bw.y, bw.z, bw.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float2 f = E::to_float2(wv[e]);
                                bvals[8 * q + 2 * e] = f.x;
                                bvals[8 * q + 2 * e + 1] = f.y;
                            }
                        }
                    } else {
                        const int64_t brow = (static_cast<int64_t>(h) * p.Sq + (row_ok ? row : 0)) * p.Sk;
#pragma unroll
                        for (int k = 0; k < 16; ++k) {
                            const int j = j0 + col0 + k;
                            bvals[k] = (row_ok && j < p.Sk) ? E::to_float(p.bias[brow + j]) : 0.f;
                        }
                    }
                    uint32_t pk[8], dk[8];
                    const float2 scale2 = make_float2(scale, scale);
                    const float2 l2 = make_float2(kLog2e, kLog2e);
                    const float2 nlse2 = make_float2(-lseL, -lseL);
                    const float2 nsdelta2 = make_float2(-sdelta, -sdelta);
#pragma unroll
                    for (int k = 0; k < 16; k += 2) {
                        const float2 t2 = ffma2(make_float2(__uint_as_float(sv[k]),
                                                            __uint_as_float(sv[k + 1])),
                                                scale2, make_float2(bvals[k], bvals[k + 1]));
                        const float2 a2 = ffma2(t2, l2, nlse2);
                        float2 p2 = make_float2(ex2(a2.x), ex2(a2.y));
                        const float2 d2 = ffma2(make_float2(__uint_as_float(dpv[k]),
                                                            __uint_as_float(dpv[k + 1])),
                                                scale2, nsdelta2);
                        float2 ds2 = fmul2(p2, d2);
                        if (kSel && select) {
                            const uint8_t c0 = keep[16 * c + k], c1 = keep[16 * c + k + 1];
                            if (c0 != 2) {
                                p2.x = (c0 == 1) ? p_masked : 0.f;
                                ds2.x = 0.f;
                            }
                            if (c1 != 2) {
                                p2.y = (c1 == 1) ? p_masked : 0.f;
                                ds2.y = 0.f;
                            }
                        }
                        const float2 db2 = fadd2(make_float2(dbias[16 * c + k],
                                                             dbias[16 * c + k + 1]), ds2);
                        dbias[16 * c + k] = db2.x;
                        dbias[16 * c + k + 1] = db2.y;
                        pk[k / 2] = E::pack(p2.x, p2.y);
                        dk[k / 2] = E::pack(ds2.x, ds2.y);
                    }
                    if (c == 0 && g > 0) {
                        // the previous step's partial-sum MMAs must be done reading P and dS
                        if (!mbar_wait(pds_empty, (g - 1) & 1, abort_flag)) {
                            return false;
                        }
                    }
                    // 16 columns = chunks 2c, 2c+1 of this warpgroup's panel row
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const uint32_t off = ((2 * c + q) ^ (r & 7)) << 4;
                        sts128(p_s + off, make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]));
                        sts128(ds_s + off, make_uint4(dk[4 * q], dk[4 * q + 1], dk[4 * q + 2], dk[4 * q + 3]));
                    }
                }
                return true;
                };
                const bool ok = __any_sync(0xffffffffu, select)
                                    ? ds_tile(std::integral_constant<bool, true>())
                                    : ds_tile(std::integral_constant<bool, false>());
                if (!ok) {
                    goto done;
                }
                tc_fence_before();
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(pds_full);
                    mbar_arrive(&kv_empty[s]);
                }
                if (g > 0 && !drain(g - 1, prev_b * p.H + prev_h, prev_i0, prev_j0)) {
                    goto done;
                }
                prev_b = b;
                prev_h = h;
                prev_i0 = i0;
                prev_j0 = j0;
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(bias_empty);
            }
            // dbias tile: row `row`, key columns [j0 + 64w, +64); the sums are of scale * dS
            if (row_ok) {
                const float inv_scale = 1.f / scale;
#pragma unroll
                for (int k = 0; k < 64; ++k) {
                    dbias[k] *= inv_scale;
                }
                float* dst = p.dbias + (static_cast<int64_t>(h) * p.Sq + row) * p.Sk + j0 + 64 * w;
                const int ncol = min(64, p.Sk - (j0 + 64 * w));
                if (p.dbias_atomic) {
#pragma unroll
                    for (int k = 0; k < 64; ++k) {
                        if (k < ncol) {
                            atomicAdd(dst + k, dbias[k]);
                        }
                    }
                } else if (ncol == 64 && (p.Sk & 3) == 0) {
#pragma unroll
                    for (int k = 0; k < 64; k += 4) {
                        *reinterpret_cast<float4*>(dst + k) =
                            make_float4(dbias[k], dbias[k + 1], dbias[k + 2], dbias[k + 3]);
                    }
                } else {
#pragma unroll
                    for (int k = 0; k < 64; ++k) {
                        if (k < ncol) {
                            dst[k] = dbias[k];
                        }
                    }
                }
            }
        }
        if (g > 0 && !drain(g - 1, prev_b * p.H + prev_h, prev_i0, prev_j0)) {
            goto done;
        }
        if (threadIdx.x == 0) {
            bulk_wait<0>(); // reductions complete before the CTA retires
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
    if (warp == C::kMmaWarp) {
        tmem_dealloc(tmem, C::kTmemCols);
    }
}

// delta[row] = sum_d dout[row, d] * out[row, d] (f32), one thread per row.
template <typename T, int D>
__global__ void attn_bwd_delta_kernel(const T* __restrict__ out, const T* __restrict__ dout,
                                      float* __restrict__ delta, int64_t rows) {
    using E = Elem<T>;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (row >= rows) {
        return;
    }
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < D / 8; ++c) {
        const uint4 a = ld_global_nc_v4(out + row * D + c * 8);
        const uint4 b = ld_global_nc_v4(dout + row * D + c * 8);
        const uint32_t wa[4] = {a.x, a.y, a.z, a.w};
        const uint32_t wb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 fa = E::to_float2(wa[e]);
            const float2 fb = E::to_float2(wb[e]);
            acc = fmaf(fa.x, fb.x, acc);
            acc = fmaf(fa.y, fb.y, acc);
        }
    }
    delta[row] = acc;
}

// dst[i] = (16-bit) src[i], 8 elements per thread.
template <typename T>
__global__ void f32_to_16_kernel(const float* __restrict__ src, T* __restrict__ dst, int64_t n8) {
    using E = Elem<T>;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float4 a = *reinterpret_cast<const float4*>(src + i * 8);
        const float4 b = *reinterpret_cast<const float4*>(src + i * 8 + 4);
        st_global_v4(dst + i * 8, make_uint4(E::pack(a.x, a.y), E::pack(a.z, a.w),
                                             E::pack(b.x, b.y), E::pack(b.z, b.w)));
    }
}

constexpr size_t align256(size_t x) {
    return (x + 255) & ~static_cast<size_t>(255);
}

struct BwdWorkspace {
    size_t dq_off, dk_off, dv_off, delta_off, total;
};

BwdWorkspace bwd_workspace(int64_t N, int64_t H, int64_t Sq, int64_t Sk, int64_t D) {
    BwdWorkspace w;
    const size_t eq = static_cast<size_t>(N * H * Sq * D) * 4;
    const size_t ekv = static_cast<size_t>(N * H * Sk * D) * 4;
    w.dq_off = 0;
    w.dk_off = align256(eq);
    w.dv_off = w.dk_off + align256(ekv);
    w.delta_off = w.dv_off + align256(ekv);
    w.total = w.delta_off + align256(static_cast<size_t>(N * H * Sq) * 4);
    return w;
}

template <typename T, int D, bool kBiasTma>
int launch_bwd(cudaStream_t st, const DeviceInfo& dev, const void* q, const void* k,
               const void* v, const void* bias, const uint8_t* kmask, const void* out,
               const float* lse, const void* dout, void* dq, void* dk, void* dv, float* dbias,
               uint8_t* ws, int N, int H, int Sq, int Sk, float scale, int phases) {
    using C = BwdCfg<D>;
    using G = Geo<D>;
    const BwdWorkspace wl = bwd_workspace(N, H, Sq, Sk, D);
    float* dq_acc = reinterpret_cast<float*>(ws + wl.dq_off);
    float* dk_acc = reinterpret_cast<float*>(ws + wl.dk_off);
    float* dv_acc = reinterpret_cast<float*>(ws + wl.dv_off);
    float* delta = reinterpret_cast<float*>(ws + wl.delta_off);

    const uint64_t nh = static_cast<uint64_t>(N) * H;
    const uint64_t row = 2ull * D;
    CUtensorMap tq, tk, tv, tdo, tb, tdq, tdk, tdv;
    CFK_TRY(make_tmap_3d(&tq, q, D, Sq, nh, row, row * Sq, D, kBM, 1, G::kSwizzleBytes, "bwd q"));
    CFK_TRY(make_tmap_3d(&tdo, dout, D, Sq, nh, row, row * Sq, D, kBM, 1, G::kSwizzleBytes,
                         "bwd dout"));
    CFK_TRY(make_tmap_3d(&tk, k, D, Sk, nh, row, row * Sk, D, kBN, 1, G::kSwizzleBytes, "bwd k"));
    CFK_TRY(make_tmap_3d(&tv, v, D, Sk, nh, row, row * Sk, D, kBN, 1, G::kSwizzleBytes, "bwd v"));
    if (kBiasTma) {
        CFK_TRY(make_tmap_3d(&tb, bias, Sk, Sq, H, 2ull * Sk, 2ull * Sk * Sq, 64, kBM, 1, 128,
                             "bwd bias"));
    } else {
        tb = tq;
    }
    const uint64_t frow = 4ull * D;
    CFK_TRY(make_tmap_3d(&tdq, dq_acc, D, Sq, nh, frow, frow * Sq, C::kPW, kBM, 1, C::kRowB,
                         "bwd dq acc", true));
    CFK_TRY(make_tmap_3d(&tdk, dk_acc, D, Sk, nh, frow, frow * Sk, C::kPW, kBN, 1, C::kRowB,
                         "bwd dk acc", true));
    CFK_TRY(make_tmap_3d(&tdv, dv_acc, D, Sk, nh, frow, frow * Sk, C::kPW, kBN, 1, C::kRowB,
                         "bwd dv acc", true));

    BwdParams p;
    p.kmask = kmask;
    p.bias = static_cast<const uint16_t*>(bias);
    p.lse = lse;
    p.delta = delta;
    p.dbias = dbias;
    p.N = N;
    p.H = H;
    p.Sq = Sq;
    p.Sk = Sk;
    p.n_it = (Sq + kBM - 1) / kBM;
    p.n_jt = (Sk + kBN - 1) / kBN;
    const int64_t base = static_cast<int64_t>(H) * p.n_it * p.n_jt;
    // batch chunks: as many as fit in one wave of CTAs, at least one
    int64_t nbc = base >= dev.num_sms ? 1 : std::max<int64_t>(1, dev.num_sms / base);
    nbc = std::min<int64_t>(nbc, N);
    p.bchunk = static_cast<int>((N + nbc - 1) / nbc);
    p.n_bc = static_cast<int>((N + p.bchunk - 1) / p.bchunk);
    p.items = base * p.n_bc;
    p.scale = scale;
    p.mask_bits = mask_bias_bits(scale);
    p.dbias_atomic = p.n_bc > 1 ? 1 : 0;

    const int64_t rows = static_cast<int64_t>(N) * H * Sq;
    if (phases & 1) {
        const size_t acc_bytes = wl.delta_off;
        if (cudaMemsetAsync(ws, 0, acc_bytes, st) != cudaSuccess ||
            (p.dbias_atomic &&
             cudaMemsetAsync(dbias, 0, static_cast<size_t>(H) * Sq * Sk * 4, st) != cudaSuccess)) {
            return fail(CFK_ERR_LAUNCH, "cfk_attn_bwd: memset failed");
        }
        attn_bwd_delta_kernel<T, D><<<static_cast<int>((rows + 255) / 256), 256, 0, st>>>(
            static_cast<const T*>(out), static_cast<const T*>(dout), delta, rows);
        CFK_TRY(check_launch("attn_bwd_delta"));
    }
    if (phases & 2) {
        auto kern = attn_bwd_kernel<T, D, kBiasTma>;
        CFK_TRY(ensure_smem_attr(reinterpret_cast<const void*>(kern), dev.device, C::kSmemBytes,
                                 "attn_bwd"));
        const int grid = static_cast<int>(std::min<int64_t>(p.items, dev.num_sms));
        kern<<<grid, C::kThreads, C::kSmemBytes, st>>>(tq, tk, tv, tdo, tb, tdq, tdk, tdv, p);
        CFK_TRY(check_launch("attn_bwd"));
    }
    if (!(phases & 4)) {
        return CFK_OK;
    }
    const int cgrid = dev.num_sms * 8;
    f32_to_16_kernel<T><<<cgrid, 256, 0, st>>>(dq_acc, static_cast<T*>(dq), rows * D / 8);
    const int64_t kv8 = static_cast<int64_t>(N) * H * Sk * D / 8;
    f32_to_16_kernel<T><<<cgrid, 256, 0, st>>>(dk_acc, static_cast<T*>(dk), kv8);
    f32_to_16_kernel<T><<<cgrid, 256, 0, st>>>(dv_acc, static_cast<T*>(dv), kv8);
    return check_launch("attn_bwd convert");
}

template <typename T>
int dispatch_bwd(cudaStream_t st, const DeviceInfo& dev, const void* q, const void* k,
                 const void* v, const void* bias, const uint8_t* kmask, const void* out,
                 const float* lse, const void* dout, void* dq, void* dk, void* dv, float* dbias,
                 uint8_t* ws, int N, int H, int Sq, int Sk, int D, float scale, int phases) {
    const bool bias_tma = (Sk % 8 == 0) && aligned16(bias);
#define CFK_BWD_D(DD)                                                                              \
    if (D == DD) {                                                                                 \
        return bias_tma ? launch_bwd<T, DD, true>(st, dev, q, k, v, bias, kmask, out, lse, dout,   \
                                                  dq, dk, dv, dbias, ws, N, H, Sq, Sk, scale,      \
                                                  phases)                                          \
                        : launch_bwd<T, DD, false>(st, dev, q, k, v, bias, kmask, out, lse, dout,  \
                                                   dq, dk, dv, dbias, ws, N, H, Sq, Sk, scale,     \
                                                   phases);                                        \
    }
    CFK_BWD_D(8)
    CFK_BWD_D(16)
    CFK_BWD_D(32)
    CFK_BWD_D(64)
#undef CFK_BWD_D
    return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_attn_bwd: head dim %d not in {8,16,32,64}", D);
}

} // namespace
} // namespace attn
} // namespace cfk

using namespace cfk;

extern "C" int cfk_attn_bwd_workspace_size(int64_t N, int64_t H, int64_t Sq, int64_t Sk,
                                           int64_t D, size_t* bytes) {
    clear_error();
    CFK_TRY(check_attn_args("cfk_attn_bwd_workspace_size", CFK_BF16, N, H, Sq, Sk, D));
    if (!bytes) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_attn_bwd_workspace_size: null pointer");
    }
    *bytes = attn::bwd_workspace(N, H, Sq, Sk, D).total;
    return CFK_OK;
}

namespace {

// Shared body of cfk_attn_bwd (phases = 7) and cfk_attn_bwd_phase (one bit).
int attn_bwd_entry(const char* fn, int phases, cfk_stream_t stream, cfk_dtype dtype,
                   const void* q, const void* k, const void* v, const void* bias,
                   const uint8_t* kmask, const void* out, const float* lse, const void* dout,
                   void* dq, void* dk, void* dv, float* dbias, void* workspace,
                   size_t workspace_bytes, int64_t N, int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                   float scale) {
    clear_error();
    CFK_TRY(check_attn_args(fn, dtype, N, H, Sq, Sk, D));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (H == 0 || Sq == 0 || Sk == 0 || N == 0) {
        // Empty: gradients are zero (dq for Sk == 0; dk, dv for Sq == 0; dbias always).
        if (!(phases & 4)) {
            return CFK_OK;
        }
        cudaError_t e = cudaSuccess;
        if (dbias && H * Sq * Sk > 0) {
            e = cudaMemsetAsync(dbias, 0, static_cast<size_t>(H * Sq * Sk) * 4, st);
        }
        if (e == cudaSuccess && dq && N * H * Sq * D > 0) {
            e = cudaMemsetAsync(dq, 0, static_cast<size_t>(N * H * Sq * D) * 2, st);
        }
        if (e == cudaSuccess && N * H * Sk * D > 0) {
            if (dk) {
                e = cudaMemsetAsync(dk, 0, static_cast<size_t>(N * H * Sk * D) * 2, st);
            }
            if (e == cudaSuccess && dv) {
                e = cudaMemsetAsync(dv, 0, static_cast<size_t>(N * H * Sk * D) * 2, st);
            }
        }
        return e == cudaSuccess ? CFK_OK : fail(CFK_ERR_LAUNCH, "%s: memset failed", fn);
    }
    if (!q || !k || !v || !bias || !kmask || !out || !lse || !dout || !dq || !dk || !dv ||
        !dbias) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: null buffer", fn);
    }
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || !aligned16(dout) ||
        !aligned16(dq) || !aligned16(dk) || !aligned16(dv)) {
        return fail(CFK_ERR_INVALID_ARGUMENT,
                    "%s: q, k, v, out, dout, dq, dk and dv must be 16-byte aligned", fn);
    }
    const size_t need = attn::bwd_workspace(N, H, Sq, Sk, D).total;
    if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255)) {
        return fail(CFK_ERR_INVALID_ARGUMENT,
                    "%s: workspace must be 256-byte aligned and hold %zu bytes (got %zu)", fn,
                    need, workspace_bytes);
    }
    DeviceInfo dev;
    CFK_TRY(current_device(&dev));
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const int n = static_cast<int>(N), h = static_cast<int>(H), sq = static_cast<int>(Sq),
              sk = static_cast<int>(Sk), d = static_cast<int>(D);
    return dtype == CFK_BF16
               ? attn::dispatch_bwd<__nv_bfloat16>(st, dev, q, k, v, bias, kmask, out, lse, dout,
                                                   dq, dk, dv, dbias, ws, n, h, sq, sk, d, scale,
                                                   phases)
               : attn::dispatch_bwd<__half>(st, dev, q, k, v, bias, kmask, out, lse, dout, dq, dk,
                                            dv, dbias, ws, n, h, sq, sk, d, scale, phases);
}

} // namespace

extern "C" int cfk_attn_bwd(cfk_stream_t stream, cfk_dtype dtype, const void* q, const void* k,
                            const void* v, const void* bias, const uint8_t* kmask,
                            const void* out, const float* lse, const void* dout, void* dq,
                            void* dk, void* dv, float* dbias, void* workspace,
                            size_t workspace_bytes, int64_t N, int64_t H, int64_t Sq, int64_t Sk,
                            int64_t D, float scale) {
    return attn_bwd_entry("cfk_attn_bwd", 7, stream, dtype, q, k, v, bias, kmask, out, lse, dout,
                          dq, dk, dv, dbias, workspace, workspace_bytes, N, H, Sq, Sk, D, scale);
}

extern "C" int cfk_attn_bwd_phase(int phase, cfk_stream_t stream, cfk_dtype dtype,
                                  const void* q, const void* k, const void* v, const void* bias,
                                  const uint8_t* kmask, const void* out, const float* lse,
                                  const void* dout, void* dq, void* dk, void* dv, float* dbias,
                                  void* workspace, size_t workspace_bytes, int64_t N, int64_t H,
                                  int64_t Sq, int64_t Sk, int64_t D, float scale) {
    if (phase < 0 || phase > 2) {
        clear_error();
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_attn_bwd_phase: phase %d not in {0,1,2}",
                    phase);
    }
    return attn_bwd_entry("cfk_attn_bwd_phase", 1 << phase, stream, dtype, q, k, v, bias, kmask,
                          out, lse, dout, dq, dk, dv, dbias, workspace, workspace_bytes, N, H, Sq,
                          Sk, D, scale);
}
