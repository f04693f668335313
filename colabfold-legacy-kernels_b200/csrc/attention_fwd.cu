// attention_fwd.cu -- flash attention forward with pair bias and key mask, tcgen05 + TMA.
//
// Semantics: cuda/volta_mma_attn.cu:139-271 (VoltaMma).  logit = scale * q.k + bias where the
// key is kept, -1e4 where kmask[n, j] == 0 (replaced, bias dropped); base-2 online softmax in
// f32; out = sum_j p_j v_j / sum_j p_j; the kernel also returns lse = m + ln(l) per row.
//
// Design (one persistent CTA per SM; work item = head h, 128-query tile, and NWG batch rows n
// that share the same bias tile):
//
//   warp NWG*4     TMA producer: q tiles per item; per 128-key tile and stage, the k and v
//                  tiles of every batch row, the bias tile [128 x 128] (shared by the NWG
//                  rows), and the key-mask operand described below.
//   warp NWG*4+1   MMA issuer (one thread): S_w = q_w k_w^T + ones * maskcol_w^T into tensor
//                  memory, then O_w = P_w v_w with P read from tensor memory.
//   warpgroup w    softmax of batch row w of the item: thread r owns query row r.  It loads
//                  its 128 scores from tensor memory, adds scale and bias, keeps the running
//                  max and sum, writes P (16-bit) back over the scores, and accumulates the
//                  O tile that the MMA writes in registers.
//
// Masked keys cost no per-score work in the common case: a second K=16 MMA adds
// ones[128 x 16] * maskcol^T, where maskcol[j, 0] = -big for a masked or out-of-range key and 0
// otherwise, so masked scores come out near -2^100 and vanish from max and sum.  That equals
// the reference's replacement by -1e4 whenever a row's running max exceeds -1e4 + 104, where
// exp(-1e4 - max) underflows in f32.  Rows that do not (all their keys masked, or pathological
// biases) take an exact select path that sets masked logits to -1e4 and out-of-range ones to
// -inf.
#include "attention_common.cuh"
#include "host.h"

namespace cfk {
namespace attn {
namespace {

template <int D>
struct FwdCfg {
    using G = Geo<D>;
    static constexpr int NWG = (D == 64) ? 1 : 2; // batch rows per item (bias reuse)
    static constexpr int NST = 2;                 // pipeline stages of k/v/bias
    static constexpr int kThreads = NWG * 128 + 64;
    static constexpr int kProducerWarp = NWG * 4;
    static constexpr int kMmaWarp = NWG * 4 + 1;
    static constexpr uint32_t kTmemCols = NWG == 2 ? 512 : 256; // S/P 128 + O Dp per group
    static constexpr int kSCol = 0;   // S/P of warpgroup w at w*256
    static constexpr int kOCol = 128; // O accumulator of warpgroup w at w*256 + 128

    static constexpr int kTile = ((G::kTileAlloc + 1023) / 1024) * 1024;
    static constexpr int kBiasBytes = 128 * 128 * 2;
    static constexpr int kMaskOpBytes = 128 * 16 * 2; // [128 x 16] bf16 interleave
    // stage: k_w, v_w, bias, maskcol_w
    static constexpr int kOffK = 0;
    static constexpr int kOffV = NWG * kTile;
    static constexpr int kOffBias = 2 * NWG * kTile;
    static constexpr int kOffMaskOp = kOffBias + kBiasBytes;
    static constexpr int kStageBytes = kOffMaskOp + NWG * kMaskOpBytes;
    static constexpr int kOffQ = 0;
    static constexpr int kOffStages = NWG * kTile;
    static constexpr int kOffOnes = kOffStages + NST * kStageBytes;
    static constexpr int kOffKeep = kOffOnes + kMaskOpBytes;          // u8 [NST][NWG][128]
    static constexpr int kOffFlag = kOffKeep + NST * NWG * 128;        // u32 [NST][NWG]
    static constexpr int kOffBar = ((kOffFlag + NST * NWG * 4 + 7) / 8) * 8;
    // barriers: q_full[NWG], q_empty[NWG], kv_full[NST], kv_empty[NST], s_full[NWG],
    // p_full[NWG], o_full[NWG]
    static constexpr int kNumBars = 5 * NWG + 2 * NST;
    static constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
    static constexpr int kOffAbort = kOffTmemSlot + 4;
    static constexpr int kSmemBytes = kOffAbort + 4 + 1024; // + alignment slack
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

    static constexpr uint32_t kStageTx = 2 * NWG * G::kTileBytes; // + bias when by TMA
};

struct FwdParams {
    const uint8_t* kmask;
    const uint16_t* bias; // raw pointer (used when the bias tile is not loaded by TMA)
    uint16_t* out;
    float* lse;
    int N, H, Sq, Sk;
    int n_qt, n_kt, n_groups;
    int64_t items;
    float scale;
    uint32_t mask_bits;   // bf16 bits of -big, or 0 when masked keys are excluded by select
};

template <typename T, int D, bool kBiasTma>
__global__ void __launch_bounds__(FwdCfg<D>::kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v,
                    const __grid_constant__ CUtensorMap tm_bias, const FwdParams p) {
    using C = FwdCfg<D>;
    using G = Geo<D>;
    using E = Elem<T>;
    constexpr int NWG = C::NWG;
    constexpr int NST = C::NST;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
    uint64_t* q_full = bars;
    uint64_t* q_empty = bars + NWG;
    uint64_t* kv_full = bars + 2 * NWG;
    uint64_t* kv_empty = bars + 2 * NWG + NST;
    uint64_t* s_full = bars + 2 * NWG + 2 * NST;
    uint64_t* p_full = s_full + NWG;
    uint64_t* o_full = p_full + NWG;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffTmemSlot);
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + C::kOffAbort);
    uint8_t* keep_all = smem + C::kOffKeep;
    uint32_t* flag_all = reinterpret_cast<uint32_t*>(smem + C::kOffFlag);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // ---- one-time set-up ----
    if (threadIdx.x == 0) {
        for (int w = 0; w < NWG; ++w) {
            mbar_init(&q_full[w], 1);
            mbar_init(&q_empty[w], 1);
            mbar_init(&s_full[w], 1);
            mbar_init(&p_full[w], 4);
            mbar_init(&o_full[w], 1);
        }
        for (int s = 0; s < NST; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1 + 4 * NWG);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    // ones[r, 0] = 1, all else 0 (bf16); maskcol operands: all 0 except column 0 (per tile).
    {
        uint32_t* ones = reinterpret_cast<uint32_t*>(smem + C::kOffOnes);
        for (int i = threadIdx.x; i < C::kMaskOpBytes / 4; i += blockDim.x) {
            // word i holds elements (r, c), (r, c + 1) with r = (i % 512) / 4, c = 8 * (i / 512)
            // + 2 * (i % 4)
            const bool first = (i < 512) && ((i & 3) == 0); // chunk 0, column 0
            ones[i] = first ? 0x3F80u : 0u;
        }
        for (int s = 0; s < NST; ++s) {
            uint32_t* mo = reinterpret_cast<uint32_t*>(smem + C::kOffStages + s * C::kStageBytes +
                                                       C::kOffMaskOp);
            for (int i = threadIdx.x; i < NWG * C::kMaskOpBytes / 4; i += blockDim.x) {
                mo[i] = 0u;
            }
        }
        if constexpr (D == 8) {
            // zero halves of the q / k / v tiles (the head dim is padded to 16)
            for (int t = 0; t < NWG; ++t) {
                uint32_t* z = reinterpret_cast<uint32_t*>(smem + C::kOffQ + t * C::kTile +
                                                          G::kTileBytes);
                for (int i = threadIdx.x; i < G::kTileBytes / 4; i += blockDim.x) {
                    z[i] = 0u;
                }
            }
            for (int s = 0; s < NST; ++s) {
                for (int t = 0; t < 2 * NWG; ++t) {
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
        if constexpr (kBiasTma) {
            tma_prefetch_desc(&tm_bias);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int n_items_mine =
        static_cast<int>((p.items - blockIdx.x + gridDim.x - 1) / gridDim.x);

    if (warp == C::kProducerWarp) {
        // =============================== TMA producer ===============================
        uint32_t g = 0;
        for (int it = 0; it < n_items_mine; ++it) {
            const int64_t item = blockIdx.x + static_cast<int64_t>(it) * gridDim.x;
            const int qt = static_cast<int>(item % p.n_qt);
            const int64_t rest = item / p.n_qt;
            const int h = static_cast<int>(rest % p.H);
            const int grp = static_cast<int>(rest / p.H);
            const int q0 = qt * kBM;
            for (int w = 0; w < NWG; ++w) {
                const int b = grp * NWG + w;
                if (it > 0 && !mbar_wait(&q_empty[w], (it - 1) & 1, abort_flag)) {
                    goto done;
                }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&q_full[w], G::kTileBytes);
                    tma_load_3d(smem + C::kOffQ + w * C::kTile, &tm_q, &q_full[w], 0, q0,
                                b * p.H + h);
                }
            }
            for (int t = 0; t < p.n_kt; ++t, ++g) {
                const int s = g % NST;
                if (g >= NST && !mbar_wait(&kv_empty[s], ((g / NST) - 1) & 1, abort_flag)) {
                    goto done;
                }
                uint8_t* stage = smem + C::kOffStages + s * C::kStageBytes;
                const int j0 = t * kBN;
                // key-mask operand and keep codes (0 out of range, 1 masked, 2 kept)
                for (int w = 0; w < NWG; ++w) {
                    const int b = grp * NWG + w;
                    uint16_t* mo = reinterpret_cast<uint16_t*>(stage + C::kOffMaskOp +
                                                               w * C::kMaskOpBytes);
                    uint8_t* keep = keep_all + (s * NWG + w) * 128;
                    bool any_excluded = false;
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const int jj = lane * 4 + r;
                        const int j = j0 + jj;
                        uint8_t code;
                        if (j >= p.Sk) {
                            code = 0;
                        } else if (b >= p.N) {
                            code = 2;
                        } else {
                            code = p.kmask[static_cast<int64_t>(b) * p.Sk + j] ? 2 : 1;
                        }
                        keep[jj] = code;
                        mo[jj * 8] = (code == 2 || p.mask_bits == 0) ? uint16_t(0)
                                                                     : uint16_t(p.mask_bits);
                        any_excluded |= (code != 2);
                    }
                    const uint32_t anyx = __any_sync(0xffffffffu, any_excluded);
                    if (lane == 0) {
                        flag_all[s * NWG + w] = anyx;
                    }
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive_expect_tx(&kv_full[s],
                                          C::kStageTx + (kBiasTma ? C::kBiasBytes : 0));
                    for (int w = 0; w < NWG; ++w) {
                        const int b = grp * NWG + w;
                        tma_load_3d(stage + C::kOffK + w * C::kTile, &tm_k, &kv_full[s], 0, j0,
                                    b * p.H + h);
                        tma_load_3d(stage + C::kOffV + w * C::kTile, &tm_v, &kv_full[s], 0, j0,
                                    b * p.H + h);
                    }
                    if constexpr (kBiasTma) {
                        tma_load_3d(stage + C::kOffBias, &tm_bias, &kv_full[s], j0, q0, h);
                        tma_load_3d(stage + C::kOffBias + 16384, &tm_bias, &kv_full[s], j0 + 64,
                                    q0, h);
                    }
                }
                __syncwarp();
            }
        }
    } else if (warp == C::kMmaWarp) {
        // =============================== MMA issuer ===============================
        if (lane == 0) {
            constexpr uint32_t kIdS = idesc_f16(128, 128, false, false, E::kBf16);
            constexpr uint32_t kIdMask = idesc_f16(128, 128, false, false, true);
            constexpr uint32_t kIdPV = idesc_f16(128, G::kDp, false, true, E::kBf16);
            const uint64_t ones_desc = interleave16_kmajor(sbase + C::kOffOnes);
            uint32_t g = 0;
            int sp = 0;
            for (int it = 0; it < n_items_mine; ++it) {
                for (int w = 0; w < NWG; ++w) {
                    if (!mbar_wait(&q_full[w], it & 1, abort_flag)) {
                        goto done;
                    }
                }
                for (int t = 0; t < p.n_kt; ++t, ++g) {
                    const int s = g % NST;
                    if (!mbar_wait(&kv_full[s], (g / NST) & 1, abort_flag)) {
                        goto done;
                    }
                    tc_fence_after();
                    const uint32_t stage = sbase + C::kOffStages + s * C::kStageBytes;
                    for (int w = 0; w < NWG; ++w) {
                        const uint32_t s_tm = tmem + w * 256 + C::kSCol;
                        const uint32_t o_tm = tmem + w * 256 + C::kOCol;
                        if (t > 0) {
                            if (!mbar_wait(&p_full[w], (g - 1) & 1, abort_flag)) {
                                goto done;
                            }
                            tc_fence_after();
                            const uint32_t vb = sbase + C::kOffStages + sp * C::kStageBytes +
                                                C::kOffV + w * C::kTile;
#pragma unroll
                            for (int ks = 0; ks < kBN / 16; ++ks) {
                                umma_ts(o_tm, s_tm + ks * 8, G::mnmajor(vb, ks), kIdPV,
                                        (t > 1 || ks > 0) ? 1u : 0u);
                            }
                            umma_commit(&o_full[w]);
                        }
                        const uint32_t qb = sbase + C::kOffQ + w * C::kTile;
                        const uint32_t kb = stage + C::kOffK + w * C::kTile;
#pragma unroll
                        for (int ks = 0; ks < G::kKSteps; ++ks) {
                            umma_ss(s_tm, G::kmajor(qb, ks), G::kmajor(kb, ks), kIdS, ks > 0);
                        }
                        umma_ss(s_tm, ones_desc,
                                interleave16_kmajor(stage + C::kOffMaskOp + w * C::kMaskOpBytes),
                                kIdMask, 1);
                        umma_commit(&s_full[w]);
                    }
                    if (t > 0) {
                        umma_commit(&kv_empty[sp]);
                    }
                    if (t == p.n_kt - 1) {
                        for (int w = 0; w < NWG; ++w) {
                            umma_commit(&q_empty[w]);
                        }
                    }
                    sp = s;
                }
                // P V of the item's last key tile
                for (int w = 0; w < NWG; ++w) {
                    if (!mbar_wait(&p_full[w], (g - 1) & 1, abort_flag)) {
                        goto done;
                    }
                    tc_fence_after();
                    const uint32_t s_tm = tmem + w * 256 + C::kSCol;
                    const uint32_t o_tm = tmem + w * 256 + C::kOCol;
                    const uint32_t vb =
                        sbase + C::kOffStages + sp * C::kStageBytes + C::kOffV + w * C::kTile;
#pragma unroll
                    for (int ks = 0; ks < kBN / 16; ++ks) {
                        umma_ts(o_tm, s_tm + ks * 8, G::mnmajor(vb, ks), kIdPV,
                                (p.n_kt > 1 || ks > 0) ? 1u : 0u);
                    }
                    umma_commit(&o_full[w]);
                }
                umma_commit(&kv_empty[sp]);
            }
        }
    } else {
        // =============================== softmax warpgroups ===============================
        const int w = warp >> 2;
        const int r = static_cast<int>(warp_lane_base()) + lane; // query row within the tile
        const uint32_t lane_off = warp_lane_base() << 16;
        const uint32_t s_tm = tmem + lane_off + w * 256 + C::kSCol;
        const uint32_t o_tm = tmem + lane_off + w * 256 + C::kOCol;
        const float scale = p.scale;
        const bool always_select = (p.mask_bits == 0);
        uint32_t g = 0;
        for (int it = 0; it < n_items_mine; ++it) {
            const int64_t item = blockIdx.x + static_cast<int64_t>(it) * gridDim.x;
            const int qt = static_cast<int>(item % p.n_qt);
            const int64_t rest = item / p.n_qt;
            const int h = static_cast<int>(rest % p.H);
            const int grp = static_cast<int>(rest / p.H);
            const int b = grp * NWG + w;
            const int row = qt * kBM + r;

            // m_run is the max that P is scaled by.  It is raised lazily, only when the tile max
            // exceeds it by more than ln(256) (P then stays <= 256), which makes the rescale of
            // O and l rare.
            float m_run = -INFINITY, l_run = 0.f;
            for (int t = 0; t < p.n_kt; ++t, ++g) {
                const int s = g % NST;
                if (!mbar_wait(&s_full[w], g & 1, abort_flag) ||
                    !mbar_wait(&kv_full[s], (g / NST) & 1, abort_flag)) {
                    goto done;
                }
                __syncwarp();
                tc_fence_after();
                float x[kBN];
#pragma unroll
                for (int c = 0; c < kBN / 32; ++c) {
                    uint32_t v[32];
                    tmem_ld32(s_tm + c * 32, v);
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        x[c * 32 + i] = __uint_as_float(v[i]);
                    }
                }
                tmem_ld_wait();
                // logit = scale * s + bias (natural-log units)
                if constexpr (kBiasTma) {
                    const uint32_t bias_s =
                        sbase + C::kOffStages + s * C::kStageBytes + C::kOffBias;
#pragma unroll
                    for (int c = 0; c < 16; ++c) {
                        const uint4 bw = lds128(bias_s + sw128_chunk(r, c));
                        const uint32_t wv[4] = {bw.x, bw.y, bw.z, bw.w};
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const float2 bf = E::to_float2(wv[q]);
                            x[c * 8 + 2 * q] = fmaf(x[c * 8 + 2 * q], scale, bf.x);
                            x[c * 8 + 2 * q + 1] = fmaf(x[c * 8 + 2 * q + 1], scale, bf.y);
                        }
                    }
                } else {
                    const int64_t brow =
                        (static_cast<int64_t>(h) * p.Sq + (row < p.Sq ? row : 0)) * p.Sk;
                    const int j0 = t * kBN;
#pragma unroll
                    for (int j = 0; j < kBN; ++j) {
                        const float bv = (j0 + j < p.Sk && row < p.Sq)
                                             ? E::to_float(p.bias[brow + j0 + j])
                                             : 0.f;
                        x[j] = fmaf(x[j], scale, bv);
                    }
                }
                float tmax = x[0];
#pragma unroll
                for (int j = 1; j < kBN; ++j) {
                    tmax = fmaxf(tmax, x[j]);
                }
                if (flag_all[s * NWG + w] != 0 &&
                    (always_select || fmaxf(m_run, tmax) < kMaskedLogit + 104.f)) {
                    // exact path: masked keys -> -1e4, out-of-range keys -> -inf
                    const uint8_t* keep = keep_all + (s * NWG + w) * 128;
#pragma unroll
                    for (int j = 0; j < kBN; ++j) {
                        const uint8_t code = keep[j];
                        x[j] = code == 2 ? x[j] : (code == 1 ? kMaskedLogit : -INFINITY);
                    }
                    tmax = x[0];
#pragma unroll
                    for (int j = 1; j < kBN; ++j) {
                        tmax = fmaxf(tmax, x[j]);
                    }
                }
                float alpha = 1.f;
                if (t == 0) {
                    m_run = tmax;
                } else if (tmax > m_run + 5.545177444479562f) { // ln(256)
                    alpha = ex2((m_run - tmax) * kLog2e);
                    m_run = tmax;
                }
                const float mL = (m_run == -INFINITY ? 0.f : m_run) * kLog2e;
                float rs = 0.f;
#pragma unroll
                for (int c = 0; c < kBN / 32; ++c) {
                    uint32_t pk[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float p0 = ex2(fmaf(x[c * 32 + 2 * i], kLog2e, -mL));
                        const float p1 = ex2(fmaf(x[c * 32 + 2 * i + 1], kLog2e, -mL));
                        rs += p0 + p1;
                        pk[i] = E::pack(p0, p1);
                    }
                    tmem_st16(s_tm + c * 16, pk);
                }
                l_run = l_run * alpha + rs;
                // Rescale the O accumulated so far (needs the previous P V to have landed).
                if (t > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
                    if (!mbar_wait(&o_full[w], (g - 1) & 1, abort_flag)) {
                        goto done;
                    }
                    __syncwarp();
                    tc_fence_after();
#pragma unroll
                    for (int c = 0; c < G::kDp / 16; ++c) {
                        uint32_t v[16];
                        tmem_ld16(o_tm + c * 16, v);
                        tmem_ld_wait();
#pragma unroll
                        for (int d = 0; d < 16; ++d) {
                            v[d] = __float_as_uint(__uint_as_float(v[d]) * alpha);
                        }
                        tmem_st16(o_tm + c * 16, v);
                    }
                }
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&p_full[w]);
                    mbar_arrive(&kv_empty[s]);
                }
            }
            // O after the item's last P V: normalise and store
            if (!mbar_wait(&o_full[w], (g - 1) & 1, abort_flag)) {
                goto done;
            }
            __syncwarp();
            tc_fence_after();
            {
                float o[G::kDp];
#pragma unroll
                for (int c = 0; c < G::kDp / 16; ++c) {
                    uint32_t v[16];
                    tmem_ld16(o_tm + c * 16, v);
#pragma unroll
                    for (int d = 0; d < 16; ++d) {
                        o[c * 16 + d] = __uint_as_float(v[d]);
                    }
                }
                tmem_ld_wait();
                const float inv = 1.0f / fmaxf(l_run, 1e-30f);
                if (b < p.N && row < p.Sq) {
                    const int64_t orow = (static_cast<int64_t>(b) * p.H + h) * p.Sq + row;
                    uint16_t* dst = p.out + orow * D;
#pragma unroll
                    for (int c = 0; c < D / 8; ++c) {
                        uint32_t wv[4];
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const int d = c * 8 + 2 * q;
                            wv[q] = E::pack(o[d] * inv, o[d + 1] * inv);
                        }
                        st_global_v4(dst + c * 8, make_uint4(wv[0], wv[1], wv[2], wv[3]));
                    }
                    if (p.lse) {
                        p.lse[orow] = (m_run == -INFINITY ? 0.f : m_run) + __logf(l_run);
                    }
                }
            }
        }
    }

done:
    __syncwarp();
    if (*abort_flag) {
        // Give copies and MMAs already in flight time to land before the CTA retires.
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

template <typename T, int D, bool kBiasTma>
int launch_fwd(cudaStream_t st, const DeviceInfo& dev, const void* q, const void* k,
               const void* v, const void* bias, const uint8_t* kmask, void* out, float* lse,
               int N, int H, int Sq, int Sk, float scale) {
    using C = FwdCfg<D>;
    using G = Geo<D>;
    CUtensorMap tq, tk, tv, tb;
    const uint64_t row = 2ull * D;
    CFK_TRY(make_tmap_3d(&tq, q, D, Sq, static_cast<uint64_t>(N) * H, row, row * Sq, D, kBM, 1,
                         G::kSwizzleBytes, "attn q"));
    CFK_TRY(make_tmap_3d(&tk, k, D, Sk, static_cast<uint64_t>(N) * H, row, row * Sk, D, kBN, 1,
                         G::kSwizzleBytes, "attn k"));
    CFK_TRY(make_tmap_3d(&tv, v, D, Sk, static_cast<uint64_t>(N) * H, row, row * Sk, D, kBN, 1,
                         G::kSwizzleBytes, "attn v"));
    if (kBiasTma) {
        CFK_TRY(make_tmap_3d(&tb, bias, Sk, Sq, H, 2ull * Sk, 2ull * Sk * Sq, 64, kBM, 1, 128,
                             "attn bias"));
    } else {
        tb = tq; // unused
    }
    FwdParams p;
    p.kmask = kmask;
    p.bias = static_cast<const uint16_t*>(bias);
    p.out = static_cast<uint16_t*>(out);
    p.lse = lse;
    p.N = N;
    p.H = H;
    p.Sq = Sq;
    p.Sk = Sk;
    p.n_qt = (Sq + kBM - 1) / kBM;
    p.n_kt = (Sk + kBN - 1) / kBN;
    p.n_groups = (N + C::NWG - 1) / C::NWG;
    p.items = static_cast<int64_t>(p.n_groups) * H * p.n_qt;
    p.scale = scale;
    p.mask_bits = mask_bias_bits(scale);
    auto kern = attn_fwd_kernel<T, D, kBiasTma>;
    CFK_TRY(ensure_smem_attr(reinterpret_cast<const void*>(kern), dev.device, C::kSmemBytes,
                             "attn_fwd"));
    const int grid = static_cast<int>(std::min<int64_t>(p.items, dev.num_sms));
    kern<<<grid, C::kThreads, C::kSmemBytes, st>>>(tq, tk, tv, tb, p);
    return check_launch("attn_fwd");
}

template <typename T>
int dispatch_fwd(cudaStream_t st, const DeviceInfo& dev, const void* q, const void* k,
                 const void* v, const void* bias, const uint8_t* kmask, void* out, float* lse,
                 int N, int H, int Sq, int Sk, int D, float scale) {
    const bool bias_tma = (Sk % 8 == 0) && aligned16(bias);
#define CFK_FWD_D(DD)                                                                              \
    if (D == DD) {                                                                                 \
        return bias_tma ? launch_fwd<T, DD, true>(st, dev, q, k, v, bias, kmask, out, lse, N, H,   \
                                                  Sq, Sk, scale)                                   \
                        : launch_fwd<T, DD, false>(st, dev, q, k, v, bias, kmask, out, lse, N, H,  \
                                                   Sq, Sk, scale);                                 \
    }
    CFK_FWD_D(8)
    CFK_FWD_D(16)
    CFK_FWD_D(32)
    CFK_FWD_D(64)
#undef CFK_FWD_D
    return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_attn_fwd: head dim %d not in {8,16,32,64}", D);
}

} // namespace
} // namespace attn
} // namespace cfk

namespace cfk {

int check_attn_args(const char* fn, int dtype, int64_t N, int64_t H, int64_t Sq, int64_t Sk,
                        int64_t D) {
    if (dtype != CFK_F16 && dtype != CFK_BF16) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: dtype must be CFK_F16 or CFK_BF16", fn);
    }
    if (N < 0 || H < 0 || Sq < 0 || Sk < 0) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: negative dimension", fn);
    }
    if (D != 8 && D != 16 && D != 32 && D != 64) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: head dim D=%lld not in {8,16,32,64}", fn,
                    static_cast<long long>(D));
    }
    const int64_t lim = (1ll << 31) - 1;
    if (N * H > lim || Sq > lim || Sk > lim || N * H * std::max(Sq, Sk) > (1ll << 40)) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: tensor too large", fn);
    }
    return CFK_OK;
}

} // namespace cfk

using namespace cfk;

extern "C" int cfk_attn_fwd(cfk_stream_t stream, cfk_dtype dtype, const void* q, const void* k,
                            const void* v, const void* bias, const uint8_t* kmask, void* out,
                            float* lse, int64_t N, int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                            float scale) {
    clear_error();
    CFK_TRY(check_attn_args("cfk_attn_fwd", dtype, N, H, Sq, Sk, D));
    if (N == 0 || H == 0 || Sq == 0) {
        return CFK_OK;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (Sk == 0) {
        // No keys: the reference's loop never runs and it writes 0 (volta_mma_attn.cu:139,265).
        if (!out) {
            return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_attn_fwd: null out");
        }
        cudaError_t e = cudaMemsetAsync(out, 0, static_cast<size_t>(N * H * Sq * D) * 2, st);
        if (e == cudaSuccess && lse) {
            // lse = -inf (0xff800000) for an empty row
            e = cudaMemsetAsync(lse, 0xff, static_cast<size_t>(N * H * Sq) * 4, st);
        }
        return e == cudaSuccess ? CFK_OK : fail(CFK_ERR_LAUNCH, "cfk_attn_fwd: memset failed");
    }
    if (!q || !k || !v || !bias || !kmask || !out) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_attn_fwd: null buffer");
    }
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) {
        return fail(CFK_ERR_INVALID_ARGUMENT,
                    "cfk_attn_fwd: q, k, v and out must be 16-byte aligned");
    }
    DeviceInfo dev;
    CFK_TRY(current_device(&dev));
    return dtype == CFK_BF16
               ? attn::dispatch_fwd<__nv_bfloat16>(st, dev, q, k, v, bias, kmask, out, lse,
                                                   static_cast<int>(N), static_cast<int>(H),
                                                   static_cast<int>(Sq), static_cast<int>(Sk),
                                                   static_cast<int>(D), scale)
               : attn::dispatch_fwd<__half>(st, dev, q, k, v, bias, kmask, out, lse,
                                            static_cast<int>(N), static_cast<int>(H),
                                            static_cast<int>(Sq), static_cast<int>(Sk),
                                            static_cast<int>(D), scale);
}
