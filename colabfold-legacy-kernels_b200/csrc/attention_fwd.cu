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
//                  memory, then O_w += P_w v_w per 64-key half, P read from tensor memory.
//   warpgroup w    softmax of batch row w of the item: thread r owns query row r.  It works
//                  on each 128-key tile in two 64-key halves: loads the half's scores from
//                  tensor memory, adds scale and bias, keeps the running max and sum, and
//                  writes that half's P (16-bit) to tensor memory, whose P V the MMA warp
//                  starts while the second half is computed.
//
// Batch rows per item: D = 64 runs one (NWG = 1).  D <= 32 runs three (NWG = 3, 448 threads)
// when there are enough items to fill the SMs, else two (NWG = 2, 320 threads; see
// rows_per_item): the softmax is latency bound at these head sizes, and a third warp per SM
// sub-partition hides more of it.
//
// Tensor memory with NWG = 3: 160 columns per warpgroup, S [128] | O [Dp], and P half h is
// written over S columns 32h..32h+31, which the softmax has already read.  The MMA warp
// therefore issues the last P V of tile g-1 before S of tile g: tcgen05.mma operations issued
// by one thread run in order, so that P V has read P before the S MMA overwrites those columns.
// With NWG <= 2: 256 columns per warpgroup, S [128] | P half 0 [32] | P half 1 [32] | O [Dp];
// there the MMA warp may write the next tile's S as soon as both halves of S are in registers.
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

template <int D, int NW>
struct FwdCfg {
    using G = Geo<D>;
    static constexpr int NWG = NW; // batch rows per item (bias reuse), one warpgroup each
    static_assert((D == 64 && NW == 1) || (D < 64 && (NW == 2 || NW == 3)), "rows per item");
    // three warpgroups: P is written over S columns already read (tensor memory budget)
    static constexpr bool kAlias = NWG == 3;
    static constexpr int NST = 2;                 // pipeline stages of k/v/bias
    static constexpr int kThreads = NWG * 128 + 64;
    static constexpr int kProducerWarp = NWG * 4;
    static constexpr int kMmaWarp = NWG * 4 + 1;
    static constexpr uint32_t kTmemCols = NWG == 1 ? 256 : 512;
    static constexpr int kWgCols = kAlias ? 160 : 256; // tensor-memory columns per warpgroup
    static constexpr int kSCol = 0;                  // S of warpgroup w at w*kWgCols
    static constexpr int kPCol = kAlias ? 0 : 128;   // P half h (16-bit pairs, 32 cols) at +32h
    static constexpr int kOCol = kAlias ? 128 : 192; // O accumulator (Dp columns)

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
    // barriers (index): q_full[w] 0.., q_empty[w], kv_full[s], kv_empty[s], s_full[w],
    // s_free[w], p_full[w][2], o_full[w][2]
    static constexpr int kBarQFull = 0;
    static constexpr int kBarQEmpty = NWG;
    static constexpr int kBarKvFull = 2 * NWG;
    static constexpr int kBarKvEmpty = 2 * NWG + NST;
    static constexpr int kBarSFull = 2 * NWG + 2 * NST;
    static constexpr int kBarSFree = kBarSFull + NWG;
    static constexpr int kBarPFull = kBarSFree + NWG;  // + 2w + h
    static constexpr int kBarOFull = kBarPFull + 2 * NWG; // + 2w + h
    static constexpr int kNumBars = kBarOFull + 2 * NWG;
    static constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
    static constexpr int kOffAbort = kOffTmemSlot + 4;
    static constexpr int kSmemBytes = kOffAbort + 4 + 1024; // + alignment slack
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
    static_assert(kOCol + G::kDp <= kWgCols && NWG * kWgCols <= int(kTmemCols),
                  "tensor memory budget");

    static constexpr uint32_t kStageTx = 2 * NWG * G::kTileBytes; // + bias when by TMA
};

struct FwdParams {
    const uint8_t* kmask;
    const uint16_t* bias; // raw pointer (used when the bias tile is not loaded by TMA)
    uint16_t* out;
    int64_t ob, oh, os; // element strides of out's batch, head and query axes
    float* lse;
    int N, H, Sq, Sk;
    int n_qt, n_kt, n_groups;
    int64_t items;
    float scale;
    uint32_t mask_bits;   // bf16 bits of -big, or 0 when masked keys are excluded by select
};

// (query tile, head, row group) of work item `item`, query tile fastest.  Item counts below
// 2^32 (every practical launch) take 32-bit divisions, which cost a fraction of 64-bit ones.
struct ItemCoords {
    int qt, h, grp;
};

__device__ __forceinline__ ItemCoords item_coords(const FwdParams& p, int64_t item) {
    ItemCoords c;
    if (p.items < (1ll << 32)) {
        const uint32_t i = static_cast<uint32_t>(item);
        const uint32_t rest = i / static_cast<uint32_t>(p.n_qt);
        c.qt = static_cast<int>(i - rest * static_cast<uint32_t>(p.n_qt));
        c.grp = static_cast<int>(rest / static_cast<uint32_t>(p.H));
        c.h = static_cast<int>(rest - static_cast<uint32_t>(c.grp) * static_cast<uint32_t>(p.H));
    } else {
        const int64_t rest = item / p.n_qt;
        c.qt = static_cast<int>(item - rest * p.n_qt);
        c.grp = static_cast<int>(rest / p.H);
        c.h = static_cast<int>(rest - static_cast<int64_t>(c.grp) * p.H);
    }
    return c;
}

template <typename T, int D, int NW, bool kBiasTma>
__global__ void __launch_bounds__(FwdCfg<D, NW>::kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v,
                    const __grid_constant__ CUtensorMap tm_bias, const FwdParams p) {
    using C = FwdCfg<D, NW>;
    using G = Geo<D>;
    using E = Elem<T>;
    constexpr int NWG = C::NWG;
    constexpr int NST = C::NST;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + C::kOffBar; // barrier i at bar0 + 8 i
    const uint32_t abort_s = sbase + C::kOffAbort;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffTmemSlot);
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + C::kOffAbort);
    uint8_t* keep_all = smem + C::kOffKeep;
    uint32_t* flag_all = reinterpret_cast<uint32_t*>(smem + C::kOffFlag);
    auto BAR = [bar0](int i) { return bar0 + 8u * static_cast<uint32_t>(i); };

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // ---- one-time set-up ----
    if (threadIdx.x == 0) {
        for (int w = 0; w < NWG; ++w) {
            mbar_init(&bars[C::kBarQFull + w], 1);
            mbar_init(&bars[C::kBarQEmpty + w], 1);
            mbar_init(&bars[C::kBarSFull + w], 1);
            mbar_init(&bars[C::kBarSFree + w], 4);
            for (int h = 0; h < 2; ++h) {
                mbar_init(&bars[C::kBarPFull + 2 * w + h], 4);
                mbar_init(&bars[C::kBarOFull + 2 * w + h], 1);
            }
        }
        for (int s = 0; s < NST; ++s) {
            mbar_init(&bars[C::kBarKvFull + s], 2); // TMA bytes + mask operand
            mbar_init(&bars[C::kBarKvEmpty + s], 1 + 4 * NWG);
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
            const ItemCoords ic = item_coords(p, blockIdx.x + static_cast<int64_t>(it) * gridDim.x);
            const int qt = ic.qt, h = ic.h, grp = ic.grp;
            const int q0 = qt * kBM;
            for (int w = 0; w < NWG; ++w) {
                const int b = grp * NWG + w;
                if (it > 0 && !mbar_wait_s(BAR(C::kBarQEmpty + w), (it - 1) & 1, abort_s)) {
                    goto done;
                }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&bars[C::kBarQFull + w], G::kTileBytes);
                    tma_load_4d(smem + C::kOffQ + w * C::kTile, &tm_q, &bars[C::kBarQFull + w], 0,
                                q0, h, b);
                }
            }
            for (int t = 0; t < p.n_kt; ++t, ++g) {
                const int s = g % NST;
                const int j0 = t * kBN;
                // keep codes of this lane's 4 keys per batch row (0 out of range, 1 masked,
                // 2 kept), read before waiting for the stage so the loads overlap the wait
                uint32_t codes[NWG];
#pragma unroll
                for (int w = 0; w < NWG; ++w) {
                    const int b = grp * NWG + w;
                    codes[w] = 0;
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const int j = j0 + lane * 4 + r;
                        uint32_t code;
                        if (j >= p.Sk) {
                            code = 0;
                        } else if (b >= p.N) {
                            code = 2;
                        } else {
                            code = p.kmask[static_cast<int64_t>(b) * p.Sk + j] ? 2 : 1;
                        }
                        codes[w] |= code << (8 * r);
                    }
                }
                if (g >= NST &&
                    !mbar_wait_s(BAR(C::kBarKvEmpty + s), ((g / NST) - 1) & 1, abort_s)) {
                    goto done;
                }
                uint8_t* stage = smem + C::kOffStages + s * C::kStageBytes;
                uint64_t* full = &bars[C::kBarKvFull + s];
                // the tiles first (first of the two arrivals), then the mask operand
                if (lane == 0) {
                    mbar_arrive_expect_tx(full, C::kStageTx + (kBiasTma ? C::kBiasBytes : 0));
                    for (int w = 0; w < NWG; ++w) {
                        const int b = grp * NWG + w;
                        tma_load_4d(stage + C::kOffK + w * C::kTile, &tm_k, full, 0, j0, h, b);
                        tma_load_4d(stage + C::kOffV + w * C::kTile, &tm_v, full, 0, j0, h, b);
                    }
                    if constexpr (kBiasTma) {
                        tma_load_3d(stage + C::kOffBias, &tm_bias, full, j0, q0, h);
                        tma_load_3d(stage + C::kOffBias + 16384, &tm_bias, full, j0 + 64, q0, h);
                    }
                }
#pragma unroll
                for (int w = 0; w < NWG; ++w) {
                    uint16_t* mo = reinterpret_cast<uint16_t*>(stage + C::kOffMaskOp +
                                                               w * C::kMaskOpBytes);
                    uint8_t* keep = keep_all + (s * NWG + w) * 128;
                    *reinterpret_cast<uint32_t*>(keep + lane * 4) = codes[w];
                    bool any_excluded = false;
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const uint32_t code = (codes[w] >> (8 * r)) & 0xFFu;
                        mo[(lane * 4 + r) * 8] = (code == 2 || p.mask_bits == 0)
                                                     ? uint16_t(0)
                                                     : uint16_t(p.mask_bits);
                        any_excluded |= (code != 2);
                    }
                    // bit h: the 64-key half h holds an excluded key
                    const uint32_t lo = __any_sync(0xffffffffu, any_excluded && lane < 16);
                    const uint32_t hi = __any_sync(0xffffffffu, any_excluded && lane >= 16);
                    if (lane == 0) {
                        flag_all[s * NWG + w] = (lo ? 1u : 0u) | (hi ? 2u : 0u);
                    }
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(full); // second arrival: mask operand and flags written
                }
            }
        }
    } else if (warp == C::kMmaWarp) {
        // =============================== MMA issuer ===============================
        if (lane == 0) {
            constexpr uint32_t kIdS = idesc_f16(128, 128, false, false, E::kBf16);
            constexpr uint32_t kIdMask = idesc_f16(128, 128, false, false, true);
            constexpr uint32_t kIdPV = idesc_f16(128, G::kDp, false, true, E::kBf16);
            const uint64_t ones_desc = interleave16_kmajor(sbase + C::kOffOnes);
            // P V of half `hf` of global tile gp for warpgroup w (V from stage gp % NST);
            // `first`: tile gp is the first of its item, so half 0 overwrites O
            auto issue_pv = [&](int w, uint32_t gp, int hf, bool first) -> bool {
                if (!mbar_wait_s(BAR(C::kBarPFull + 2 * w + hf), gp & 1, abort_s)) {
                    return false;
                }
                tc_fence_after();
                const uint32_t vb = sbase + C::kOffStages + (gp % NST) * C::kStageBytes +
                                    C::kOffV + w * C::kTile;
                const uint32_t p_tm = tmem + w * C::kWgCols + C::kPCol + 32 * hf;
                const uint32_t o_tm = tmem + w * C::kWgCols + C::kOCol;
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    umma_ts(o_tm, p_tm + ks * 8, G::mnmajor(vb, 4 * hf + ks), kIdPV,
                            (!first || hf > 0 || ks > 0) ? 1u : 0u);
                }
                umma_commit(&bars[C::kBarOFull + 2 * w + hf]);
                return true;
            };
            // One flat sequence over the tiles of all items: S(g) once the softmax has read
            // S(g-1), then P V of the second half of tile g-1, then of the first half of g.
            uint32_t g = 0;
            bool prev_first = false; // tile g - 1 was the first tile of its item
            bool pend = false;       // P V of half 1 of tile g - 1 (and its stage) outstanding
            for (int it = 0; it < n_items_mine; ++it) {
                if (pend) {
                    // The previous item's last P V goes now, not after the next item's q tiles
                    // arrive: its softmax warpgroups wait for it to normalise and store O.
                    for (int w = 0; w < NWG; ++w) {
                        if (!issue_pv(w, g - 1, 1, prev_first)) {
                            goto done;
                        }
                    }
                    umma_commit(&bars[C::kBarKvEmpty + (g - 1) % NST]);
                    pend = false;
                }
                for (int w = 0; w < NWG; ++w) {
                    if (!mbar_wait_s(BAR(C::kBarQFull + w), it & 1, abort_s)) {
                        goto done;
                    }
                }
                for (int t = 0; t < p.n_kt; ++t, ++g) {
                    const int s = g % NST;
                    if (!mbar_wait_s(BAR(C::kBarKvFull + s), (g / NST) & 1, abort_s)) {
                        goto done;
                    }
                    tc_fence_after();
                    const uint32_t stage = sbase + C::kOffStages + s * C::kStageBytes;
                    for (int w = 0; w < NWG; ++w) {
                        if constexpr (C::kAlias) {
                            // S(g) overwrites P(g-1): its last P V goes first (in-order pipe)
                            if (pend && !issue_pv(w, g - 1, 1, prev_first)) {
                                goto done;
                            }
                        } else if (g > 0 &&
                                   !mbar_wait_s(BAR(C::kBarSFree + w), (g - 1) & 1, abort_s)) {
                            goto done;
                        }
                        tc_fence_after();
                        const uint32_t s_tm = tmem + w * C::kWgCols + C::kSCol;
                        const uint32_t qb = sbase + C::kOffQ + w * C::kTile;
                        const uint32_t kb = stage + C::kOffK + w * C::kTile;
#pragma unroll
                        for (int ks = 0; ks < G::kKSteps; ++ks) {
                            umma_ss(s_tm, G::kmajor(qb, ks), G::kmajor(kb, ks), kIdS, ks > 0);
                        }
                        umma_ss(s_tm, ones_desc,
                                interleave16_kmajor(stage + C::kOffMaskOp + w * C::kMaskOpBytes),
                                kIdMask, 1);
                        umma_commit(&bars[C::kBarSFull + w]);
                    }
                    if (t == p.n_kt - 1) {
                        for (int w = 0; w < NWG; ++w) {
                            umma_commit(&bars[C::kBarQEmpty + w]);
                        }
                    }
                    if (pend) {
                        if constexpr (!C::kAlias) {
                            for (int w = 0; w < NWG; ++w) {
                                if (!issue_pv(w, g - 1, 1, prev_first)) {
                                    goto done;
                                }
                            }
                        }
                        umma_commit(&bars[C::kBarKvEmpty + (g - 1) % NST]);
                    }
                    for (int w = 0; w < NWG; ++w) {
                        if (!issue_pv(w, g, 0, t == 0)) {
                            goto done;
                        }
                    }
                    prev_first = (t == 0);
                    pend = true;
                }
            }
            if (pend) {
                for (int w = 0; w < NWG; ++w) {
                    if (!issue_pv(w, g - 1, 1, prev_first)) {
                        goto done;
                    }
                }
                umma_commit(&bars[C::kBarKvEmpty + (g - 1) % NST]);
            }
        }
    } else {
        // =============================== softmax warpgroups ===============================
        const int w = warp >> 2;
        const int r = static_cast<int>(warp_lane_base()) + lane; // query row within the tile
        const uint32_t lane_off = warp_lane_base() << 16;
        const uint32_t s_tm = tmem + lane_off + w * C::kWgCols + C::kSCol;
        const uint32_t p_tm = tmem + lane_off + w * C::kWgCols + C::kPCol;
        const uint32_t o_tm = tmem + lane_off + w * C::kWgCols + C::kOCol;
        const uint32_t flag_s = sbase + C::kOffFlag;
        const float scale = p.scale;
        const float2 scale2 = make_float2(scale, scale);
        const float2 log2e2 = make_float2(kLog2e, kLog2e);
        const bool always_select = (p.mask_bits == 0);
        uint32_t g = 0;
        for (int it = 0; it < n_items_mine; ++it) {
            const ItemCoords ic = item_coords(p, blockIdx.x + static_cast<int64_t>(it) * gridDim.x);
            const int qt = ic.qt, h = ic.h, grp = ic.grp;
            const int b = grp * NWG + w;
            const int row = qt * kBM + r;

            // m_run is the max that P is scaled by.  It is raised lazily, only when a half-tile
            // max exceeds it by more than ln(256) (P then stays <= 256), which makes the rescale
            // of O and l rare.
            float m_run = -INFINITY, l_run = 0.f;
            for (int t = 0; t < p.n_kt; ++t, ++g) {
                const int s = g % NST;
                if (!mbar_wait_s(BAR(C::kBarSFull + w), g & 1, abort_s) ||
                    !mbar_wait_s(BAR(C::kBarKvFull + s), (g / NST) & 1, abort_s)) {
                    goto done;
                }
                __syncwarp();
                tc_fence_after();
                const uint32_t flags = ld_shared_u32(flag_s + 4 * (s * NWG + w));
#pragma unroll 1
                for (int hf = 0; hf < 2; ++hf) {
                    float x[64];
                    {
                        uint32_t v[32];
                        tmem_ld32(s_tm + 64 * hf, v);
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            x[i] = __uint_as_float(v[i]);
                        }
                        tmem_ld32(s_tm + 64 * hf + 32, v);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            x[32 + i] = __uint_as_float(v[i]);
                        }
                    }
                    if (!C::kAlias && hf == 1) {
                        // all of S is in registers: the MMA may write the next tile's S
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) {
                            mbar_arrive_s(BAR(C::kBarSFree + w));
                        }
                    }
                    // logit = scale * s + bias (natural-log units)
                    if constexpr (kBiasTma) {
                        const uint32_t bias_s = sbase + C::kOffStages + s * C::kStageBytes +
                                                C::kOffBias + hf * 16384 + r * 128;
#pragma unroll
                        for (int c = 0; c < 8; ++c) {
                            const uint4 bw = lds128(bias_s + ((c ^ (r & 7)) << 4));
                            const uint32_t wv[4] = {bw.x, bw.y, bw.z, bw.w};
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                const float2 t2 =
                                    ffma2(make_float2(x[c * 8 + 2 * q], x[c * 8 + 2 * q + 1]),
                                          scale2, E::to_float2(wv[q]));
                                x[c * 8 + 2 * q] = t2.x;
                                x[c * 8 + 2 * q + 1] = t2.y;
                            }
                        }
                    } else {
                        const int64_t brow =
                            (static_cast<int64_t>(h) * p.Sq + (row < p.Sq ? row : 0)) * p.Sk;
                        const int j0 = t * kBN + 64 * hf;
#pragma unroll
                        for (int j = 0; j < 64; ++j) {
                            const float bv = (j0 + j < p.Sk && row < p.Sq)
                                                 ? E::to_float(p.bias[brow + j0 + j])
                                                 : 0.f;
                            x[j] = fmaf(x[j], scale, bv);
                        }
                    }
                    // four independent max chains (short dependency latency)
                    float mx[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        mx[u] = fmax3(x[16 * u], x[16 * u + 1], x[16 * u + 2]);
#pragma unroll
                        for (int j = 3; j < 15; j += 2) {
                            mx[u] = fmax3(mx[u], x[16 * u + j], x[16 * u + j + 1]);
                        }
                        mx[u] = fmaxf(mx[u], x[16 * u + 15]);
                    }
                    float tmax = fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]);
                    if ((flags >> hf & 1u) &&
                        (always_select || fmaxf(m_run, tmax) < kMaskedLogit + 104.f)) {
                        // exact path: masked keys -> -1e4, out-of-range keys -> -inf
                        const uint8_t* keep = keep_all + (s * NWG + w) * 128 + 64 * hf;
#pragma unroll
                        for (int j = 0; j < 64; ++j) {
                            const uint8_t code = keep[j];
                            x[j] = code == 2 ? x[j] : (code == 1 ? kMaskedLogit : -INFINITY);
                        }
                        tmax = x[0];
#pragma unroll
                        for (int j = 1; j < 64; ++j) {
                            tmax = fmaxf(tmax, x[j]);
                        }
                    }
                    const bool first_half = (t == 0 && hf == 0);
                    float alpha = 1.f;
                    if (first_half) {
                        m_run = tmax;
                    } else if (tmax > m_run + 5.545177444479562f) { // ln(256)
                        alpha = ex2((m_run - tmax) * kLog2e);
                        m_run = tmax;
                    }
                    // This half's P columns are free once the previous tile's P V of the same
                    // half is done; a rescale of O needs every earlier P V done (the latest is
                    // half 1 of the previous tile, or half 0 of this tile).
                    if (t > 0 && !mbar_wait_s(BAR(C::kBarOFull + 2 * w + hf), (g - 1) & 1,
                                              abort_s)) {
                        goto done;
                    }
                    const bool rescale = __any_sync(0xffffffffu, alpha != 1.f);
                    if (rescale) {
                        const bool ok =
                            hf == 1 ? mbar_wait_s(BAR(C::kBarOFull + 2 * w), g & 1, abort_s)
                                    : mbar_wait_s(BAR(C::kBarOFull + 2 * w + 1), (g - 1) & 1,
                                                  abort_s);
                        if (!ok) {
                            goto done;
                        }
                    }
                    __syncwarp();
                    tc_fence_after();
                    if (rescale) {
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
                    const float mL = (m_run == -INFINITY ? 0.f : m_run) * kLog2e;
                    const float2 nmL2 = make_float2(-mL, -mL);
                    float2 rs2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        uint32_t pk[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const int j = c * 32 + 2 * i;
                            const float2 a = ffma2(make_float2(x[j], x[j + 1]), log2e2, nmL2);
                            const float2 e = make_float2(ex2(a.x), ex2(a.y));
                            rs2[i & 1] = fadd2(rs2[i & 1], e);
                            pk[i] = E::pack(e.x, e.y);
                        }
                        tmem_st16(p_tm + 32 * hf + c * 16, pk);
                    }
                    l_run = l_run * alpha + ((rs2[0].x + rs2[0].y) + (rs2[1].x + rs2[1].y));
                    tmem_st_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive_s(BAR(C::kBarPFull + 2 * w + hf));
                        if (hf == 1) {
                            mbar_arrive_s(BAR(C::kBarKvEmpty + s));
                        }
                    }
                }
            }
            // O after the item's last P V (half 1 of its last tile): normalise and store
            if (!mbar_wait_s(BAR(C::kBarOFull + 2 * w + 1), (g - 1) & 1, abort_s)) {
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
                    uint16_t* dst = p.out + b * p.ob + h * p.oh + row * p.os;
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

template <typename T, int D, int NW, bool kBiasTma>
int launch_fwd(cudaStream_t st, const DeviceInfo& dev, const void* q, const void* k,
               const void* v, const void* bias, const uint8_t* kmask, void* out, float* lse,
               int N, int H, int Sq, int Sk, float scale, const RowView* views) {
    using C = FwdCfg<D, NW>;
    using G = Geo<D>;
    CUtensorMap tq, tk, tv, tb;
    CFK_TRY(make_tmap_rows(&tq, q, views[0], D, kBM, G::kSwizzleBytes, "attn q"));
    CFK_TRY(make_tmap_rows(&tk, k, views[1], D, kBN, G::kSwizzleBytes, "attn k"));
    CFK_TRY(make_tmap_rows(&tv, v, views[2], D, kBN, G::kSwizzleBytes, "attn v"));
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
    p.ob = views[3].b;
    p.oh = views[3].h;
    p.os = views[3].s;
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
    auto kern = attn_fwd_kernel<T, D, NW, kBiasTma>;
    CFK_TRY(ensure_smem_attr(reinterpret_cast<const void*>(kern), dev.device, C::kSmemBytes,
                             "attn_fwd"));
    const int grid = static_cast<int>(std::min<int64_t>(p.items, dev.num_sms));
    kern<<<grid, C::kThreads, C::kSmemBytes, st>>>(tq, tk, tv, tb, p);
    return check_launch("attn_fwd");
}

// Batch rows per work item for D <= 32.  Three warpgroups run a row about 2 % faster than two
// (measured at tri-768), but an item then holds more rows, so with few items per SM the last
// wave of items leaves more SMs idle.  Pick the smaller estimate of waves x rows x cost.
int rows_per_item(int N, int H, int Sq, int num_sms) {
    const auto cost = [&](int nw, double per_row) {
        const int64_t items = static_cast<int64_t>((N + nw - 1) / nw) * H * ((Sq + kBM - 1) / kBM);
        const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(items, num_sms));
        return static_cast<double>((items + grid - 1) / grid) * nw * per_row;
    };
    return cost(3, 0.982) < cost(2, 1.0) ? 3 : 2;
}

template <typename T>
int dispatch_fwd(cudaStream_t st, const DeviceInfo& dev, const void* q, const void* k,
                 const void* v, const void* bias, const uint8_t* kmask, void* out, float* lse,
                 int N, int H, int Sq, int Sk, int D, float scale, const RowView* views) {
    const bool bias_tma = (Sk % 8 == 0) && aligned16(bias);
    const int nw = D == 64 ? 1 : rows_per_item(N, H, Sq, dev.num_sms);
#define CFK_FWD_L(DD, NN)                                                                          \
    return bias_tma ? launch_fwd<T, DD, NN, true>(st, dev, q, k, v, bias, kmask, out, lse, N, H,   \
                                                  Sq, Sk, scale, views)                            \
                    : launch_fwd<T, DD, NN, false>(st, dev, q, k, v, bias, kmask, out, lse, N, H,  \
                                                   Sq, Sk, scale, views);
#define CFK_FWD_D(DD)                                                                              \
    if (D == DD) {                                                                                 \
        if (nw == 3) {                                                                             \
            CFK_FWD_L(DD, 3)                                                                       \
        }                                                                                          \
        CFK_FWD_L(DD, 2)                                                                           \
    }
    CFK_FWD_D(8)
    CFK_FWD_D(16)
    CFK_FWD_D(32)
    if (D == 64) {
        CFK_FWD_L(64, 1)
    }
#undef CFK_FWD_D
#undef CFK_FWD_L
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

namespace {

int attn_fwd_entry(const char* fn, cfk_stream_t stream, cfk_dtype dtype, const void* q,
                   const void* k, const void* v, const void* bias, const uint8_t* kmask,
                   void* out, float* lse, int64_t N, int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                   float scale, const cfk_view* user_views) {
    clear_error();
    CFK_TRY(check_attn_args(fn, dtype, N, H, Sq, Sk, D));
    static const char* const names[4] = {"q", "k", "v", "out"};
    RowView views[4];
    for (int t = 0; t < 4; ++t) {
        const int64_t S = (t == 1 || t == 2) ? Sk : Sq;
        CFK_TRY(view_of(fn, names[t], user_views ? &user_views[t] : nullptr, N, H, S, D,
                        &views[t]));
    }
    if (N == 0 || H == 0 || Sq == 0) {
        return CFK_OK;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (Sk == 0) {
        // No keys: the reference's loop never runs and it writes 0 (volta_mma_attn.cu:139,265).
        if (!out || !aligned16(out)) {
            return fail(CFK_ERR_INVALID_ARGUMENT, "%s: out must be non-null and 16-byte aligned",
                        fn);
        }
        cudaError_t e = cudaSuccess;
        if (is_packed(views[3], D)) {
            e = cudaMemsetAsync(out, 0, static_cast<size_t>(N * H * Sq * D) * 2, st);
        } else {
            DeviceInfo dev;
            CFK_TRY(current_device(&dev));
            const attn::ConvertJob job{{nullptr, nullptr, nullptr},
                                       {out, out, out},
                                       {N * H * Sq * D / 8, 0, 0},
                                       {attn::row_strides(views[3], D),
                                        attn::row_strides(views[3], D),
                                        attn::row_strides(views[3], D)},
                                       {1.f, 1.f, 1.f},
                                       {0, 0, 0},
                                       attn::d8_log2(static_cast<int>(D))};
            attn::f32_to_16_kernel<__half><<<dev.num_sms * 8, 256, 0, st>>>(job);
            CFK_TRY(check_launch("attn_fwd zero"));
        }
        if (e == cudaSuccess && lse) {
            // lse = -inf (0xff800000) for an empty row
            e = cudaMemsetAsync(lse, 0xff, static_cast<size_t>(N * H * Sq) * 4, st);
        }
        return e == cudaSuccess ? CFK_OK : fail(CFK_ERR_LAUNCH, "%s: memset failed", fn);
    }
    if (!q || !k || !v || !bias || !kmask || !out) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: null buffer", fn);
    }
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: q, k, v and out must be 16-byte aligned", fn);
    }
    DeviceInfo dev;
    CFK_TRY(current_device(&dev));
    return dtype == CFK_BF16
               ? attn::dispatch_fwd<__nv_bfloat16>(st, dev, q, k, v, bias, kmask, out, lse,
                                                   static_cast<int>(N), static_cast<int>(H),
                                                   static_cast<int>(Sq), static_cast<int>(Sk),
                                                   static_cast<int>(D), scale, views)
               : attn::dispatch_fwd<__half>(st, dev, q, k, v, bias, kmask, out, lse,
                                            static_cast<int>(N), static_cast<int>(H),
                                            static_cast<int>(Sq), static_cast<int>(Sk),
                                            static_cast<int>(D), scale, views);
}

} // namespace

extern "C" int cfk_attn_fwd(cfk_stream_t stream, cfk_dtype dtype, const void* q, const void* k,
                            const void* v, const void* bias, const uint8_t* kmask, void* out,
                            float* lse, int64_t N, int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                            float scale) {
    return attn_fwd_entry("cfk_attn_fwd", stream, dtype, q, k, v, bias, kmask, out, lse, N, H,
                          Sq, Sk, D, scale, nullptr);
}

extern "C" int cfk_attn_fwd_strided(cfk_stream_t stream, cfk_dtype dtype, const void* q,
                                    const void* k, const void* v, const void* bias,
                                    const uint8_t* kmask, void* out, float* lse, int64_t N,
                                    int64_t H, int64_t Sq, int64_t Sk, int64_t D, float scale,
                                    const cfk_view* views) {
    return attn_fwd_entry("cfk_attn_fwd_strided", stream, dtype, q, k, v, bias, kmask, out, lse,
                          N, H, Sq, Sk, D, scale, views);
}
