// attention_bwd.cu -- backward of attention with pair bias and key mask, tcgen05 + TMA.
//
// The reference is forward-only; this is the exact derivative of cuda/volta_mma_attn.cu:139-271
// (masked logits are constants -1e4, so they pass no gradient):
//
//   P = exp(logit - lse)        dV = P^T dO        dP = dO V^T        delta_i = sum_d dO O
//   dS = P * (dP - delta)       dQ = scale dS K    dK = scale dS^T Q  dbias = sum_n dS
//
// dbias sums over the batch rows n, so a work item keeps its (query tile, key tile) fixed and
// walks the batch rows: its 128 x 128 dbias tile lives in registers for the whole walk and is
// written once (no atomics when the item covers every row, a deterministic result).  dQ, dK
// and dV of one batch row are then partial sums over key tiles (dQ) or query tiles (dK, dV);
// the MMA writes those partials into tensor memory and a TMA tensor reduce-add folds them into
// f32 accumulators in the workspace.  A final kernel converts the accumulators to 16 bits.
//
// The scores are computed transposed, S^T = K Q^T and dP^T = V dO^T, so that a thread owns one
// key row j of the tile: the key mask is then a per-thread constant, and the thread writes
// P^T and dS^T rows straight into tensor memory, where they are the A operands of dV = P^T dO
// and dK = dS^T Q (tcgen05.mma with A in tensor memory).  dQ = dS K reads dS from shared memory
// (the same rows, taken as an MN-major operand).
//
//   warps 0-15  dS warps: warp w4 + 4w owns key rows [32 w4, +32) (its tensor-memory lane
//               quarter) and query columns [32w, +32) of warpgroup w.  Warpgroups 0-2 also
//               drain the dV, dK and dQ partials.
//   warp 16     TMA producer: per batch row q, dO, k, v tiles and the row statistics
//               (-lse log2 e, -scale delta) of the query tile.
//   warp 17     MMA issuer.
#include <type_traits>

#include "attention_common.cuh"
#include "host.h"

namespace cfk {
namespace attn {
namespace {

template <int D>
struct BwdCfg {
    using G = Geo<D>;
    // D = 64: P^T and dS^T overwrite S^T and dP^T in tensor memory (the partial-sum buffers
    // need the room); the next batch row's S^T waits for the partial-sum MMAs.
    static constexpr bool kInPlace = (D == 64);
    static constexpr int NST = (D == 64) ? 1 : 3; // operand stages
    static constexpr int kDsWarps = 16;
    static constexpr int kThreads = (kDsWarps + 2) * 32;
    static constexpr int kProducerWarp = 16;
    static constexpr int kMmaWarp = 17;
    static constexpr uint32_t kTmemCols = 512;
    static constexpr int kSCol = 0;
    static constexpr int kDPCol = 128;
    // P^T / dS^T as packed 16-bit pairs: warpgroup w's 32 query columns at col + kPStride * w
    static constexpr int kPCol = kInPlace ? kSCol : 256;
    static constexpr int kDSCol = kInPlace ? kDPCol : 320;
    static constexpr int kPStride = kInPlace ? 32 : 16;
    static constexpr int kPartBase = kInPlace ? 256 : 384; // buffer pb: dV, dK, dQ
    static constexpr int NPB = (kPartBase + 6 * G::kDp <= 512) ? 2 : 1;

    static constexpr int kTile = ((G::kTileAlloc + 1023) / 1024) * 1024;
    static constexpr int kOffSQ = 0;
    static constexpr int kOffSdO = kTile;
    static constexpr int kOffSK = 2 * kTile;
    static constexpr int kOffSV = 3 * kTile;
    static constexpr int kOffRS = 4 * kTile; // f32 [2][128]: -lse*log2(e), -scale*delta
    static constexpr int kStageBytes = 4 * kTile + 1024;

    // f32 staging of one [128 x D] partial for the TMA reduce: panels of kPW floats per row
    static constexpr int kPW = D < 32 ? D : 32;
    static constexpr int kRowB = kPW * 4; // bytes of one staging row (= swizzle span)
    static constexpr int kPanelBytes = 128 * kRowB;
    static constexpr int kStgBytes = 128 * D * 4;

    static constexpr int kOffStages = 0;
    static constexpr int kOffDS = NST * kStageBytes; // dS^T rows, MN-major operand of dQ
    static constexpr int kOffBiasT = kOffDS + 32768; // bias^T: row j = 128 queries, 16-bit
    static constexpr int kOffStg = kOffBiasT + 32768;
    static constexpr int kOffBar = kOffStg + 3 * kStgBytes;
    // kv_full[NST], kv_empty[NST], sdp_full, sdp_free, pds_full, pds_empty, part_full[NPB],
    // part_empty[NPB]
    static constexpr int kNumBars = 2 * NST + 4 + 2 * NPB;
    static constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
    static constexpr int kOffAbort = kOffTmemSlot + 4;
    static constexpr int kSmemBytes = kOffAbort + 4 + 1024;
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
    static_assert(kPartBase + NPB * 3 * G::kDp <= 512, "tensor memory budget");
};

struct BwdParams {
    const uint8_t* kmask;
    const uint16_t* bias;
    const float* rowstat; // [N*H][n_it][2][128]
    float* dbias;
    int N, H, Sq, Sk;
    int n_it, n_jt, n_bc, bchunk;
    int64_t items;
    float scale;
    int dbias_atomic; // several batch chunks add into a zeroed dbias
};

// Byte offset of the 16-byte chunk `c` of row `r` in a staging panel of kRowB-byte rows
// (TMA swizzle of span kRowB).
template <int kRowB>
__device__ __forceinline__ uint32_t stg_chunk(int r, int c) {
    constexpr int kMask = kRowB / 16 - 1;
    return static_cast<uint32_t>(r * kRowB + ((c ^ ((r * kRowB >> 7) & kMask)) << 4));
}

// 16-byte chunk c (0..15) of a 256-byte bias^T row r, XOR-swizzled within each 128 bytes so
// that 32 consecutive rows touching the same chunk spread over all banks.
__device__ __forceinline__ uint32_t biast_chunk(int r, int c) {
    return static_cast<uint32_t>(r * 256 + (((c & 8) | ((c & 7) ^ (r & 7))) << 4));
}

// Key-mask code of key j of batch row b: 2 = attended, 1 = masked (logit -1e4), 0 = past Sk.
__device__ __forceinline__ uint32_t key_code(const BwdParams& p, int b, int j) {
    if (j >= p.Sk) {
        return 0;
    }
    return p.kmask[static_cast<int64_t>(b) * p.Sk + j] ? 2u : 1u;
}

template <typename T, int D>
__global__ void __launch_bounds__(BwdCfg<D>::kThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v,
                    const __grid_constant__ CUtensorMap tm_do,
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
    uint64_t* sdp_full = bars + 2 * NST;     // S^T, dP^T of the step in tensor memory
    uint64_t* sdp_free = sdp_full + 1;       // ... read out by every dS warp
    uint64_t* pds_full = sdp_full + 2;       // P^T, dS^T of the step written
    uint64_t* pds_empty = sdp_full + 3;      // ... consumed by the partial-sum MMAs
    uint64_t* part_full = sdp_full + 4;      // [NPB] partial sums in tensor memory
    uint64_t* part_empty = part_full + NPB;  // [NPB] ... read out by the draining warps
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffTmemSlot);
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + C::kOffAbort);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1 + C::kDsWarps);
        }
        mbar_init(sdp_full, 1);
        mbar_init(sdp_free, C::kDsWarps);
        mbar_init(pds_full, C::kDsWarps);
        mbar_init(pds_empty, 1);
        for (int b = 0; b < NPB; ++b) {
            mbar_init(&part_full[b], 1);
            mbar_init(&part_empty[b], 12); // the warps of warpgroups 0-2
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if constexpr (D == 8) {
        // zero halves that pad the head dim of the D = 8 tiles to the MMA's K of 16
        for (int s = 0; s < NST; ++s) {
            for (int t = 0; t < 4; ++t) {
                uint32_t* z = reinterpret_cast<uint32_t*>(smem + C::kOffStages +
                                                          s * C::kStageBytes + t * C::kTile +
                                                          G::kTileBytes);
                for (int i = threadIdx.x; i < G::kTileBytes / 4; i += blockDim.x) {
                    z[i] = 0u;
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
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int n_items_mine = static_cast<int>((p.items - blockIdx.x + gridDim.x - 1) / gridDim.x);

    if (warp == C::kProducerWarp) {
        // =============================== TMA producer ===============================
        // The whole warp runs the loop (converged); one elected lane issues the copies.
        {
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
                bool ok = true;
                for (int b = b_lo; b < b_hi; ++b, ++g) {
                    const int s = g % NST;
                    if (g >= NST && !mbar_wait_w(&kv_empty[s], ((g / NST) - 1) & 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    uint8_t* stage = smem + C::kOffStages + s * C::kStageBytes;
                    const int bh = b * p.H + h;
                    if (elect_one()) {
                        mbar_arrive_expect_tx(&kv_full[s], 4 * G::kTileBytes + 1024);
                        tma_load_4d(stage + C::kOffSK, &tm_k, &kv_full[s], 0, j0, h, b);
                        tma_load_4d(stage + C::kOffSQ, &tm_q, &kv_full[s], 0, i0, h, b);
                        tma_load_4d(stage + C::kOffSV, &tm_v, &kv_full[s], 0, j0, h, b);
                        tma_load_4d(stage + C::kOffSdO, &tm_do, &kv_full[s], 0, i0, h, b);
                        bulk_load(stage + C::kOffRS,
                                  p.rowstat + (static_cast<int64_t>(bh) * p.n_it + itile) * 256,
                                  1024, &kv_full[s]);
                    }
                    __syncwarp();
                }
                if (!ok) {
                    break;
                }
            }
        }
    } else if (warp == C::kMmaWarp) {
        // =============================== MMA issuer ===============================
        // The whole warp runs the loop (converged); MMAs and commits are elect.sync-issued.
        {
            constexpr uint32_t kIdS = idesc_f16(128, 128, false, false, E::kBf16);
            constexpr uint32_t kIdPart = idesc_f16(128, G::kDp, false, true, E::kBf16); // A in TMEM
            constexpr uint32_t kIdDQ = idesc_f16(128, G::kDp, true, true, E::kBf16);
            const uint32_t ds_s = sbase + C::kOffDS;
            uint32_t g = 0;
            int total_steps = 0;
            for (int it = 0; it < n_items_mine; ++it) {
                const int64_t item = blockIdx.x + static_cast<int64_t>(it) * gridDim.x;
                const int bc = static_cast<int>(item / p.n_jt / p.n_it / p.H);
                const int b_lo = bc * p.bchunk, b_hi = min(p.N, b_lo + p.bchunk);
                total_steps += max(0, b_hi - b_lo);
            }
            // dV = P^T dO, dK = dS^T Q (A in tensor memory), dQ = dS K (A = dS^T rows in shared
            // memory, MN-major) of step gp into partial buffer gp % NPB
            auto issue_partials = [&](uint32_t gp) -> bool {
                const int pb = gp % NPB;
                if (gp >= static_cast<uint32_t>(NPB) &&
                    !mbar_wait_w(&part_empty[pb], ((gp / NPB) - 1) & 1, abort_flag)) {
                    return false;
                }
                tc_fence_after();
                const uint32_t st = sbase + C::kOffStages + (gp % NST) * C::kStageBytes;
                const uint32_t dv_tm = tmem + C::kPartBase + pb * 3 * G::kDp;
                const uint32_t dk_tm = dv_tm + G::kDp;
                const uint32_t dq_tm = dv_tm + 2 * G::kDp;
#pragma unroll
                for (int ks = 0; ks < kBM / 16; ++ks) {
                    // K-step ks = queries [16 ks, +16): warpgroup ks / 2, its half ks % 2
                    const uint32_t col = C::kPStride * (ks >> 1) + 8 * (ks & 1);
                    umma_ts_w(dv_tm, tmem + C::kPCol + col, G::mnmajor(st + C::kOffSdO, ks), kIdPart,
                            ks > 0);
                    umma_ts_w(dk_tm, tmem + C::kDSCol + col, G::mnmajor(st + C::kOffSQ, ks), kIdPart,
                            ks > 0);
                }
#pragma unroll
                for (int ks = 0; ks < kBN / 16; ++ks) {
                    const uint64_t da = smem_desc(ds_s + ks * 2048, 16384, 1024, kSwizzle128);
                    umma_ss_w(dq_tm, da, G::mnmajor(st + C::kOffSK, ks), kIdDQ, ks > 0);
                }
                umma_commit_w(&part_full[pb]);
                umma_commit_w(pds_empty);
                umma_commit_w(&kv_empty[gp % NST]);
                return true;
            };
            for (int step = 0; step < total_steps; ++step, ++g) {
                const int s = g % NST;
                if (C::kInPlace && g > 0) {
                    // P^T / dS^T of g-1 live where S^T / dP^T of g go: consume them first
                    if (!mbar_wait_w(pds_full, (g - 1) & 1, abort_flag) || !issue_partials(g - 1)) {
                        break;
                    }
                }
                if (!mbar_wait_w(&kv_full[s], (g / NST) & 1, abort_flag)) {
                    break;
                }
                if (!C::kInPlace && g > 0 && !mbar_wait_w(sdp_free, (g - 1) & 1, abort_flag)) {
                    break;
                }
                tc_fence_after();
                const uint32_t st = sbase + C::kOffStages + s * C::kStageBytes;
#pragma unroll
                for (int ks = 0; ks < G::kKSteps; ++ks) {
                    umma_ss_w(tmem + C::kSCol, G::kmajor(st + C::kOffSK, ks),
                            G::kmajor(st + C::kOffSQ, ks), kIdS, ks > 0);
                }
#pragma unroll
                for (int ks = 0; ks < G::kKSteps; ++ks) {
                    umma_ss_w(tmem + C::kDPCol, G::kmajor(st + C::kOffSV, ks),
                            G::kmajor(st + C::kOffSdO, ks), kIdS, ks > 0);
                }
                umma_commit_w(sdp_full);
                if (!C::kInPlace && g > 0) {
                    if (!mbar_wait_w(pds_full, (g - 1) & 1, abort_flag) || !issue_partials(g - 1)) {
                        break;
                    }
                }
            }
            if (g > 0 && __all_sync(0xffffffffu, *abort_flag == 0)) {
                if (mbar_wait_w(pds_full, (g - 1) & 1, abort_flag)) {
                    issue_partials(g - 1);
                }
            }
        }
    } else {
        // =============================== dS warps ===============================
        const int w = warp >> 2;                         // warpgroup: query columns [32w, +32)
        const int jl = static_cast<int>(warp_lane_base()) + lane; // key row within the tile
        const uint32_t lane_off = warp_lane_base() << 16;
        const float scale = p.scale;
        const uint32_t ds_row = sbase + C::kOffDS + (w >> 1) * 16384 + jl * 128;
        const uint32_t bias_row = sbase + C::kOffBiasT;
        const bool drainer = (w < 3);
        const uint32_t stg = sbase + C::kOffStg + w * C::kStgBytes; // warpgroup w: partial w
        const CUtensorMap* tm_part = w == 0 ? &tm_dv_acc : (w == 1 ? &tm_dk_acc : &tm_dq_acc);
        uint32_t g = 0;
        int prev_bh = 0, prev_i0 = 0, prev_j0 = 0;

        // Partial sum w of step gp: tensor memory -> swizzled staging -> TMA reduce-add into
        // the f32 accumulator (dV, dK at key rows, dQ at query rows).  Every thread of the
        // warpgroup reaches both named barriers, also when a wait gave up.
        auto drain = [&](uint32_t gp, int bh, int i0, int j0) -> bool {
            const int pb = gp % NPB;
            const bool ok = mbar_wait(&part_full[pb], (gp / NPB) & 1, abort_flag);
            if (threadIdx.x == 128 * w) {
                bulk_wait_read<0>(); // the previous reduction has read the staging buffer
            }
            named_bar_sync(1 + w, 128);
            if (!ok || *abort_flag) {
                return false;
            }
            __syncwarp();
            tc_fence_after();
            const uint32_t part = tmem + lane_off + C::kPartBase + pb * 3 * G::kDp + w * G::kDp;
            {
                // the whole partial with one wait, and the buffer released before the stores
                uint32_t raw[D];
#pragma unroll
                for (int c0 = 0; c0 < D; c0 += 8) {
                    tmem_ld8(part + c0, *reinterpret_cast<uint32_t (*)[8]>(&raw[c0]));
                }
                tmem_ld_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&part_empty[pb]);
                }
#pragma unroll
                for (int q = 0; q < D / 4; ++q) {
                    const int col = q * 4;
                    sts128(stg + (col / C::kPW) * C::kPanelBytes +
                               stg_chunk<C::kRowB>(jl, (col % C::kPW) / 4),
                           make_uint4(raw[4 * q], raw[4 * q + 1], raw[4 * q + 2], raw[4 * q + 3]));
                }
            }
            fence_proxy_async_smem();
            named_bar_sync(1 + w, 128);
            if (threadIdx.x == 128 * w) {
                const int row0 = (w == 2) ? i0 : j0;
#pragma unroll
                for (int pn = 0; pn < D / C::kPW; ++pn) {
                    tma_reduce_add_3d(tm_part, smem + (stg - sbase) + pn * C::kPanelBytes,
                                      pn * C::kPW, row0, bh);
                }
                bulk_commit();
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
            const int j = j0 + jl;
            // bias^T: this thread's key j against queries [i0 + 32w, +32), as 16-bit pairs in
            // its own shared-memory row (read back by this thread only)
            {
                uint32_t wv[16];
#pragma unroll
                for (int t = 0; t < 16; ++t) {
                    uint32_t lo = 0, hi = 0;
                    const int i = i0 + 32 * w + 2 * t;
                    if (j < p.Sk) {
                        const uint16_t* src = p.bias + (static_cast<int64_t>(h) * p.Sq + i) * p.Sk + j;
                        if (i < p.Sq) {
                            lo = src[0];
                        }
                        if (i + 1 < p.Sq) {
                            hi = src[p.Sk];
                        }
                    }
                    wv[t] = lo | (hi << 16);
                }
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    sts128(bias_row + biast_chunk(jl, 4 * w + q),
                           make_uint4(wv[4 * q], wv[4 * q + 1], wv[4 * q + 2], wv[4 * q + 3]));
                }
            }
            float dbias[32];
#pragma unroll
            for (int t = 0; t < 32; ++t) {
                dbias[t] = 0.f;
            }
            uint32_t code = b_lo < b_hi ? key_code(p, b_lo, j) : 0u;
            for (int b = b_lo; b < b_hi; ++b, ++g) {
                const int s = g % NST;
                const uint32_t next_code = (b + 1 < b_hi) ? key_code(p, b + 1, j) : 0u;
                if (!mbar_wait(sdp_full, g & 1, abort_flag) ||
                    !mbar_wait(&kv_full[s], (g / NST) & 1, abort_flag)) {
                    goto done;
                }
                __syncwarp();
                tc_fence_after();
                const uint32_t rs = sbase + C::kOffStages + s * C::kStageBytes + C::kOffRS;

                // kAll: every key of this warp is attended (the common case); otherwise the
                // per-thread key code selects the masked-logit constant (-1e4) or exclusion.
                auto ds_tile = [&](auto all_tag) -> bool {
                    constexpr bool kAll = decltype(all_tag)::value;
                    const float2 scale2 = make_float2(scale, scale);
                    const float2 l2 = make_float2(kLog2e, kLog2e);
                    float sc = scale, bm = 1.f, bcst = 0.f, dm = 1.f;
                    if constexpr (!kAll) {
                        if (code != 2) {
                            sc = 0.f;
                            bm = 0.f;
                            dm = 0.f;
                            bcst = (code == 1) ? kMaskedLogit : -INFINITY;
                        }
                    }
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int icol = 32 * w + 8 * c; // query column within the tile
                        uint32_t sv[8], dpv[8];
                        tmem_ld8(tmem + lane_off + C::kSCol + icol, sv);
                        tmem_ld8(tmem + lane_off + C::kDPCol + icol, dpv);
                        tmem_ld_wait();
                        if (!C::kInPlace && c == 3) {
                            // S^T and dP^T are in registers: the next batch row's may go there
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) {
                                mbar_arrive(sdp_free);
                            }
                        }
                        uint32_t pk[4], dk[4];
                        {
                            const uint4 bw = lds128(bias_row + biast_chunk(jl, 4 * w + c));
                            const uint32_t bwv[4] = {bw.x, bw.y, bw.z, bw.w};
#pragma unroll
                            for (int e = 0; e < 4; e += 2) {
                                // queries icol + 2e .. +4: row statistics (broadcast reads)
                                const int ii = icol + 2 * e;
                                const uint4 nl = lds128(rs + 4 * ii);
                                const uint4 nd = lds128(rs + 512 + 4 * ii);
                                const float nlv[4] = {__uint_as_float(nl.x), __uint_as_float(nl.y),
                                                      __uint_as_float(nl.z), __uint_as_float(nl.w)};
                                const float ndv[4] = {__uint_as_float(nd.x), __uint_as_float(nd.y),
                                                      __uint_as_float(nd.z), __uint_as_float(nd.w)};
#pragma unroll
                                for (int u = 0; u < 2; ++u) {
                                    const int k = 2 * e + 2 * u; // element in chunk
                                    float2 b2 = E::to_float2(bwv[e + u]);
                                    float2 t2;
                                    if constexpr (kAll) {
                                        t2 = ffma2(make_float2(__uint_as_float(sv[k]),
                                                               __uint_as_float(sv[k + 1])),
                                                   scale2, b2);
                                    } else {
                                        b2 = ffma2(b2, make_float2(bm, bm), make_float2(bcst, bcst));
                                        t2 = ffma2(make_float2(__uint_as_float(sv[k]),
                                                               __uint_as_float(sv[k + 1])),
                                                   make_float2(sc, sc), b2);
                                    }
                                    const float2 a2 =
                                        ffma2(t2, l2, make_float2(nlv[2 * u], nlv[2 * u + 1]));
                                    const float2 p2 = make_float2(ex2(a2.x), ex2(a2.y));
                                    const float2 d2 = ffma2(make_float2(__uint_as_float(dpv[k]),
                                                                        __uint_as_float(dpv[k + 1])),
                                                            scale2,
                                                            make_float2(ndv[2 * u], ndv[2 * u + 1]));
                                    float2 ds2 = fmul2(p2, d2);
                                    if constexpr (!kAll) {
                                        ds2 = fmul2(ds2, make_float2(dm, dm));
                                    }
                                    const int t = 8 * c + k; // dbias slot
                                    const float2 db2 =
                                        fadd2(make_float2(dbias[t], dbias[t + 1]), ds2);
                                    dbias[t] = db2.x;
                                    dbias[t + 1] = db2.y;
                                    pk[k / 2] = E::pack(p2.x, p2.y);
                                    dk[k / 2] = E::pack(ds2.x, ds2.y);
                                }
                            }
                        }
                        if (c == 0 && g > 0) {
                            // the previous step's partial-sum MMAs must be done reading P^T and
                            // dS^T (tensor memory) and the dS^T rows (shared memory)
                            if (!mbar_wait(pds_empty, (g - 1) & 1, abort_flag)) {
                                return false;
                            }
                            tc_fence_after();
                        }
                        tmem_st4(tmem + lane_off + C::kPCol + C::kPStride * w + 4 * c, pk);
                        tmem_st4(tmem + lane_off + C::kDSCol + C::kPStride * w + 4 * c, dk);
                        // dS^T row jl, queries [icol, +8): 16-byte chunk 4(w&1) + c of the
                        // 128-byte row of panel w/2
                        sts128(ds_row + (((4 * (w & 1) + c) ^ (jl & 7)) << 4),
                               make_uint4(dk[0], dk[1], dk[2], dk[3]));
                    }
                    return true;
                };
                const bool ok = __all_sync(0xffffffffu, code == 2)
                                    ? ds_tile(std::integral_constant<bool, true>())
                                    : ds_tile(std::integral_constant<bool, false>());
                if (!ok) {
                    goto done;
                }
                tmem_st_wait();
                tc_fence_before();
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(pds_full);
                    mbar_arrive(&kv_empty[s]);
                }
                if (drainer && g > 0 && !drain(g - 1, prev_bh, prev_i0, prev_j0)) {
                    goto done;
                }
                prev_bh = b * p.H + h;
                prev_i0 = i0;
                prev_j0 = j0;
                code = next_code;
            }
            // dbias tile: key column j, queries [i0 + 32w, +32); the sums are of scale * dS
            if (j < p.Sk) {
                const float inv_scale = 1.f / scale;
#pragma unroll
                for (int t = 0; t < 32; ++t) {
                    const int i = i0 + 32 * w + t;
                    if (i < p.Sq) {
                        float* dst = p.dbias + (static_cast<int64_t>(h) * p.Sq + i) * p.Sk + j;
                        if (p.dbias_atomic) {
                            atomicAdd(dst, dbias[t] * inv_scale);
                        } else {
                            *dst = dbias[t] * inv_scale;
                        }
                    }
                }
            }
        }
        if (drainer && g > 0 && !drain(g - 1, prev_bh, prev_i0, prev_j0)) {
            goto done;
        }
        if (drainer && threadIdx.x == 128 * w) {
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

// Row statistics of every query tile, padded to whole tiles: rowstat[bh][it][0][ii] =
// -lse * log2(e) and rowstat[bh][it][1][ii] = -scale * delta with delta = sum_d dout * out (f32),
// for query i = 128 it + ii; zeros past Sq.  One thread per padded row.
template <typename T, int D>
__global__ void attn_bwd_rowstat_kernel(const T* __restrict__ out, const T* __restrict__ dout,
                                        const float* __restrict__ lse, float* __restrict__ rowstat,
                                        int64_t bh_count, int Sq, int n_it, float scale,
                                        const RowStrides out_view, const RowStrides dout_view) {
    using E = Elem<T>;
    const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (r >= bh_count * n_it * 128) {
        return;
    }
    const int64_t bh = r / (static_cast<int64_t>(n_it) * 128);
    const int it = static_cast<int>((r / 128) % n_it);
    const int ii = static_cast<int>(r % 128);
    const int i = it * 128 + ii;
    float nl = 0.f, nd = 0.f;
    if (i < Sq) {
        const int64_t row = bh * Sq + i;
        const T* orow = out + view_row_offset(out_view, row, D);
        const T* drow = dout + view_row_offset(dout_view, row, D);
        float acc = 0.f;
#pragma unroll
        for (int c = 0; c < D / 8; ++c) {
            const uint4 a = ld_global_nc_v4(orow + c * 8);
            const uint4 b = ld_global_nc_v4(drow + c * 8);
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
        nl = -lse[row] * kLog2e;
        nd = -scale * acc;
    }
    float* dst = rowstat + (bh * n_it + it) * 256 + ii;
    dst[0] = nl;
    dst[128] = nd;
}

constexpr size_t align256(size_t x) {
    return (x + 255) & ~static_cast<size_t>(255);
}

struct BwdWorkspace {
    size_t dq_off, dk_off, dv_off, rs_off, total;
};

BwdWorkspace bwd_workspace(int64_t N, int64_t H, int64_t Sq, int64_t Sk, int64_t D) {
    BwdWorkspace w;
    const size_t eq = static_cast<size_t>(N * H * Sq * D) * 4;
    const size_t ekv = static_cast<size_t>(N * H * Sk * D) * 4;
    const int64_t n_it = (Sq + kBM - 1) / kBM;
    w.dq_off = 0;
    w.dk_off = align256(eq);
    w.dv_off = w.dk_off + align256(ekv);
    w.rs_off = w.dv_off + align256(ekv);
    w.total = w.rs_off + align256(static_cast<size_t>(N * H * n_it) * 256 * 4);
    return w;
}

template <typename T, int D>
int launch_bwd(cudaStream_t st, const DeviceInfo& dev, const void* q, const void* k,
               const void* v, const void* bias, const uint8_t* kmask, const void* out,
               const float* lse, const void* dout, void* dq, void* dk, void* dv, float* dbias,
               uint8_t* ws, int N, int H, int Sq, int Sk, float scale, int phases,
               const RowView* views) {
    using C = BwdCfg<D>;
    using G = Geo<D>;
    const BwdWorkspace wl = bwd_workspace(N, H, Sq, Sk, D);
    float* dq_acc = reinterpret_cast<float*>(ws + wl.dq_off);
    float* dk_acc = reinterpret_cast<float*>(ws + wl.dk_off);
    float* dv_acc = reinterpret_cast<float*>(ws + wl.dv_off);
    float* rowstat = reinterpret_cast<float*>(ws + wl.rs_off);

    const uint64_t nh = static_cast<uint64_t>(N) * H;
    CUtensorMap tq, tk, tv, tdo, tdq, tdk, tdv;
    CFK_TRY(make_tmap_rows(&tq, q, views[0], D, kBM, G::kSwizzleBytes, "bwd q"));
    CFK_TRY(make_tmap_rows(&tk, k, views[1], D, kBN, G::kSwizzleBytes, "bwd k"));
    CFK_TRY(make_tmap_rows(&tv, v, views[2], D, kBN, G::kSwizzleBytes, "bwd v"));
    CFK_TRY(make_tmap_rows(&tdo, dout, views[4], D, kBM, G::kSwizzleBytes, "bwd dout"));
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
    p.rowstat = rowstat;
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
    p.dbias_atomic = p.n_bc > 1 ? 1 : 0;

    const int64_t rows = static_cast<int64_t>(N) * H * Sq;
    if (phases & 1) {
        const size_t acc_bytes = wl.rs_off;
        if (cudaMemsetAsync(ws, 0, acc_bytes, st) != cudaSuccess ||
            (p.dbias_atomic &&
             cudaMemsetAsync(dbias, 0, static_cast<size_t>(H) * Sq * Sk * 4, st) != cudaSuccess)) {
            return fail(CFK_ERR_LAUNCH, "cfk_attn_bwd: memset failed");
        }
        const int64_t prow = static_cast<int64_t>(nh) * p.n_it * 128;
        attn_bwd_rowstat_kernel<T, D><<<static_cast<int>((prow + 255) / 256), 256, 0, st>>>(
            static_cast<const T*>(out), static_cast<const T*>(dout), lse, rowstat,
            static_cast<int64_t>(nh), Sq, p.n_it, scale, row_strides(views[3], D),
            row_strides(views[4], D));
        CFK_TRY(check_launch("attn_bwd_rowstat"));
    }
    if (phases & 2) {
        auto kern = attn_bwd_kernel<T, D>;
        CFK_TRY(ensure_smem_attr(reinterpret_cast<const void*>(kern), dev.device, C::kSmemBytes,
                                 "attn_bwd"));
        const int grid = static_cast<int>(std::min<int64_t>(p.items, dev.num_sms));
        kern<<<grid, C::kThreads, C::kSmemBytes, st>>>(tq, tk, tv, tdo, tdq, tdk, tdv, p);
        CFK_TRY(check_launch("attn_bwd"));
    }
    if (!(phases & 4)) {
        return CFK_OK;
    }
    const int64_t kv8 = static_cast<int64_t>(N) * H * Sk * D / 8;
    const ConvertJob job{{dq_acc, dk_acc, dv_acc},
                         {dq, dk, dv},
                         {rows * D / 8, kv8, kv8},
                         {row_strides(views[5], D), row_strides(views[6], D),
                          row_strides(views[7], D)},
                         d8_log2(D)};
    f32_to_16_kernel<T><<<dev.num_sms * 8, 256, 0, st>>>(job);
    return check_launch("attn_bwd convert");
}

template <typename T>
int dispatch_bwd(cudaStream_t st, const DeviceInfo& dev, const void* q, const void* k,
                 const void* v, const void* bias, const uint8_t* kmask, const void* out,
                 const float* lse, const void* dout, void* dq, void* dk, void* dv, float* dbias,
                 uint8_t* ws, int N, int H, int Sq, int Sk, int D, float scale, int phases,
                 const RowView* views) {
#define CFK_BWD_D(DD)                                                                              \
    if (D == DD) {                                                                                 \
        return launch_bwd<T, DD>(st, dev, q, k, v, bias, kmask, out, lse, dout, dq, dk, dv, dbias, \
                                 ws, N, H, Sq, Sk, scale, phases, views);                          \
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

// Shared body of cfk_attn_bwd (phases = 7), cfk_attn_bwd_phase (one bit) and their strided
// forms (user_views: q, k, v, out, dout, dq, dk, dv; NULL = packed).
int attn_bwd_entry(const char* fn, int phases, cfk_stream_t stream, cfk_dtype dtype,
                   const void* q, const void* k, const void* v, const void* bias,
                   const uint8_t* kmask, const void* out, const float* lse, const void* dout,
                   void* dq, void* dk, void* dv, float* dbias, void* workspace,
                   size_t workspace_bytes, int64_t N, int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                   float scale, const cfk_view* user_views) {
    clear_error();
    CFK_TRY(check_attn_args(fn, dtype, N, H, Sq, Sk, D));
    static const char* const names[8] = {"q", "k", "v", "out", "dout", "dq", "dk", "dv"};
    RowView views[8];
    for (int t = 0; t < 8; ++t) {
        const int64_t S = (t == 1 || t == 2 || t == 6 || t == 7) ? Sk : Sq;
        CFK_TRY(view_of(fn, names[t], user_views ? &user_views[t] : nullptr, N, H, S, D,
                        &views[t]));
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (H == 0 || Sq == 0 || Sk == 0 || N == 0) {
        // Empty: gradients are zero (dq for Sk == 0; dk, dv for Sq == 0; dbias always).
        if (!(phases & 4)) {
            return CFK_OK;
        }
        if (dbias && H * Sq * Sk > 0 &&
            cudaMemsetAsync(dbias, 0, static_cast<size_t>(H * Sq * Sk) * 4, st) != cudaSuccess) {
            return fail(CFK_ERR_LAUNCH, "%s: memset failed", fn);
        }
        const int64_t nq8 = dq ? N * H * Sq * D / 8 : 0;
        const int64_t nk8 = dk ? N * H * Sk * D / 8 : 0;
        const int64_t nv8 = dv ? N * H * Sk * D / 8 : 0;
        if (nq8 + nk8 + nv8 == 0) {
            return CFK_OK;
        }
        if (!aligned16(dq) || !aligned16(dk) || !aligned16(dv)) {
            return fail(CFK_ERR_INVALID_ARGUMENT, "%s: dq, dk and dv must be 16-byte aligned", fn);
        }
        DeviceInfo dev;
        CFK_TRY(current_device(&dev));
        const attn::ConvertJob job{{nullptr, nullptr, nullptr},
                                   {dq, dk, dv},
                                   {nq8, nk8, nv8},
                                   {attn::row_strides(views[5], D), attn::row_strides(views[6], D),
                                    attn::row_strides(views[7], D)},
                                   attn::d8_log2(static_cast<int>(D))};
        attn::f32_to_16_kernel<__half><<<dev.num_sms * 8, 256, 0, st>>>(job);
        return check_launch("attn_bwd zero");
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
                                                   phases, views)
               : attn::dispatch_bwd<__half>(st, dev, q, k, v, bias, kmask, out, lse, dout, dq, dk,
                                            dv, dbias, ws, n, h, sq, sk, d, scale, phases, views);
}

} // namespace

extern "C" int cfk_attn_bwd(cfk_stream_t stream, cfk_dtype dtype, const void* q, const void* k,
                            const void* v, const void* bias, const uint8_t* kmask,
                            const void* out, const float* lse, const void* dout, void* dq,
                            void* dk, void* dv, float* dbias, void* workspace,
                            size_t workspace_bytes, int64_t N, int64_t H, int64_t Sq, int64_t Sk,
                            int64_t D, float scale) {
    return attn_bwd_entry("cfk_attn_bwd", 7, stream, dtype, q, k, v, bias, kmask, out, lse, dout,
                          dq, dk, dv, dbias, workspace, workspace_bytes, N, H, Sq, Sk, D, scale,
                          nullptr);
}

extern "C" int cfk_attn_bwd_strided(cfk_stream_t stream, cfk_dtype dtype, const void* q,
                                    const void* k, const void* v, const void* bias,
                                    const uint8_t* kmask, const void* out, const float* lse,
                                    const void* dout, void* dq, void* dk, void* dv, float* dbias,
                                    void* workspace, size_t workspace_bytes, int64_t N, int64_t H,
                                    int64_t Sq, int64_t Sk, int64_t D, float scale,
                                    const cfk_view* views) {
    return attn_bwd_entry("cfk_attn_bwd_strided", 7, stream, dtype, q, k, v, bias, kmask, out,
                          lse, dout, dq, dk, dv, dbias, workspace, workspace_bytes, N, H, Sq, Sk,
                          D, scale, views);
}

namespace {

int bwd_phase(const char* fn, int phase, cfk_stream_t stream, cfk_dtype dtype, const void* q,
              const void* k, const void* v, const void* bias, const uint8_t* kmask,
              const void* out, const float* lse, const void* dout, void* dq, void* dk, void* dv,
              float* dbias, void* workspace, size_t workspace_bytes, int64_t N, int64_t H,
              int64_t Sq, int64_t Sk, int64_t D, float scale, const cfk_view* views) {
    if (phase < 0 || phase > 2) {
        clear_error();
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: phase %d not in {0,1,2}", fn, phase);
    }
    return attn_bwd_entry(fn, 1 << phase, stream, dtype, q, k, v, bias, kmask, out, lse, dout,
                          dq, dk, dv, dbias, workspace, workspace_bytes, N, H, Sq, Sk, D, scale,
                          views);
}

} // namespace

extern "C" int cfk_attn_bwd_phase(int phase, cfk_stream_t stream, cfk_dtype dtype,
                                  const void* q, const void* k, const void* v, const void* bias,
                                  const uint8_t* kmask, const void* out, const float* lse,
                                  const void* dout, void* dq, void* dk, void* dv, float* dbias,
                                  void* workspace, size_t workspace_bytes, int64_t N, int64_t H,
                                  int64_t Sq, int64_t Sk, int64_t D, float scale) {
    return bwd_phase("cfk_attn_bwd_phase", phase, stream, dtype, q, k, v, bias, kmask, out, lse,
                     dout, dq, dk, dv, dbias, workspace, workspace_bytes, N, H, Sq, Sk, D, scale,
                     nullptr);
}

extern "C" int cfk_attn_bwd_phase_strided(int phase, cfk_stream_t stream, cfk_dtype dtype,
                                          const void* q, const void* k, const void* v,
                                          const void* bias, const uint8_t* kmask,
                                          const void* out, const float* lse, const void* dout,
                                          void* dq, void* dk, void* dv, float* dbias,
                                          void* workspace, size_t workspace_bytes, int64_t N,
                                          int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                                          float scale, const cfk_view* views) {
    return bwd_phase("cfk_attn_bwd_phase_strided", phase, stream, dtype, q, k, v, bias, kmask,
                     out, lse, dout, dq, dk, dv, dbias, workspace, workspace_bytes, N, H, Sq, Sk,
                     D, scale, views);
}
