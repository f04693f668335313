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
// written once, with plain stores (when the batch rows are split into chunks to fill the SMs,
// each chunk writes its own partial tile and a second launch adds the chunks in a fixed
// order, so the result does not depend on scheduling).  dQ, dK and dV of one batch row are then
// partial sums over key tiles (dQ) or query tiles (dK, dV); the MMA writes those partials into
// tensor memory.  Head dims 8-32: the drain rounds each partial to the output's 16-bit type and
// a TMA tensor reduce-add adds it straight into dQ, dK, dV (zeroed first; the reduce rounds
// once per add, 6 adds at S = 768), which halves the bytes the L2 reduces -- the bound of this
// kernel -- against f32 accumulators, and needs no conversion pass.  Head dim 64 keeps f32
// accumulators in the workspace and a final conversion kernel.
//
// The scores are computed transposed, S^T = K Q^T and dP^T = V dO^T, so that a thread owns one
// key row j of the tile and writes P^T and dS^T rows straight into tensor memory, where they
// are the A operands of dV = P^T dO and dK = dS^T Q (tcgen05.mma with A in tensor memory).
// dQ = dS K reads dS from shared memory (the same rows, taken as an MN-major operand).
//
// Head dims 8, 16 and 32 (attn_bwd_kernel): the per-query row statistics and the key mask ride
// on the score MMAs, as one more K = 16 step of bf16 operands built by the prep kernel and the
// producer warp:
//
//   S'^T  = K Q^T     + [m_j 1 1 1 0 0 0 0] [1 c_hi c_lo c_lo2 0 d_hi d_lo d_lo2]^T
//   dP'^T = V dO^T    + [0   0 0 0 0 1 1 1] [ same rows                          ]^T
//
// with c_i = -lse_i / scale and d_i = -delta_i split into three bf16 parts each (24 bits, an
// f32 value), and m_j = -2^e (2^e scale >= 2^100) for a masked or out-of-range key, 0 otherwise.
// Then P = exp2(scale log2(e) S' + log2(e) bias) and dS = P dP' need no per-query loads, and a
// masked key gets P = 0 exactly.  That equals the reference's -1e4 replacement whenever its
// weight exp(-1e4 - lse) underflows, i.e. for every query tile whose rows all have
// lse > -9900; the prep kernel flags the other tiles (rows with every key masked, or biases
// below -1e4), and those take an exact path that evaluates the masked logit -1e4 per key.
// dS is kept unscaled; the drain multiplies the dQ and dK partials by the softmax scale.
//
//   warps 0-15   dS warps: warp w4 + 4w owns key rows [32 w4, +32) (its tensor-memory lane
//                quarter) and query columns [32w, +32) of warpgroup w.
//   warps 16-19  drain warpgroup: the dV, dK and dQ partials of each step, tensor memory ->
//                16-bit swizzled staging -> TMA reduce-add into the outputs, beside the dS
//                warps' next step.
//   warp 20      TMA producer: per batch row q, dO, k, v tiles, the query tile's statistics
//                block, and the key-mask operand rows it writes itself.
//   warp 21      score MMA issuer: S'^T and dP'^T of each batch row.
//   warp 22      partial-sum MMA issuer: dV, dK, dQ of each batch row, so that the next row's
//                score MMAs never queue behind a wait for the drain (warp 23 idle: it
//                completes the last warpgroup, which setmaxnreg needs).
//
// Head dim 64 (attn_bwd_inplace_kernel) keeps the first design: its partial-sum buffers need the
// tensor-memory columns, so P^T and dS^T overwrite S^T and dP^T, the row statistics come from
// shared memory per score, and the dS warps drain the partials themselves.
#include <type_traits>

#include "attention_common.cuh"
#include "host.h"

namespace cfk {
namespace attn {
namespace {

struct BwdParams {
    const uint8_t* kmask;
    const uint16_t* bias;
    const uint8_t* stats;  // kStatBytes per (batch row, head, query tile)
    float* dbias_out;      // dbias, or the first batch chunk's partial tile set
    int64_t dbias_stride;  // floats between the partials of consecutive batch chunks (0: one)
    int dbias_accumulate;  // add this launch's sums to dbias_out instead of storing them
    int b_base, b_end;     // the batch rows of this launch (head dim 64's accumulators hold
                           // rows b - b_base)
    int N, H, Sq, Sk;
    int n_it, n_jt, n_bc, bchunk;
    int64_t items;
    float scale;
    uint32_t mask_bits;    // bf16 bits of -2^e for masked keys (0: none usable, exact path only)
};

// Statistics block of one (batch row, head, query tile), written by attn_bwd_prep_kernel:
//   [0, 2048)     bf16 [128 queries][8]: 1, c_hi, c_lo, c_lo2, 0, d_hi, d_lo, d_lo2
//   [2048, 2560)  f32 [128]: -lse log2(e)                 (0 past Sq)
//   [2560, 3072)  f32 [128]: -scale delta                 (0 past Sq)
//   [3072, 3088)  u32 flag: 1 when the masked-key MMA column is exact for every row
constexpr int kStatNl = 2048;
constexpr int kStatNd = 2560;
constexpr int kStatFlag = 3072;
constexpr int kStatBytes = 3088;
// A row whose lse is above this gives a masked key the weight exp(-1e4 - lse) < 2^-126, which
// the exponential flushes to 0 like the masked-key MMA column does.
constexpr float kSafeLse = -9900.f;

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

// (query tile, key tile, head, batch chunk) of work item `item` (key tile fastest).
struct BwdItem {
    int jt, itile, h, bc;
};

__device__ __forceinline__ BwdItem decode_item(const BwdParams& p, int64_t item) {
    BwdItem r;
    r.jt = static_cast<int>(item % p.n_jt);
    int64_t rest = item / p.n_jt;
    r.itile = static_cast<int>(rest % p.n_it);
    rest /= p.n_it;
    r.h = static_cast<int>(rest % p.H);
    r.bc = static_cast<int>(rest / p.H);
    return r;
}

template <int D>
struct BwdCfg {
    using G = Geo<D>;
    static_assert(D <= 32, "head dim 64 uses attn_bwd_inplace_kernel");
    static constexpr int NST = 3; // operand stages
    static constexpr int kDsWarps = 16;
    static constexpr int kDrainWarp0 = 16;
    static constexpr int kProducerWarp = 20;
    static constexpr int kMmaWarp = 21;                // score MMAs
    static constexpr int kPartWarp = 22;               // partial-sum MMAs (23 idle)
    static constexpr int kThreads = 24 * 32;
    // Registers per thread: 80 at launch (65536 / 768, in units of 8); the dS warpgroups take
    // 96 and the other two give theirs down to 48 (4 x 128 x 96 + 2 x 128 x 48 = 768 x 80).
    static constexpr int kDsRegs = 96;
    static constexpr int kOtherRegs = 48;
    static constexpr int kLaunchRegs = 80;
    static_assert(4 * kDsRegs + 2 * kOtherRegs == (kThreads / 128) * kLaunchRegs,
                  "register split");
    static constexpr uint32_t kTmemCols = 512;
    static constexpr int kSCol = 0;
    static constexpr int kDPCol = 128;
    // P^T / dS^T as packed 16-bit pairs: warpgroup w's 32 query columns at col + kPStride * w
    static constexpr int kPCol = 256;
    static constexpr int kDSCol = 320;
    static constexpr int kPStride = 16;
    static constexpr int kPartBase = 384; // dV, dK, dQ partials, kDp columns each
    static_assert(kPartBase + 3 * G::kDp <= 512, "tensor memory budget");

    static constexpr int kTile = ((G::kTileAlloc + 1023) / 1024) * 1024;
    static constexpr int kOffQ = 0;
    static constexpr int kOffDO = kTile;
    static constexpr int kOffK = 2 * kTile;
    static constexpr int kOffV = 3 * kTile;
    static constexpr int kOffStat = 4 * kTile;                              // statistics block
    static constexpr int kOffAS = kOffStat + ((kStatBytes + 127) / 128) * 128; // key-mask rows
    static constexpr int kStageBytes = ((kOffAS + 2048 + 1023) / 1024) * 1024;

    // 16-bit staging of one [128 x D] partial for the TMA reduce (rows of 2D bytes, the
    // swizzle span of the output maps)
    static constexpr int kRowB = 2 * D;
    static constexpr int kStgBytes = 128 * kRowB;

    static constexpr int kOffStages = 0;
    static constexpr int kOffDS = NST * kStageBytes;    // dS^T rows, MN-major operand of dQ
    static constexpr int kOffBiasT = kOffDS + 32768;    // bias^T: row j = 128 queries, 16-bit
    static constexpr int kOffStg = kOffBiasT + 32768;   // two staging buffers
    static constexpr int kOffADP = kOffStg + 2 * kStgBytes; // [0 0 0 0 0 1 1 1] rows (bf16)
    static constexpr int kOffZero = kOffADP + 2048;     // zero upper K half of the ext operands
    static constexpr int kOffBar = kOffZero + 2048;
    // kv_full[NST], kv_empty[NST], sdp_full, sdp_free, pds_full, pds_empty, part_full,
    // part_empty
    static constexpr int kNumBars = 2 * NST + 6;
    static constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
    static constexpr int kOffAbort = kOffTmemSlot + 4;
    static constexpr int kSmemBytes = kOffAbort + 4 + 1024;
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

// bf16 bits of x rounded to nearest even (finite x).
__device__ __forceinline__ uint32_t bf16_bits(float x) {
    return static_cast<uint32_t>(Elem<__nv_bfloat16>::from_float(x));
}

// x as three bf16 parts whose sum equals x to f32 precision.
__device__ __forceinline__ void split3_bf16(float x, uint32_t& h0, uint32_t& h1, uint32_t& h2) {
    h0 = bf16_bits(x);
    const float r1 = x - __uint_as_float(h0 << 16);
    h1 = bf16_bits(r1);
    const float r2 = r1 - __uint_as_float(h1 << 16);
    h2 = bf16_bits(r2);
}

template <typename T, int D>
__global__ void __launch_bounds__(BwdCfg<D>::kThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v,
                    const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_dq,
                    const __grid_constant__ CUtensorMap tm_dk,
                    const __grid_constant__ CUtensorMap tm_dv, const BwdParams p) {
    using C = BwdCfg<D>;
    using G = Geo<D>;
    using E = Elem<T>;
    constexpr int NST = C::NST;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
    uint64_t* kv_full = bars;
    uint64_t* kv_empty = bars + NST;
    uint64_t* sdp_full = bars + 2 * NST;     // S'^T, dP'^T of the step in tensor memory
    uint64_t* sdp_free = sdp_full + 1;       // ... read out by every dS warp
    uint64_t* pds_full = sdp_full + 2;       // P^T, dS^T of the step written
    uint64_t* pds_empty = sdp_full + 3;      // ... consumed by the partial-sum MMAs
    uint64_t* part_full = sdp_full + 4;      // partial sums in tensor memory
    uint64_t* part_empty = sdp_full + 5;     // ... read out by the drain warpgroup
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
        mbar_init(part_full, 1);
        mbar_init(part_empty, 4);
        *abort_flag = 0;
        fence_mbar_init();
    }
    {
        // constant operands: the dP' extension rows [0 0 0 0 0 1 1 1] and the zero block that
        // serves as the upper K half of every extension operand
        uint32_t* adp = reinterpret_cast<uint32_t*>(smem + C::kOffADP);
        uint32_t* zero = reinterpret_cast<uint32_t*>(smem + C::kOffZero);
        for (int i = threadIdx.x; i < 512; i += blockDim.x) {
            const int k = i & 3;
            adp[i] = k == 2 ? 0x3F800000u : (k == 3 ? 0x3F803F80u : 0u);
            zero[i] = 0u;
        }
        if constexpr (D == 8) {
            // zero halves that pad the head dim of the D = 8 tiles to the MMA's K of 16
            for (int s = 0; s < NST; ++s) {
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
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int n_items_mine = static_cast<int>((p.items - blockIdx.x + gridDim.x - 1) / gridDim.x);
    // Roles by warpgroup, each moving its register share first (setmaxnreg applies to the
    // code it dominates): dS warpgroups 0-3, the drain warpgroup 4, warpgroup 5 = producer,
    // the two MMA issuers and one idle warp.
    const int wgrp = warp >> 2;
    if (wgrp == 5) {
        setmaxnreg_dec<C::kOtherRegs>();
      if (warp == C::kProducerWarp) {
        // =============================== TMA producer ===============================
        // The whole warp runs the loop (converged): every lane writes four key-mask operand
        // rows, then one elected lane issues the copies.
        uint32_t g = 0;
        for (int it = 0; it < n_items_mine; ++it) {
            const BwdItem w = decode_item(p, blockIdx.x + static_cast<int64_t>(it) * gridDim.x);
            const int i0 = w.itile * kBM, j0 = w.jt * kBN;
            const int b_lo = p.b_base + w.bc * p.bchunk, b_hi = min(p.b_end, b_lo + p.bchunk);
            bool ok = true;
            for (int b = b_lo; b < b_hi; ++b, ++g) {
                const int s = g % NST;
                if (g >= NST && !mbar_wait_w(&kv_empty[s], ((g / NST) - 1) & 1, abort_flag)) {
                    ok = false;
                    break;
                }
                uint8_t* stage = smem + C::kOffStages + s * C::kStageBytes;
                const uint32_t as_rows = sbase + C::kOffStages + s * C::kStageBytes + C::kOffAS;
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int jj = 4 * lane + r;
                    const uint32_t code = key_code(p, b, j0 + jj);
                    // [m_j 1 1 1 0 0 0 0]
                    const uint32_t w0 = (code == 2 ? 0u : p.mask_bits) | 0x3F800000u;
                    sts128(as_rows + jj * 16, make_uint4(w0, 0x3F803F80u, 0u, 0u));
                }
                fence_proxy_async_smem();
                __syncwarp();
                const int bh = b * p.H + w.h;
                if (elect_one()) {
                    mbar_arrive_expect_tx(&kv_full[s], 4 * G::kTileBytes + kStatBytes);
                    tma_load_4d(stage + C::kOffK, &tm_k, &kv_full[s], 0, j0, w.h, b);
                    tma_load_4d(stage + C::kOffQ, &tm_q, &kv_full[s], 0, i0, w.h, b);
                    tma_load_4d(stage + C::kOffV, &tm_v, &kv_full[s], 0, j0, w.h, b);
                    tma_load_4d(stage + C::kOffDO, &tm_do, &kv_full[s], 0, i0, w.h, b);
                    bulk_load(stage + C::kOffStat,
                              p.stats + (static_cast<int64_t>(bh) * p.n_it + w.itile) * kStatBytes,
                              kStatBytes, &kv_full[s]);
                }
                __syncwarp();
            }
            if (!ok) {
                break;
            }
        }
      } else if (warp == C::kMmaWarp || warp == C::kPartWarp) {
        // =============================== MMA issuers ===============================
        // Each warp runs its loop converged; MMAs and commits are elect.sync-issued.  Warp
        // kMmaWarp issues the score MMAs of every step, warp kPartWarp the partial-sum MMAs:
        // each tcgen05.commit tracks the MMAs of its own thread, and the partial sums of step g
        // are issued only after pds_full(g), which the dS warps signal after sdp_full(g), so the
        // stage's operands are released (kv_empty) by the partial-sum warp alone.
        constexpr uint32_t kIdS = idesc_f16(128, 128, false, false, E::kBf16);
        constexpr uint32_t kIdExt = idesc_f16(128, 128, false, false, true); // bf16 operands
        constexpr uint32_t kIdPart = idesc_f16(128, G::kDp, false, true, E::kBf16); // A in TMEM
        constexpr uint32_t kIdDQ = idesc_f16(128, G::kDp, true, true, E::kBf16);
        const uint32_t ds_s = sbase + C::kOffDS;
        const uint32_t zero_s = sbase + C::kOffZero;
        // [128 rows x 16] bf16 K-major operand in the interleave layout whose upper 8 columns
        // are the zero block
        auto ext_desc = [&](uint32_t addr) { return smem_desc(addr, zero_s - addr, 128, kInterleave); };
        const uint64_t adp_desc = ext_desc(sbase + C::kOffADP);
        uint32_t g = 0;
        int total_steps = 0;
        for (int it = 0; it < n_items_mine; ++it) {
            const BwdItem w = decode_item(p, blockIdx.x + static_cast<int64_t>(it) * gridDim.x);
            const int b_lo = p.b_base + w.bc * p.bchunk, b_hi = min(p.b_end, b_lo + p.bchunk);
            total_steps += max(0, b_hi - b_lo);
        }
        // dV = P^T dO, dK = dS^T Q (A in tensor memory), dQ = dS K (A = dS^T rows in shared
        // memory, MN-major) of step gp
        auto issue_partials = [&](uint32_t gp) -> bool {
            if (gp >= 1 && !mbar_wait_w(part_empty, (gp - 1) & 1, abort_flag)) {
                return false;
            }
            tc_fence_after();
            const uint32_t st = sbase + C::kOffStages + (gp % NST) * C::kStageBytes;
            const uint32_t dv_tm = tmem + C::kPartBase;
            const uint32_t dk_tm = dv_tm + G::kDp;
            const uint32_t dq_tm = dv_tm + 2 * G::kDp;
            // the three accumulators' K-steps interleaved (independent chains)
            static_assert(kBM == kBN, "one K-step loop for the three partials");
#pragma unroll
            for (int ks = 0; ks < kBM / 16; ++ks) {
                // dV, dK: K-step ks = queries [16 ks, +16): warpgroup ks / 2, its half ks % 2
                const uint32_t col = C::kPStride * (ks >> 1) + 8 * (ks & 1);
                umma_ts_w(dv_tm, tmem + C::kPCol + col, G::mnmajor(st + C::kOffDO, ks), kIdPart,
                          ks > 0);
                umma_ts_w(dk_tm, tmem + C::kDSCol + col, G::mnmajor(st + C::kOffQ, ks), kIdPart,
                          ks > 0);
                // dQ: K-step ks = keys [16 ks, +16)
                const uint64_t da = smem_desc(ds_s + ks * 2048, 16384, 1024, kSwizzle128);
                umma_ss_w(dq_tm, da, G::mnmajor(st + C::kOffK, ks), kIdDQ, ks > 0);
            }
            umma_commit_w(part_full);
            umma_commit_w(pds_empty);
            umma_commit_w(&kv_empty[gp % NST]);
            return true;
        };
        if (warp == C::kPartWarp) {
            for (; static_cast<int>(g) < total_steps; ++g) {
                if (!mbar_wait_w(pds_full, g & 1, abort_flag) || !issue_partials(g)) {
                    break;
                }
            }
        } else {
        for (int step = 0; step < total_steps; ++step, ++g) {
            const int s = g % NST;
            if (!mbar_wait_w(&kv_full[s], (g / NST) & 1, abort_flag)) {
                break;
            }
            if (g > 0 && !mbar_wait_w(sdp_free, (g - 1) & 1, abort_flag)) {
                break;
            }
            tc_fence_after();
            const uint32_t st = sbase + C::kOffStages + s * C::kStageBytes;
            const uint64_t bext = ext_desc(st + C::kOffStat);
            // S'^T and dP'^T K-steps interleaved (independent chains)
#pragma unroll
            for (int ks = 0; ks < G::kKSteps; ++ks) {
                umma_ss_w(tmem + C::kSCol, G::kmajor(st + C::kOffK, ks),
                          G::kmajor(st + C::kOffQ, ks), kIdS, ks > 0);
                umma_ss_w(tmem + C::kDPCol, G::kmajor(st + C::kOffV, ks),
                          G::kmajor(st + C::kOffDO, ks), kIdS, ks > 0);
            }
            umma_ss_w(tmem + C::kSCol, ext_desc(st + C::kOffAS), bext, kIdExt, 1);
            umma_ss_w(tmem + C::kDPCol, adp_desc, bext, kIdExt, 1);
            umma_commit_w(sdp_full);
        }
        }
      }
    } else if (wgrp == 4) {
        // =============================== drain warpgroup ===============================
        // Partial sums of step g: tensor memory -> registers (the buffer is released after the
        // third) -> 16-bit, dK and dQ times the softmax scale -> swizzled staging (two buffers,
        // alternating) -> TMA reduce-add into dV, dK (key rows) and dQ (query rows) of batch
        // row b.  Every thread reaches every named barrier of a step, also when a wait gave up.
        setmaxnreg_dec<C::kOtherRegs>();
        const int dw = warp - C::kDrainWarp0;
        const int row = 32 * dw + lane;
        const uint32_t lane_off = static_cast<uint32_t>(32 * dw) << 16;
        const bool leader = threadIdx.x == C::kDrainWarp0 * 32;
        uint32_t g = 0, pc = 0;
        for (int it = 0; it < n_items_mine; ++it) {
            const BwdItem w = decode_item(p, blockIdx.x + static_cast<int64_t>(it) * gridDim.x);
            const int i0 = w.itile * kBM, j0 = w.jt * kBN;
            const int b_lo = p.b_base + w.bc * p.bchunk, b_hi = min(p.b_end, b_lo + p.bchunk);
            for (int b = b_lo; b < b_hi; ++b, ++g) {
                const bool ok = mbar_wait(part_full, g & 1, abort_flag);
                // one decision for the whole warpgroup, or some threads would wait at the next
                // named barrier for threads that left
                if (!named_bar_and(1, 128, ok && !*abort_flag)) {
                    goto done;
                }
                __syncwarp();
                tc_fence_after();
#pragma unroll 1
                for (int pp = 0; pp < 3; ++pp) {
                    const uint32_t stg = sbase + C::kOffStg + (pc & 1) * C::kStgBytes;
                    if (leader) {
                        bulk_wait_read<1>(); // the reduce two partials back has read this buffer
                    }
                    named_bar_sync(1, 128);
                    // at most 16 columns in registers at a time (this warpgroup runs with few)
                    constexpr int kHalf = D < 16 ? D : 16;
#pragma unroll
                    for (int h0 = 0; h0 < D; h0 += kHalf) {
                        uint32_t raw[kHalf];
#pragma unroll
                        for (int c0 = 0; c0 < kHalf; c0 += 8) {
                            tmem_ld8(tmem + lane_off + C::kPartBase + pp * G::kDp + h0 + c0,
                                     *reinterpret_cast<uint32_t (*)[8]>(&raw[c0]));
                        }
                        tmem_ld_wait();
                        if (pp == 2 && h0 + kHalf == D) {
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) {
                                mbar_arrive(part_empty);
                            }
                        }
                        const float mul = pp == 0 ? 1.f : p.scale;
#pragma unroll
                        for (int q = 0; q < kHalf / 8; ++q) {
                            uint32_t o[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                o[e] = E::pack(__uint_as_float(raw[8 * q + 2 * e]) * mul,
                                               __uint_as_float(raw[8 * q + 2 * e + 1]) * mul);
                            }
                            sts128(stg + stg_chunk<C::kRowB>(row, (h0 + 8 * q) / 8),
                                   make_uint4(o[0], o[1], o[2], o[3]));
                        }
                    }
                    fence_proxy_async_smem();
                    named_bar_sync(1, 128);
                    if (leader) {
                        const CUtensorMap* tm = pp == 0 ? &tm_dv : (pp == 1 ? &tm_dk : &tm_dq);
                        tma_reduce_add_4d(tm, smem + (stg - sbase), 0, pp == 2 ? i0 : j0, w.h, b);
                        bulk_commit();
                    }
                    ++pc;
                }
            }
        }
    } else {
        // =============================== dS warps ===============================
        setmaxnreg_inc<C::kDsRegs>();
        const int w = warp >> 2;                         // warpgroup: query columns [32w, +32)
        const int jl = static_cast<int>(warp_lane_base()) + lane; // key row within the tile
        const uint32_t lane_off = warp_lane_base() << 16;
        const float sl2 = p.scale * kLog2e;
        const uint32_t ds_row = sbase + C::kOffDS + (w >> 1) * 16384 + jl * 128;
        const uint32_t bias_row = sbase + C::kOffBiasT;
        // barriers and the abort word as 32-bit shared-memory addresses (fewer registers)
        const uint32_t bar_s = sbase + C::kOffBar;
        const uint32_t sdp_full_s = bar_s + 8 * (2 * NST);
        const uint32_t sdp_free_s = sdp_full_s + 8;
        const uint32_t pds_full_s = sdp_full_s + 16;
        const uint32_t pds_empty_s = sdp_full_s + 24;
        const uint32_t abort_s = sbase + C::kOffAbort;
        uint32_t g = 0;

        for (int it = 0; it < n_items_mine; ++it) {
            const BwdItem wi = decode_item(p, blockIdx.x + static_cast<int64_t>(it) * gridDim.x);
            const int h = wi.h;
            const int i0 = wi.itile * kBM, j0 = wi.jt * kBN;
            const int b_lo = p.b_base + wi.bc * p.bchunk, b_hi = min(p.b_end, b_lo + p.bchunk);
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
            for (int b = b_lo; b < b_hi; ++b, ++g) {
                const int s = g % NST;
                if (!mbar_wait_s(sdp_full_s, g & 1, abort_s) ||
                    !mbar_wait_s(bar_s + 8 * s, (g / NST) & 1, abort_s)) {
                    goto done;
                }
                __syncwarp();
                tc_fence_after();
                const uint32_t stat = sbase + C::kOffStages + s * C::kStageBytes + C::kOffStat;
                const bool fast = ld_shared_u32(stat + kStatFlag) != 0;

                // kFast: P = exp2(sl2 S' + log2(e) bias), dS = P dP' (masked keys carry -2^e in
                // S').  Otherwise this thread's key code selects the logit: attended keys as
                // above, masked keys -1e4 (from the row statistic -lse log2 e), keys past Sk none.
                auto ds_tile = [&](auto fast_tag, uint32_t code) -> bool {
                    constexpr bool kFast = decltype(fast_tag)::value;
                    const float2 sl2v = make_float2(sl2, sl2);
                    const float2 l2v = make_float2(kLog2e, kLog2e);
                    // exact path: the logit of a masked key is -1e4, of a key past Sk none
                    const float cmask = code == 1 ? kMaskedLogit * kLog2e : -INFINITY;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int q0 = 32 * w + 8 * c; // query column within the tile
                        uint32_t sv[8], dv[8];
                        tmem_ld8(tmem + lane_off + C::kSCol + q0, sv);
                        tmem_ld8(tmem + lane_off + C::kDPCol + q0, dv);
                        tmem_ld_wait();
                        if (c == 3) {
                            // S'^T and dP'^T are in registers: the next batch row's may go there
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) {
                                mbar_arrive_s(sdp_free_s);
                            }
                        }
                        const uint4 bw = lds128(bias_row + biast_chunk(jl, q0 >> 3));
                        const uint32_t bwv[4] = {bw.x, bw.y, bw.z, bw.w};
                        uint32_t pk[4], dk[4];
#pragma unroll
                        for (int t = 0; t < 4; ++t) {
                            const float2 b2 = E::to_float2(bwv[t]);
                            const float2 s2 = make_float2(__uint_as_float(sv[2 * t]),
                                                          __uint_as_float(sv[2 * t + 1]));
                            float2 a2 = ffma2(s2, sl2v, fmul2(b2, l2v));
                            if constexpr (!kFast) {
                                if (code != 2) {
                                    const uint2 nlw = lds64(stat + kStatNl + 4 * (q0 + 2 * t));
                                    a2 = make_float2(__uint_as_float(nlw.x) + cmask,
                                                     __uint_as_float(nlw.y) + cmask);
                                }
                            }
                            const float2 p2 = make_float2(ex2(a2.x), ex2(a2.y));
                            float2 ds2 = fmul2(p2, make_float2(__uint_as_float(dv[2 * t]),
                                                               __uint_as_float(dv[2 * t + 1])));
                            if constexpr (!kFast) {
                                if (code != 2) {
                                    ds2 = make_float2(0.f, 0.f); // masked logits are constants
                                }
                            }
                            const int u = 8 * c + 2 * t; // dbias slot
                            const float2 db2 = fadd2(make_float2(dbias[u], dbias[u + 1]), ds2);
                            dbias[u] = db2.x;
                            dbias[u + 1] = db2.y;
                            pk[t] = E::pack(p2.x, p2.y);
                            dk[t] = E::pack(ds2.x, ds2.y);
                        }
                        if (c == 0 && g > 0) {
                            // the previous step's partial-sum MMAs must be done reading P^T and
                            // dS^T (tensor memory) and the dS^T rows (shared memory)
                            if (!mbar_wait_s(pds_empty_s, (g - 1) & 1, abort_s)) {
                                return false;
                            }
                            tc_fence_after();
                        }
                        tmem_st4(tmem + lane_off + C::kPCol + C::kPStride * w + 4 * c, pk);
                        tmem_st4(tmem + lane_off + C::kDSCol + C::kPStride * w + 4 * c, dk);
                        // dS^T row jl, queries [q0, +8): 16-byte chunk 4(w&1) + c of the
                        // 128-byte row of panel w/2
                        sts128(ds_row + (((4 * (w & 1) + c) ^ (jl & 7)) << 4),
                               make_uint4(dk[0], dk[1], dk[2], dk[3]));
                    }
                    return true;
                };
                const bool ok = fast ? ds_tile(std::integral_constant<bool, true>(), 2u)
                                     : ds_tile(std::integral_constant<bool, false>(),
                                               key_code(p, b, j));
                if (!ok) {
                    goto done;
                }
                tmem_st_wait();
                tc_fence_before();
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive_s(pds_full_s);
                    mbar_arrive_s(bar_s + 8 * (NST + s));
                }
            }
            // dbias tile: key column j, queries [i0 + 32w, +32), this batch chunk's sum
            if (j < p.Sk) {
                const int ib = i0 + 32 * w;
                float* o = p.dbias_out + static_cast<int64_t>(wi.bc) * p.dbias_stride +
                           (static_cast<int64_t>(h) * p.Sq + ib) * p.Sk + j;
                const int n = min(32, p.Sq - ib);
#pragma unroll
                for (int t = 0; t < 32; ++t) {
                    if (t < n) {
                        *o = p.dbias_accumulate ? *o + dbias[t] : dbias[t];
                    }
                    o += p.Sk;
                }
            }
            // keeps the next item's bias loads (and their addresses) after these stores
            asm volatile("" ::: "memory");
        }
    }

done:
    __syncwarp();
    if (warp >= C::kDrainWarp0 && warp < C::kDrainWarp0 + 4 && threadIdx.x == C::kDrainWarp0 * 32) {
        bulk_wait<0>(); // reductions complete before the CTA retires
    }
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

// ---------------------------------------------------------------------------------------------
// Head dim 64: the first design (see the file comment).
// ---------------------------------------------------------------------------------------------
template <int D>
struct InplaceCfg {
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

template <typename T, int D>
__global__ void __launch_bounds__(InplaceCfg<D>::kThreads, 1)
    attn_bwd_inplace_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v,
                    const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_dq_acc,
                    const __grid_constant__ CUtensorMap tm_dk_acc,
                    const __grid_constant__ CUtensorMap tm_dv_acc, const BwdParams p) {
    using C = InplaceCfg<D>;
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
                                  p.stats + (static_cast<int64_t>(bh) * p.n_it + itile) *
                                                kStatBytes + kStatNl,
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
            // one decision for the whole warpgroup (see named_bar_and)
            if (!named_bar_and(1 + w, 128, ok && !*abort_flag)) {
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
                float* out = p.dbias_out + static_cast<int64_t>(bc) * p.dbias_stride;
#pragma unroll
                for (int t = 0; t < 32; ++t) {
                    const int i = i0 + 32 * w + t;
                    if (i < p.Sq) {
                        out[(static_cast<int64_t>(h) * p.Sq + i) * p.Sk + j] = dbias[t] * inv_scale;
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

// Statistics block of every (batch row, head, query tile), padded to whole tiles: one CTA of
// 128 threads per block, thread = query i = 128 it + ii.  delta = sum_d dout * out (f32).
template <typename T, int D>
__global__ void __launch_bounds__(128)
    attn_bwd_prep_kernel(const T* __restrict__ out, const T* __restrict__ dout,
                         const float* __restrict__ lse, uint8_t* __restrict__ stats, int Sq,
                         int n_it, float scale, uint32_t mask_bits, const RowStrides out_view,
                         const RowStrides dout_view) {
    using E = Elem<T>;
    const int64_t blk = blockIdx.x; // bh * n_it + it
    const int64_t bh = blk / n_it;
    const int it = static_cast<int>(blk - bh * n_it);
    const int ii = threadIdx.x;
    const int i = it * 128 + ii;
    float nl = 0.f, nd = 0.f, c = 0.f, dd = 0.f;
    bool safe = true;
    if (i < Sq) {
        const int64_t row = bh * Sq + i;
        const T* orow = out + view_row_offset(out_view, row, D);
        const T* drow = dout + view_row_offset(dout_view, row, D);
        float acc = 0.f;
#pragma unroll
        for (int c8 = 0; c8 < D / 8; ++c8) {
            const uint4 a = ld_global_nc_v4(orow + c8 * 8);
            const uint4 b = ld_global_nc_v4(drow + c8 * 8);
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
        const float l = lse[row];
        nl = -l * kLog2e;
        nd = -scale * acc;
        c = nl / (scale * kLog2e); // -lse / scale: scale log2(e) c = -lse log2(e)
        dd = -acc;
        safe = l > kSafeLse;
    }
    uint8_t* blkp = stats + blk * kStatBytes;
    uint32_t c0, c1, c2, d0, d1, d2;
    split3_bf16(c, c0, c1, c2);
    split3_bf16(dd, d0, d1, d2);
    // [1 c_hi c_lo c_lo2 0 d_hi d_lo d_lo2]
    *reinterpret_cast<uint4*>(blkp + ii * 16) =
        make_uint4(0x3F80u | (c0 << 16), c1 | (c2 << 16), d0 << 16, d1 | (d2 << 16));
    reinterpret_cast<float*>(blkp + kStatNl)[ii] = nl;
    reinterpret_cast<float*>(blkp + kStatNd)[ii] = nd;
    const int all_safe = __syncthreads_and(safe ? 1 : 0);
    if (ii < 4) {
        reinterpret_cast<uint32_t*>(blkp + kStatFlag)[ii] =
            (ii == 0 && all_safe && mask_bits != 0) ? 1u : 0u;
    }
}

// dbias (+)= the batch chunks' partial tiles added in chunk order.
__global__ void dbias_chunks_kernel(const float* __restrict__ part, float* __restrict__ dbias,
                                    int64_t n, int chunks, int accumulate) {
    for (int64_t x = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; x < n;
         x += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float acc = accumulate ? dbias[x] : 0.f;
        for (int c = 0; c < chunks; ++c) {
            acc += part[c * n + x];
        }
        dbias[x] = acc;
    }
}

constexpr size_t align256(size_t x) {
    return (x + 255) & ~static_cast<size_t>(255);
}

// SM count the workspace size assumes when it sizes the dbias chunk partials (at least the
// SM count of every compute capability 10.0 part).
constexpr int kWorkspaceSms = 160;


// Batch chunks of a launch with `base` (head, query tile, key tile) items: as many as fit in
// one wave of `sms` CTAs, at least one, at most the launch's rows.
int64_t batch_chunks(int64_t rows, int64_t base, int64_t sms) {
    if (base <= 0 || rows <= 0) {
        return 1;
    }
    int64_t nbc = base >= sms ? 1 : std::max<int64_t>(1, sms / base);
    return std::min<int64_t>(nbc, rows);
}

// Workspace of the backward: f32 dq, dk, dv accumulators (head dim 64 only; the other head dims
// reduce straight into the outputs), the row statistics blocks and, when the batch rows are
// split into chunks, the chunks' dbias partials.
struct BwdWorkspace {
    size_t dq_off, dk_off, dv_off, stat_off, dbp_off, total;
    int64_t max_chunks;  // batch chunks (dbias partials) of the launch at most
};

BwdWorkspace bwd_workspace(int64_t N, int64_t H, int64_t Sq, int64_t Sk, int64_t D) {
    BwdWorkspace w;
    const int64_t acc_rows = D == 64 ? N : 0;
    const size_t eq = static_cast<size_t>(acc_rows * H * Sq * D) * 4;
    const size_t ekv = static_cast<size_t>(acc_rows * H * Sk * D) * 4;
    const int64_t n_it = (Sq + kBM - 1) / kBM;
    const int64_t n_jt = (Sk + kBN - 1) / kBN;
    w.dq_off = 0;
    w.dk_off = align256(eq);
    w.dv_off = w.dk_off + align256(ekv);
    w.stat_off = w.dv_off + align256(ekv);
    w.dbp_off = w.stat_off + align256(static_cast<size_t>(N * H * n_it) * kStatBytes);
    // batch rows per chunk -> number of chunks, as the launch computes it
    const int64_t rows = std::max<int64_t>(N, 1);
    const int64_t nbc = batch_chunks(rows, H * n_it * n_jt, kWorkspaceSms);
    const int64_t bchunk = (rows + nbc - 1) / std::max<int64_t>(nbc, 1);
    w.max_chunks = bchunk > 0 ? (rows + bchunk - 1) / bchunk : 1;
    w.total = w.dbp_off + (w.max_chunks > 1 ? align256(static_cast<size_t>(w.max_chunks * H * Sq *
                                                                          Sk) * 4)
                                            : 0);
    return w;
}

// Phase 0 (bit 1): row statistics of every row, and dq, dk, dv zeroed (head dims 8-32: the main
// kernel adds its 16-bit partials straight into them).  Phase 1 (bit 2): zero the f32
// accumulators (head dim 64), run the main kernel and add dbias's batch chunks.  Phase 2 (bit 4):
// head dim 64 converts its accumulators to 16 bits; nothing for the others.  dbias is final
// after phase 1, so a caller can reduce it across GPUs while phase 2 runs.
template <typename T, int D>
int launch_bwd(cudaStream_t st, const DeviceInfo& dev, const void* q, const void* k,
               const void* v, const void* bias, const uint8_t* kmask, const void* out,
               const float* lse, const void* dout, void* dq, void* dk, void* dv, float* dbias,
               uint8_t* ws, int N, int H, int Sq, int Sk, float scale, int phases,
               const RowView* views) {
    using G = Geo<D>;
    constexpr bool kInplace = (D == 64);
    using C = std::conditional_t<kInplace, InplaceCfg<64>, BwdCfg<(D < 64 ? D : 32)>>;
    const BwdWorkspace wl = bwd_workspace(N, H, Sq, Sk, D);
    float* dq_acc = reinterpret_cast<float*>(ws + wl.dq_off);
    float* dk_acc = reinterpret_cast<float*>(ws + wl.dk_off);
    float* dv_acc = reinterpret_cast<float*>(ws + wl.dv_off);
    uint8_t* stats = ws + wl.stat_off;

    BwdParams p;
    p.kmask = kmask;
    p.bias = static_cast<const uint16_t*>(bias);
    p.stats = stats;
    p.N = N;
    p.H = H;
    p.Sq = Sq;
    p.Sk = Sk;
    p.n_it = (Sq + kBM - 1) / kBM;
    p.n_jt = (Sk + kBN - 1) / kBN;
    p.scale = scale;
    p.mask_bits = mask_bias_bits(scale);
    const int64_t base = static_cast<int64_t>(H) * p.n_it * p.n_jt;
    const int64_t nh = static_cast<int64_t>(N) * H;

    const int64_t rq = nh * Sq * D / 8;
    const int64_t rkv = nh * Sk * D / 8;
    const RowStrides out_views[3] = {row_strides(views[5], D), row_strides(views[6], D),
                                     row_strides(views[7], D)};
    if (phases & 1) {
        attn_bwd_prep_kernel<T, D><<<static_cast<unsigned>(nh * p.n_it), 128, 0, st>>>(
            static_cast<const T*>(out), static_cast<const T*>(dout), lse, stats, Sq, p.n_it, scale,
            kInplace ? 0u : p.mask_bits, row_strides(views[3], D), row_strides(views[4], D));
        CFK_TRY(check_launch("attn_bwd_prep"));
        if constexpr (!kInplace) {
            // the outputs (views allowed) the main kernel reduces into
            const ConvertJob zero{{nullptr, nullptr, nullptr},
                                  {dq, dk, dv},
                                  {rq, rkv, rkv},
                                  {out_views[0], out_views[1], out_views[2]},
                                  {1.f, 1.f, 1.f},
                                  {0, 0, 0},
                                  d8_log2(D)};
            f32_to_16_kernel<T><<<dev.num_sms * 8, 256, 0, st>>>(zero);
            CFK_TRY(check_launch("attn_bwd zero"));
        }
    }
    if (phases & 2) {
        CUtensorMap tq, tk, tv, tdo, tdq, tdk, tdv;
        CFK_TRY(make_tmap_rows(&tq, q, views[0], D, kBM, G::kSwizzleBytes, "bwd q"));
        CFK_TRY(make_tmap_rows(&tk, k, views[1], D, kBN, G::kSwizzleBytes, "bwd k"));
        CFK_TRY(make_tmap_rows(&tv, v, views[2], D, kBN, G::kSwizzleBytes, "bwd v"));
        CFK_TRY(make_tmap_rows(&tdo, dout, views[4], D, kBM, G::kSwizzleBytes, "bwd dout"));
        if constexpr (kInplace) {
            if (cudaMemsetAsync(ws, 0, wl.stat_off, st) != cudaSuccess) {
                return fail(CFK_ERR_LAUNCH, "cfk_attn_bwd: memset failed");
            }
            const uint64_t frow = 4ull * D;
            CFK_TRY(make_tmap_3d(&tdq, dq_acc, D, Sq, nh, frow, frow * Sq, C::kPW, kBM, 1,
                                 C::kRowB, "bwd dq acc", true));
            CFK_TRY(make_tmap_3d(&tdk, dk_acc, D, Sk, nh, frow, frow * Sk, C::kPW, kBN, 1,
                                 C::kRowB, "bwd dk acc", true));
            CFK_TRY(make_tmap_3d(&tdv, dv_acc, D, Sk, nh, frow, frow * Sk, C::kPW, kBN, 1,
                                 C::kRowB, "bwd dv acc", true));
        } else {
            // the outputs themselves (zeroed in phase 0); the maps the reduce-adds go through
            // declare the float type (the add is a float add)
            constexpr Map16 kRed = Elem<T>::kBf16 ? Map16::kBF16 : Map16::kF16;
            CFK_TRY(make_tmap_rows(&tdq, dq, views[5], D, kBM, G::kSwizzleBytes, "bwd dq", kRed));
            CFK_TRY(make_tmap_rows(&tdk, dk, views[6], D, kBN, G::kSwizzleBytes, "bwd dk", kRed));
            CFK_TRY(make_tmap_rows(&tdv, dv, views[7], D, kBN, G::kSwizzleBytes, "bwd dv", kRed));
        }
        // batch chunks: as many as fit in one wave of CTAs, within what the workspace holds
        const int64_t nbc = std::min(batch_chunks(N, base, dev.num_sms), wl.max_chunks);
        p.bchunk = static_cast<int>((N + nbc - 1) / nbc);
        p.n_bc = static_cast<int>((N + p.bchunk - 1) / p.bchunk);
        p.items = base * p.n_bc;
        p.b_base = 0;
        p.b_end = N;
        const bool chunked = p.n_bc > 1;
        p.dbias_out = chunked ? reinterpret_cast<float*>(ws + wl.dbp_off) : dbias;
        p.dbias_stride = chunked ? static_cast<int64_t>(H) * Sq * Sk : 0;
        p.dbias_accumulate = 0;
        auto kern = kInplace ? attn_bwd_inplace_kernel<T, 64>
                             : attn_bwd_kernel<T, (D < 64 ? D : 32)>;
        CFK_TRY(ensure_smem_attr(reinterpret_cast<const void*>(kern), dev.device, C::kSmemBytes,
                                 "attn_bwd",
                                 kInplace ? 0 : BwdCfg<(D < 64 ? D : 32)>::kLaunchRegs));
        const int grid = static_cast<int>(std::min<int64_t>(p.items, dev.num_sms));
        kern<<<grid, C::kThreads, C::kSmemBytes, st>>>(tq, tk, tv, tdo, tdq, tdk, tdv, p);
        CFK_TRY(check_launch("attn_bwd"));
        if (chunked) {
            const int64_t n = static_cast<int64_t>(H) * Sq * Sk;
            const int blocks =
                static_cast<int>(std::min<int64_t>((n + 255) / 256, dev.num_sms * 8));
            dbias_chunks_kernel<<<blocks, 256, 0, st>>>(p.dbias_out, dbias, n, p.n_bc, 0);
            CFK_TRY(check_launch("attn_bwd dbias chunks"));
        }
    }
    if (kInplace && (phases & 4)) {
        // the first design's dS carries the softmax scale: no multiplier here
        const ConvertJob job{{dq_acc, dk_acc, dv_acc},
                             {dq, dk, dv},
                             {rq, rkv, rkv},
                             {out_views[0], out_views[1], out_views[2]},
                             {1.f, 1.f, 1.f},
                             {0, 0, 0},
                             d8_log2(D)};
        f32_to_16_kernel<T><<<dev.num_sms * 8, 256, 0, st>>>(job);
        CFK_TRY(check_launch("attn_bwd convert"));
    }
    return CFK_OK;
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
                                   {1.f, 1.f, 1.f},
                                   {0, 0, 0},
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
