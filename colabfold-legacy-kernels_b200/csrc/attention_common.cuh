// attention_common.cuh -- tile geometry and shared-memory operand layouts of the attention
// kernels (forward and backward).
//
// Tiles are 128 queries x 128 keys.  A [128 x D] tile of q, k, v, out or dout sits in shared
// memory as TMA writes it: rows of 2*D bytes under the 2*D-byte swizzle (D = 16, 32, 64), which
// tcgen05.mma reads directly as a K-major operand (the head dim is the contraction) or as an
// MN-major one (the 128 rows are the contraction).  D = 8 rows are 16 bytes, too narrow for a
// swizzle and for the MMA's K and N granularity of 16, so that tile uses the unswizzled
// "interleave" layout with a zero half that pads the head dim to 16.
#pragma once

#include "common.cuh"
#include "host.h"
#include "sm100.cuh"

namespace cfk {
namespace attn {

constexpr int kBM = 128; // queries per tile
constexpr int kBN = 128; // keys per tile

template <int D>
struct Geo {
    static_assert(D == 8 || D == 16 || D == 32 || D == 64, "head dim must be 8, 16, 32 or 64");
    static constexpr int kDp = D < 16 ? 16 : D;     // head dim as seen by the MMA
    static constexpr int kRowBytes = 2 * D;          // one row of a tile
    static constexpr int kTileBytes = 128 * 2 * D;   // what TMA writes for a [128 x D] tile
    static constexpr int kTileAlloc = (D == 8 ? 2 * kTileBytes : kTileBytes); // + zero half
    static constexpr int kSwizzleBytes = D == 8 ? 0 : 2 * D;
    static constexpr uint32_t kLayout =
        D == 8 ? kInterleave : (D == 16 ? kSwizzle32 : (D == 32 ? kSwizzle64 : kSwizzle128));
    static constexpr int kKSteps = kDp / 16; // MMA k-steps over the head dim

    // Tile as the K-major operand [128 rows x kDp] (rows = M or N, head dim = K); k-step s.
    __device__ static __forceinline__ uint64_t kmajor(uint32_t base, int s) {
        if constexpr (D == 8) {
            // core matrices of 8 rows x 16 B; the second 8 columns of K are the zero half
            return smem_desc(base, kTileBytes, 128, kInterleave);
        } else {
            return smem_desc(base + s * 32, 16, 8 * kRowBytes, kLayout);
        }
    }

    // Tile as the MN-major operand [K = 128 rows x N = kDp] (rows = K); k-step s = 16 rows.
    __device__ static __forceinline__ uint64_t mnmajor(uint32_t base, int s) {
        if constexpr (D == 8) {
            // K groups of 8 rows at 128 B; the second 8 columns of N are the zero half
            return smem_desc(base + s * 16 * 16, 128, kTileBytes, kInterleave);
        } else {
            return smem_desc(base + s * 16 * kRowBytes, 8 * kRowBytes * 16, 8 * kRowBytes,
                             kLayout);
        }
    }
};

// A [128 rows x 16] bf16 operand in the interleave layout: element (r, c) at
// (c / 8) * 2048 + r * 16 + (c % 8) * 2.  K-major descriptor.
__device__ __forceinline__ uint64_t interleave16_kmajor(uint32_t base) {
    return smem_desc(base, 2048, 128, kInterleave);
}

// Rows [32*q, 32*q+32) of the 128-lane tensor memory belong to warp q of a warpgroup.
__device__ __forceinline__ uint32_t warp_lane_base() {
    return (threadIdx.x >> 5 & 3u) * 32u;
}

__device__ __forceinline__ uint4 lds128(uint32_t saddr) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "r"(saddr));
    return r;
}

__device__ __forceinline__ uint2 lds64(uint32_t saddr) {
    uint2 r;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "r"(saddr));
    return r;
}

__device__ __forceinline__ void sts128(uint32_t saddr, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(saddr), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

// Byte offset of the 16-byte chunk `c` (8 columns) of row `r` in a [128 x 128] 16-bit tile
// stored as two [128 x 64] panels under the 128-byte swizzle (how TMA writes the bias tile).
__device__ __forceinline__ uint32_t sw128_chunk(int r, int c) {
    return static_cast<uint32_t>((c >> 3) * 16384 + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// Smallest power of two `big` (as a bf16 bit pattern of -big) such that big * scale >= 2^100:
// adding -big to a masked key's score makes its scaled logit ~ -2^100, which exp() turns into
// exactly 0 and max() never picks.  Returns 0 when no such bf16 exists (scale <= 0, NaN, or
// tiny), in which case the kernels exclude masked keys by selection only.
inline uint16_t mask_bias_bits(float scale) {
    if (!(scale > 0.f) || !(scale < 3.0e38f)) {
        return 0;
    }
    int e = 100;
    float s = scale;
    while (s < 1.f && e < 127) {
        s *= 2.f;
        ++e;
    }
    while (s >= 2.f && e > 1) {
        s *= 0.5f;
        --e;
    }
    // big = 2^e with 2^e * scale in [2^100, 2^101)
    if (e > 126) {
        return 0;
    }
    return static_cast<uint16_t>(0x8000u | (static_cast<uint32_t>(e + 127) << 7));
}

// A [N, H, S, D] tensor as the kernels address it: element strides of the batch, head and
// sequence axes (D contiguous) and the extents H, S needed to split a row number.
struct RowStrides {
    int64_t b, h, s;
    int H, S;
    int packed; // b = H S D, h = S D, s = D: row r starts at r D
};

// Element offset of row r = (n H + h) S + i of the view.
__device__ __forceinline__ int64_t view_row_offset(const RowStrides& v, int64_t r, int d) {
    if (v.packed) {
        return r * d;
    }
    int64_t bh, n;
    int i, h;
    if (r < (1ll << 32)) {
        // 32-bit division is much cheaper than 64-bit
        const uint32_t r32 = static_cast<uint32_t>(r);
        const uint32_t bh32 = r32 / static_cast<uint32_t>(v.S);
        i = static_cast<int>(r32 - bh32 * static_cast<uint32_t>(v.S));
        const uint32_t n32 = bh32 / static_cast<uint32_t>(v.H);
        h = static_cast<int>(bh32 - n32 * static_cast<uint32_t>(v.H));
        bh = bh32;
        n = n32;
    } else {
        bh = r / v.S;
        i = static_cast<int>(r - bh * v.S);
        n = bh / v.H;
        h = static_cast<int>(bh - n * v.H);
    }
    return n * v.b + h * v.h + static_cast<int64_t>(i) * v.s;
}

namespace {

// RowStrides of a host-side RowView (host.h) of a tensor with head dim d.
inline RowStrides row_strides(const RowView& v, int64_t d) {
    return RowStrides{v.b, v.h, v.s, static_cast<int>(v.H), static_cast<int>(v.S),
                      is_packed(v, d) ? 1 : 0};
}

// log2(d / 8) for d in {8, 16, 32, 64}
inline int d8_log2(int d) {
    return d == 8 ? 0 : d == 16 ? 1 : d == 32 ? 2 : 3;
}

// dst_t = (16-bit) (mul_t * src_t) for up to three tensors t in one launch, or zeros where src_t
// is NULL: src_t packed f32 [n, H, S_t, D] (n8[t] groups of 8 elements), dst_t written through
// its view starting at row row0[t] (rows of a batch-row range).  8 elements per thread and step;
// D = 8 << d8_log2.
struct ConvertJob {
    const float* src[3];
    void* dst[3];
    int64_t n8[3];
    RowStrides view[3];
    float mul[3];
    int64_t row0[3];
    int d8_log2;
};

template <typename T>
__global__ void f32_to_16_kernel(const ConvertJob job) {
    using E = Elem<T>;
    const int64_t total = job.n8[0] + job.n8[1] + job.n8[2];
    const int d = 8 << job.d8_log2;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int t = 0;
        int64_t k = i;
        if (k >= job.n8[0]) {
            k -= job.n8[0];
            t = 1;
            if (k >= job.n8[1]) {
                k -= job.n8[1];
                t = 2;
            }
        }
        uint4 val = make_uint4(0u, 0u, 0u, 0u);
        if (job.src[t]) {
            const float m = job.mul[t];
            const float4 a = *reinterpret_cast<const float4*>(job.src[t] + k * 8);
            const float4 b = *reinterpret_cast<const float4*>(job.src[t] + k * 8 + 4);
            val = make_uint4(E::pack(a.x * m, a.y * m), E::pack(a.z * m, a.w * m),
                             E::pack(b.x * m, b.y * m), E::pack(b.z * m, b.w * m));
        }
        const int64_t r = (k >> job.d8_log2) + job.row0[t];
        const int c = static_cast<int>(k & ((1 << job.d8_log2) - 1));
        st_global_v4(static_cast<T*>(job.dst[t]) + view_row_offset(job.view[t], r, d) + c * 8,
                     val);
    }
}

} // namespace

} // namespace attn
} // namespace cfk
