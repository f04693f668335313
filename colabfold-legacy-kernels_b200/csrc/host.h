// host.h -- host-side helpers shared by the C ABI entry points: error reporting, per-device
// property caches, one-time kernel attributes and TMA tensor-map encoding.
#pragma once

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "cfk.h"

namespace cfk {

// Records a printf-style message as the calling thread's last error and returns `code`.
int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));

// Clears the calling thread's last error.
void clear_error();

struct DeviceInfo {
    int device = -1;
    int cc = 0;        // major * 10 + minor
    int num_sms = 0;
    int max_smem_optin = 0;
};

// Looks up the current device (cached per device, thread-safe).  Fails with
// CFK_ERR_UNSUPPORTED_DEVICE unless it is compute capability 10.0.
int current_device(DeviceInfo* info);

// Sets cudaFuncAttributeMaxDynamicSharedMemorySize once per (kernel, device).
// launch_regs > 0: the kernel moves registers between its warpgroups with setmaxnreg and must
// have been built with exactly that many registers per thread (checked once, else an error).
int ensure_smem_attr(const void* kernel, int device, int bytes, const char* name,
                     int launch_regs = 0);

// Maps cudaGetLastError() after a launch onto CFK_ERR_LAUNCH.
int check_launch(const char* what);

// TMA descriptor for a rank-3 tensor with dims (innermost first) d0, d1, d2 and byte strides of
// dims 1 and 2; box b0 x b1 x b2; 16-bit elements; out-of-bounds elements read as zero.
// swizzle_bytes is 0 (none), 32, 64 or 128.
int make_tmap_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                 uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1,
                 uint32_t b2, int swizzle_bytes, const char* what, bool f32 = false);

// A [N, H, S, D] tensor of 16-bit elements whose D axis is contiguous: its extents and the
// element strides of its batch, head and sequence axes.  A packed tensor has b = H S D,
// h = S D, s = D; a transposed view (attention over the other residue axis, or a [N, S, H, D]
// layout) only changes the strides.
struct RowView {
    int64_t N, H, S;
    int64_t b, h, s;
};

inline RowView packed_view(int64_t N, int64_t H, int64_t S, int64_t D) {
    return RowView{N, H, S, H * S * D, S * D, D};
}

inline bool is_packed(const RowView& v, int64_t D) {
    return (v.S <= 1 || v.s == D) && (v.H <= 1 || v.h == v.S * D) &&
           (v.N <= 1 || v.b == v.H * v.S * D);
}

// RowView of `user` (NULL = packed) with the checks the kernels rely on: every stride of an
// axis longer than 1 a positive multiple of 8 elements (16 bytes, so every row starts 16-byte
// aligned for TMA and vector access) and below 2^38, and the view's last element below 2^40.
int view_of(const char* fn, const char* name, const cfk_view* user, int64_t N, int64_t H,
            int64_t S, int64_t D, RowView* out);

// Element type a 16-bit tensor map declares: raw 16-bit words (loads and stores, where the type
// does not matter), or bf16 / f16 for a map that TMA reduce-adds into (the add needs the float
// type; an integer 16-bit add is not an operation the TMA unit has).
enum class Map16 { kBits, kBF16, kF16 };

// TMA descriptor over a RowView: dims (D, S, H, N), box D x box_rows x 1 x 1, 16-bit elements,
// out-of-bounds rows read as zero (and are not written by stores or reductions).
int make_tmap_rows(CUtensorMap* map, const void* base, const RowView& v, uint64_t d,
                   uint32_t box_rows, int swizzle_bytes, const char* what,
                   Map16 type = Map16::kBits);

// Argument checks shared by the attention entry points (dtype code, ranks, D in {8,16,32,64}).
int check_attn_args(const char* fn, int dtype, int64_t N, int64_t H, int64_t Sq, int64_t Sk,
                    int64_t D);

inline bool aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

} // namespace cfk

#define CFK_TRY(expr)                                                                              \
    do {                                                                                           \
        int cfk_rc_ = (expr);                                                                      \
        if (cfk_rc_ != CFK_OK) {                                                                   \
            return cfk_rc_;                                                                        \
        }                                                                                          \
    } while (0)
