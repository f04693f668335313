// gate.cu -- the sigmoid gate of the Evoformer's attention modules, fused:
//
//   forward   y  = sigmoid(g) * o
//   backward  do = dy * sigmoid(g),   dg = dy * o * sigmoid(g) * (1 - sigmoid(g))
//
// g (the gate's pre-activation, x Wg + bg), o (the attention output), y, dy, do, dg are 16-bit
// tensors of n elements; the arithmetic is f32 and each output is rounded once.  The modules
// otherwise run this as three to five separate elementwise passes; here the forward reads g and
// o and writes y once, the backward reads dy, g, o and writes do, dg once.  HBM-bound: 6 bytes
// per element forward, 10 backward.  No counterpart in the reference (its caller's jnp code).

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <initializer_list>

#include "common.cuh"
#include "host.h"
#include "sm100.cuh"

namespace cfk {
namespace {

__device__ __forceinline__ float gate_sigmoid(float x) {
    return rcp_approx(1.0f + ex2(-x * kLog2e));
}

// 8 elements (one 16-byte vector of each tensor) per thread and step; n8 vectors, then a tail
// of n % 8 elements handled one per thread.
template <typename T>
__global__ void gate_fwd_kernel(const uint16_t* __restrict__ g, const uint16_t* __restrict__ o,
                                uint16_t* __restrict__ y, int64_t n) {
    using E = Elem<T>;
    const int64_t n8 = n / 8;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
         i += stride) {
        const uint4 gv = ld_global_nc_v4(g + i * 8);
        const uint4 ov = ld_global_nc_v4(o + i * 8);
        const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
        const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w};
        uint32_t yw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 gf = E::to_float2(gw[e]);
            const float2 of = E::to_float2(ow[e]);
            yw[e] = E::pack(gate_sigmoid(gf.x) * of.x, gate_sigmoid(gf.y) * of.y);
        }
        st_global_v4(y + i * 8, make_uint4(yw[0], yw[1], yw[2], yw[3]));
    }
    for (int64_t i = n8 * 8 + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
         i < n; i += stride) {
        y[i] = E::from_float(gate_sigmoid(E::to_float(g[i])) * E::to_float(o[i]));
    }
}

template <typename T>
__global__ void gate_bwd_kernel(const uint16_t* __restrict__ g, const uint16_t* __restrict__ o,
                                const uint16_t* __restrict__ dy, uint16_t* __restrict__ d_o,
                                uint16_t* __restrict__ dg, int64_t n) {
    using E = Elem<T>;
    const int64_t n8 = n / 8;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
         i += stride) {
        const uint4 gv = ld_global_nc_v4(g + i * 8);
        const uint4 ov = ld_global_nc_v4(o + i * 8);
        const uint4 dv = ld_global_nc_v4(dy + i * 8);
        const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
        const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w};
        const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w};
        uint32_t ow_out[4], gw_out[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 gf = E::to_float2(gw[e]);
            const float2 of = E::to_float2(ow[e]);
            const float2 df = E::to_float2(dw[e]);
            const float s0 = gate_sigmoid(gf.x), s1 = gate_sigmoid(gf.y);
            ow_out[e] = E::pack(df.x * s0, df.y * s1);
            gw_out[e] = E::pack(df.x * of.x * s0 * (1.0f - s0), df.y * of.y * s1 * (1.0f - s1));
        }
        st_global_v4(d_o + i * 8, make_uint4(ow_out[0], ow_out[1], ow_out[2], ow_out[3]));
        st_global_v4(dg + i * 8, make_uint4(gw_out[0], gw_out[1], gw_out[2], gw_out[3]));
    }
    for (int64_t i = n8 * 8 + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
         i < n; i += stride) {
        const float s = gate_sigmoid(E::to_float(g[i]));
        const float d = E::to_float(dy[i]);
        d_o[i] = E::from_float(d * s);
        dg[i] = E::from_float(d * E::to_float(o[i]) * s * (1.0f - s));
    }
}

int check_gate_args(const char* fn, int dtype, int64_t n, std::initializer_list<const void*> ptrs) {
    if (dtype != CFK_F16 && dtype != CFK_BF16) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: dtype must be CFK_F16 or CFK_BF16", fn);
    }
    if (n < 0) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: negative element count", fn);
    }
    for (const void* p : ptrs) {
        if (n > 0 && (!p || !aligned16(p))) {
            return fail(CFK_ERR_INVALID_ARGUMENT, "%s: every buffer must be non-null and 16-byte "
                        "aligned", fn);
        }
    }
    return CFK_OK;
}

int gate_grid(const DeviceInfo& dev, int64_t n) {
    const int64_t want = (n / 8 + 255) / 256;
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, dev.num_sms * 8)));
}

} // namespace
} // namespace cfk

using namespace cfk;

extern "C" int cfk_gate_fwd(cfk_stream_t stream, cfk_dtype dtype, const void* g, const void* o,
                            void* y, int64_t n) {
    clear_error();
    CFK_TRY(check_gate_args("cfk_gate_fwd", dtype, n, {g, o, y}));
    if (n == 0) {
        return CFK_OK;
    }
    DeviceInfo dev;
    CFK_TRY(current_device(&dev));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const auto* gp = static_cast<const uint16_t*>(g);
    const auto* op = static_cast<const uint16_t*>(o);
    auto* yp = static_cast<uint16_t*>(y);
    if (dtype == CFK_BF16) {
        gate_fwd_kernel<__nv_bfloat16><<<gate_grid(dev, n), 256, 0, st>>>(gp, op, yp, n);
    } else {
        gate_fwd_kernel<__half><<<gate_grid(dev, n), 256, 0, st>>>(gp, op, yp, n);
    }
    return check_launch("gate_fwd");
}

extern "C" int cfk_gate_bwd(cfk_stream_t stream, cfk_dtype dtype, const void* g, const void* o,
                            const void* dy, void* d_o, void* dg, int64_t n) {
    clear_error();
    CFK_TRY(check_gate_args("cfk_gate_bwd", dtype, n, {g, o, dy, d_o, dg}));
    if (n == 0) {
        return CFK_OK;
    }
    DeviceInfo dev;
    CFK_TRY(current_device(&dev));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const auto* gp = static_cast<const uint16_t*>(g);
    const auto* op = static_cast<const uint16_t*>(o);
    const auto* dp = static_cast<const uint16_t*>(dy);
    auto* dop = static_cast<uint16_t*>(d_o);
    auto* dgp = static_cast<uint16_t*>(dg);
    if (dtype == CFK_BF16) {
        gate_bwd_kernel<__nv_bfloat16><<<gate_grid(dev, n), 256, 0, st>>>(gp, op, dp, dop, dgp, n);
    } else {
        gate_bwd_kernel<__half><<<gate_grid(dev, n), 256, 0, st>>>(gp, op, dp, dop, dgp, n);
    }
    return check_launch("gate_bwd");
}
