// layer_norm.cu -- LayerNorm forward and backward over the last axis.
//
// Semantics follow volta_layer_norm_kernel (cuda/volta_ops.cu:28-60): 16-bit x and y, f32
// gamma/beta and statistics, rstd = rsqrt(var + eps).  The variance is the two-pass
// mean((x - mean)^2) computed from registers; the reference's E[x^2] - mean^2 (volta_ops.cu:53)
// equals it up to f32 rounding and loses precision when |mean| >> std.
//
// The kernels are HBM-bound.  The fast path gives each row LPR lanes that each hold NV 16-byte
// vectors (C = LPR * NV * 8), so every access is a coalesced 128-bit load or store and the row
// statistics need only log2(LPR) shuffles.  Each warp keeps U row groups in flight to cover
// DRAM latency.  Any other C takes a warp-per-row path with scalar accesses.
#include <algorithm>
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "host.h"

namespace cfk {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

template <int LPR>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int off = LPR / 2; off > 0; off >>= 1) {
        v += __shfl_xor_sync(0xffffffffu, v, off);
    }
    return v;
}

// ------------------------------------------------------------------------------------------
// Forward, vectorised
// ------------------------------------------------------------------------------------------
template <typename T, int LPR, int NV, int U>
__global__ __launch_bounds__(kThreads) void ln_fwd_vec_kernel(
    const T* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
    T* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ rstd_out, int64_t M,
    float eps) {
    constexpr int C = LPR * NV * 8;
    constexpr int RPW = 32 / LPR; // rows per warp and step
    using E = Elem<T>;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int g = lane / LPR;  // row group of this lane
    const int gl = lane % LPR; // lane within the row group

    float gm[NV * 8], bt[NV * 8];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int c = (v * LPR + gl) * 8 + e;
            gm[v * 8 + e] = gamma[c];
            bt[v * 8 + e] = beta[c];
        }
    }

    const int64_t rows_per_step = static_cast<int64_t>(RPW) * U;
    const int64_t nsteps = (M + rows_per_step - 1) / rows_per_step;
    for (int64_t step = static_cast<int64_t>(blockIdx.x) * kWarps + warp; step < nsteps;
         step += static_cast<int64_t>(gridDim.x) * kWarps) {
        const int64_t row0 = step * rows_per_step;
        uint4 raw[U][NV];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t row = row0 + u * RPW + g;
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                raw[u][v] = (row < M) ? ld_global_stream_v4(x + row * C + (v * LPR + gl) * 8)
                                      : make_uint4(0, 0, 0, 0);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t row = row0 + u * RPW + g;
            float xv[NV * 8];
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                const uint32_t w[4] = {raw[u][v].x, raw[u][v].y, raw[u][v].z, raw[u][v].w};
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    const float2 f = E::to_float2(w[p]);
                    xv[v * 8 + 2 * p] = f.x;
                    xv[v * 8 + 2 * p + 1] = f.y;
                }
            }
            float s = 0.f;
#pragma unroll
            for (int e = 0; e < NV * 8; ++e) {
                s += xv[e];
            }
            const float mean = group_sum<LPR>(s) * (1.0f / C);
            float q = 0.f;
#pragma unroll
            for (int e = 0; e < NV * 8; ++e) {
                const float d = xv[e] - mean;
                q = __fmaf_rn(d, d, q);
            }
            const float var = group_sum<LPR>(q) * (1.0f / C);
            const float rstd = rsqrtf(var + eps);
            if (row < M) {
#pragma unroll
                for (int v = 0; v < NV; ++v) {
                    uint32_t w[4];
#pragma unroll
                    for (int p = 0; p < 4; ++p) {
                        const int e0 = v * 8 + 2 * p;
                        // explicit roundings: every unrolled row group evaluates the same
                        // operations, so a row's result does not depend on its place in the call
                        const float y0 = __fmaf_rn(__fmul_rn(__fsub_rn(xv[e0], mean), rstd),
                                                   gm[e0], bt[e0]);
                        const float y1 = __fmaf_rn(__fmul_rn(__fsub_rn(xv[e0 + 1], mean), rstd),
                                                   gm[e0 + 1], bt[e0 + 1]);
                        w[p] = E::pack(y0, y1);
                    }
                    st_global_v4(y + row * C + (v * LPR + gl) * 8, make_uint4(w[0], w[1], w[2], w[3]));
                }
                if (gl == 0) {
                    if (mean_out) {
                        mean_out[row] = mean;
                    }
                    if (rstd_out) {
                        rstd_out[row] = rstd;
                    }
                }
            }
        }
    }
}

// ------------------------------------------------------------------------------------------
// Forward, any C: one warp per row, scalar accesses.
// ------------------------------------------------------------------------------------------
template <typename T>
__global__ __launch_bounds__(kThreads) void ln_fwd_generic_kernel(
    const T* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
    T* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ rstd_out, int64_t M,
    int C, float eps) {
    using E = Elem<T>;
    const int lane = threadIdx.x & 31;
    const uint16_t* xs = reinterpret_cast<const uint16_t*>(x);
    uint16_t* ys = reinterpret_cast<uint16_t*>(y);
    for (int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5); row < M;
         row += static_cast<int64_t>(gridDim.x) * kWarps) {
        const uint16_t* xr = xs + row * C;
        float s = 0.f;
        for (int c = lane; c < C; c += 32) {
            s += E::to_float(xr[c]);
        }
        const float mean = group_sum<32>(s) / C;
        float q = 0.f;
        for (int c = lane; c < C; c += 32) {
            const float d = E::to_float(xr[c]) - mean;
            q = __fmaf_rn(d, d, q);
        }
        const float rstd = rsqrtf(group_sum<32>(q) / C + eps);
        for (int c = lane; c < C; c += 32) {
            ys[row * C + c] = E::from_float((E::to_float(xr[c]) - mean) * rstd * gamma[c] + beta[c]);
        }
        if (lane == 0) {
            if (mean_out) {
                mean_out[row] = mean;
            }
            if (rstd_out) {
                rstd_out[row] = rstd;
            }
        }
    }
}

// ------------------------------------------------------------------------------------------
// Backward, vectorised.  Each CTA writes its partial dgamma/dbeta to partial[blockIdx][2C].
// ------------------------------------------------------------------------------------------
template <typename T, int LPR, int NV, int U>
__global__ __launch_bounds__(kThreads) void ln_bwd_vec_kernel(
    const T* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ mean_in,
    const float* __restrict__ rstd_in, const T* __restrict__ dy, T* __restrict__ dx,
    float* __restrict__ partial, int64_t M, float eps) {
    constexpr int C = LPR * NV * 8;
    constexpr int RPW = 32 / LPR;
    using E = Elem<T>;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int g = lane / LPR;
    const int gl = lane % LPR;

    float gm[NV * 8], dg[NV * 8], db[NV * 8];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            gm[v * 8 + e] = gamma[(v * LPR + gl) * 8 + e];
            dg[v * 8 + e] = 0.f;
            db[v * 8 + e] = 0.f;
        }
    }

    const int64_t rows_per_step = static_cast<int64_t>(RPW) * U;
    const int64_t nsteps = (M + rows_per_step - 1) / rows_per_step;
    for (int64_t step = static_cast<int64_t>(blockIdx.x) * kWarps + warp; step < nsteps;
         step += static_cast<int64_t>(gridDim.x) * kWarps) {
        const int64_t row0 = step * rows_per_step;
        uint4 rx[U][NV], rd[U][NV];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t row = row0 + u * RPW + g;
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                const int64_t off = row * C + (v * LPR + gl) * 8;
                rx[u][v] = (row < M) ? ld_global_stream_v4(x + off) : make_uint4(0, 0, 0, 0);
                rd[u][v] = (row < M) ? ld_global_stream_v4(dy + off) : make_uint4(0, 0, 0, 0);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t row = row0 + u * RPW + g;
            float xv[NV * 8], dv[NV * 8];
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                const uint32_t wx[4] = {rx[u][v].x, rx[u][v].y, rx[u][v].z, rx[u][v].w};
                const uint32_t wd[4] = {rd[u][v].x, rd[u][v].y, rd[u][v].z, rd[u][v].w};
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    const float2 fx = E::to_float2(wx[p]);
                    const float2 fd = E::to_float2(wd[p]);
                    xv[v * 8 + 2 * p] = fx.x;
                    xv[v * 8 + 2 * p + 1] = fx.y;
                    dv[v * 8 + 2 * p] = fd.x;
                    dv[v * 8 + 2 * p + 1] = fd.y;
                }
            }
            float mean, rstd;
            if (mean_in && rstd_in) {
                const int64_t r = row < M ? row : 0;
                mean = mean_in[r];
                rstd = rstd_in[r];
            } else {
                float s = 0.f;
#pragma unroll
                for (int e = 0; e < NV * 8; ++e) {
                    s += xv[e];
                }
                mean = group_sum<LPR>(s) * (1.0f / C);
                float q = 0.f;
#pragma unroll
                for (int e = 0; e < NV * 8; ++e) {
                    const float d = xv[e] - mean;
                    q = __fmaf_rn(d, d, q);
                }
                rstd = rsqrtf(group_sum<LPR>(q) * (1.0f / C) + eps);
            }
            // g = dy * gamma; dx = rstd * (g - mean(g) - xhat * mean(g * xhat))
            float sg = 0.f, sgx = 0.f;
#pragma unroll
            for (int e = 0; e < NV * 8; ++e) {
                const float xh = __fmul_rn(__fsub_rn(xv[e], mean), rstd);
                const float gg = __fmul_rn(dv[e], gm[e]);
                xv[e] = xh;
                sg += gg;
                sgx = __fmaf_rn(gg, xh, sgx);
            }
            sg = group_sum<LPR>(sg) * (1.0f / C);
            sgx = group_sum<LPR>(sgx) * (1.0f / C);
            if (row < M) {
#pragma unroll
                for (int v = 0; v < NV; ++v) {
                    uint32_t w[4];
#pragma unroll
                    for (int p = 0; p < 4; ++p) {
                        const int e0 = v * 8 + 2 * p;
                        // explicit roundings (see the forward)
                        const float d0 = __fmul_rn(
                            rstd, __fmaf_rn(-xv[e0], sgx,
                                            __fsub_rn(__fmul_rn(dv[e0], gm[e0]), sg)));
                        const float d1 = __fmul_rn(
                            rstd, __fmaf_rn(-xv[e0 + 1], sgx,
                                            __fsub_rn(__fmul_rn(dv[e0 + 1], gm[e0 + 1]), sg)));
                        w[p] = E::pack(d0, d1);
                    }
                    st_global_v4(dx + row * C + (v * LPR + gl) * 8, make_uint4(w[0], w[1], w[2], w[3]));
                }
#pragma unroll
                for (int e = 0; e < NV * 8; ++e) {
                    dg[e] = __fmaf_rn(dv[e], xv[e], dg[e]);
                    db[e] += dv[e];
                }
            }
        }
    }

    // Reduce the RPW row groups of the warp, then the warps of the CTA.
#pragma unroll
    for (int e = 0; e < NV * 8; ++e) {
#pragma unroll
        for (int off = LPR; off < 32; off <<= 1) {
            dg[e] += __shfl_xor_sync(0xffffffffu, dg[e], off);
            db[e] += __shfl_xor_sync(0xffffffffu, db[e], off);
        }
    }
    // Two rounds (dgamma, then dbeta) through a [kWarps][C] buffer keep the static shared
    // memory at 32 KB for C = 1024.
    __shared__ float red[kWarps][C];
#pragma unroll
    for (int round = 0; round < 2; ++round) {
        if (g == 0) {
#pragma unroll
            for (int v = 0; v < NV; ++v) {
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    red[warp][(v * LPR + gl) * 8 + e] = round == 0 ? dg[v * 8 + e] : db[v * 8 + e];
                }
            }
        }
        __syncthreads();
        for (int c = threadIdx.x; c < C; c += kThreads) {
            float s = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                s += red[w][c];
            }
            partial[static_cast<int64_t>(blockIdx.x) * 2 * C + round * C + c] = s;
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------------------------------------
// Backward, any C: one warp per row.
// ------------------------------------------------------------------------------------------
template <typename T>
__global__ __launch_bounds__(kThreads) void ln_bwd_generic_kernel(
    const T* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ mean_in,
    const float* __restrict__ rstd_in, const T* __restrict__ dy, T* __restrict__ dx,
    float* __restrict__ partial, int64_t M, int C, float eps) {
    using E = Elem<T>;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const uint16_t* xs = reinterpret_cast<const uint16_t*>(x);
    const uint16_t* ds = reinterpret_cast<const uint16_t*>(dy);
    uint16_t* dxs = reinterpret_cast<uint16_t*>(dx);
    extern __shared__ float acc[]; // [kWarps][2C]
    for (int c = threadIdx.x; c < kWarps * 2 * C; c += kThreads) {
        acc[c] = 0.f;
    }
    __syncthreads();
    float* my = acc + warp * 2 * C;
    for (int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + warp; row < M;
         row += static_cast<int64_t>(gridDim.x) * kWarps) {
        const uint16_t* xr = xs + row * C;
        const uint16_t* dr = ds + row * C;
        float mean, rstd;
        if (mean_in && rstd_in) {
            mean = mean_in[row];
            rstd = rstd_in[row];
        } else {
            float s = 0.f;
            for (int c = lane; c < C; c += 32) {
                s += E::to_float(xr[c]);
            }
            mean = group_sum<32>(s) / C;
            float q = 0.f;
            for (int c = lane; c < C; c += 32) {
                const float d = E::to_float(xr[c]) - mean;
                q = __fmaf_rn(d, d, q);
            }
            rstd = rsqrtf(group_sum<32>(q) / C + eps);
        }
        float sg = 0.f, sgx = 0.f;
        for (int c = lane; c < C; c += 32) {
            const float xh = (E::to_float(xr[c]) - mean) * rstd;
            const float gg = E::to_float(dr[c]) * gamma[c];
            sg += gg;
            sgx += gg * xh;
        }
        sg = group_sum<32>(sg) / C;
        sgx = group_sum<32>(sgx) / C;
        for (int c = lane; c < C; c += 32) {
            const float xh = (E::to_float(xr[c]) - mean) * rstd;
            const float d = E::to_float(dr[c]);
            dxs[row * C + c] = E::from_float(rstd * (d * gamma[c] - sg - xh * sgx));
            my[c] += d * xh;
            my[C + c] += d;
        }
    }
    __syncthreads();
    for (int c = threadIdx.x; c < 2 * C; c += kThreads) {
        float s = 0.f;
        for (int w = 0; w < kWarps; ++w) {
            s += acc[w * 2 * C + c];
        }
        partial[static_cast<int64_t>(blockIdx.x) * 2 * C + c] = s;
    }
}

// Sums the per-CTA partials in a fixed order: dgamma = sum_b partial[b][c],
// dbeta = sum_b partial[b][C + c].  A CTA of 32 warps owns 32 columns: warp w adds the partials
// b = w, w + 32, ... (lane = column, coalesced rows, four chains in flight), then warp 0 adds the
// 32 warp sums in warp order, so the result does not depend on timing.
constexpr int kReduceWarps = 32;

__global__ void __launch_bounds__(kReduceWarps * 32)
    ln_bwd_reduce_kernel(const float* __restrict__ partial, int nparts, int C,
                         float* __restrict__ dgamma, float* __restrict__ dbeta) {
    __shared__ float red[kReduceWarps][33];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x * 32 + lane;
    const int64_t stride = 2 * static_cast<int64_t>(C);
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    if (c < 2 * C) {
        int b = warp;
        for (; b + 3 * kReduceWarps < nparts; b += 4 * kReduceWarps) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                s[u] += partial[(b + u * kReduceWarps) * stride + c];
            }
        }
        for (int u = 0; b < nparts; b += kReduceWarps, ++u) {
            s[u & 3] += partial[b * stride + c];
        }
    }
    red[warp][lane] = (s[0] + s[1]) + (s[2] + s[3]);
    __syncthreads();
    if (warp == 0 && c < 2 * C) {
        float t = 0.f;
        for (int w = 0; w < kReduceWarps; ++w) {
            t += red[w][lane];
        }
        if (c < C) {
            dgamma[c] = t;
        } else {
            dbeta[c - C] = t;
        }
    }
}

// ------------------------------------------------------------------------------------------
// Dispatch
// ------------------------------------------------------------------------------------------
constexpr int kU = 4; // row groups in flight per warp

// Largest number of CTAs of a backward launch (8 per SM on up to 160 SMs).
constexpr int kMaxPartials = 160 * 8;

struct VecShape {
    int lpr;
    int nv;
};

// The (LPR, NV) shapes compiled for the vectorised path.
bool vec_shape(int64_t C, VecShape* s) {
    switch (C) {
    case 64:
        *s = {8, 1};
        return true;
    case 128:
        *s = {16, 1};
        return true;
    case 256:
        *s = {32, 1};
        return true;
    case 384:
        *s = {16, 3};
        return true;
    case 512:
        *s = {32, 2};
        return true;
    case 768:
        *s = {32, 3};
        return true;
    case 1024:
        *s = {32, 4};
        return true;
    default:
        return false;
    }
}

int grid_for(int64_t nsteps, const DeviceInfo& d) {
    const int64_t want = (nsteps + kWarps - 1) / kWarps;
    const int64_t cap = std::min<int64_t>(static_cast<int64_t>(d.num_sms) * 8, kMaxPartials);
    return static_cast<int>(std::max<int64_t>(1, std::min(want, cap)));
}

// Number of CTAs (and f32 [2C] partials) of the backward launch, capped at kMaxPartials so
// that the workspace size can be known without a device.
int ln_partials(int64_t M, int64_t C, const DeviceInfo* d) {
    VecShape s;
    const int sms = d ? d->num_sms : kMaxPartials / 8;
    int64_t nsteps;
    if (vec_shape(C, &s)) {
        const int64_t rps = static_cast<int64_t>(32 / s.lpr) * kU;
        nsteps = (M + rps - 1) / rps;
    } else {
        nsteps = M;
    }
    const int64_t want = (nsteps + kWarps - 1) / kWarps;
    const int64_t cap = static_cast<int64_t>(sms) * 8;
    return static_cast<int>(std::max<int64_t>(1, std::min(want, cap)));
}

template <typename T>
int ln_fwd_impl(cudaStream_t st, const DeviceInfo& d, const void* x, const float* gamma,
                const float* beta, void* y, float* mean, float* rstd, int64_t M, int64_t C,
                float eps) {
    VecShape s;
    const T* xp = static_cast<const T*>(x);
    T* yp = static_cast<T*>(y);
    if (vec_shape(C, &s) && aligned16(x) && aligned16(y)) {
        const int64_t rps = static_cast<int64_t>(32 / s.lpr) * kU;
        const int grid = grid_for((M + rps - 1) / rps, d);
#define CFK_LN_FWD(LPR, NV)                                                                        \
    if (s.lpr == LPR && s.nv == NV) {                                                              \
        ln_fwd_vec_kernel<T, LPR, NV, kU>                                                          \
            <<<grid, kThreads, 0, st>>>(xp, gamma, beta, yp, mean, rstd, M, eps);                  \
        return check_launch("ln_fwd");                                                             \
    }
        CFK_LN_FWD(8, 1)
        CFK_LN_FWD(16, 1)
        CFK_LN_FWD(32, 1)
        CFK_LN_FWD(16, 3)
        CFK_LN_FWD(32, 2)
        CFK_LN_FWD(32, 3)
        CFK_LN_FWD(32, 4)
#undef CFK_LN_FWD
    }
    const int grid = grid_for(M, d);
    ln_fwd_generic_kernel<T><<<grid, kThreads, 0, st>>>(xp, gamma, beta, yp, mean, rstd, M,
                                                         static_cast<int>(C), eps);
    return check_launch("ln_fwd");
}

template <typename T>
int ln_bwd_impl(cudaStream_t st, const DeviceInfo& d, const void* x, const float* gamma,
                const float* mean, const float* rstd, const void* dy, void* dx, float* dgamma,
                float* dbeta, float* partial, int64_t M, int64_t C, float eps) {
    VecShape s;
    const T* xp = static_cast<const T*>(x);
    const T* dyp = static_cast<const T*>(dy);
    T* dxp = static_cast<T*>(dx);
    int grid = 0;
    bool launched = false;
    if (vec_shape(C, &s) && aligned16(x) && aligned16(dy) && aligned16(dx)) {
        const int64_t rps = static_cast<int64_t>(32 / s.lpr) * kU;
        grid = grid_for((M + rps - 1) / rps, d);
#define CFK_LN_BWD(LPR, NV)                                                                        \
    if (!launched && s.lpr == LPR && s.nv == NV) {                                                 \
        ln_bwd_vec_kernel<T, LPR, NV, kU>                                                          \
            <<<grid, kThreads, 0, st>>>(xp, gamma, mean, rstd, dyp, dxp, partial, M, eps);         \
        launched = true;                                                                           \
    }
        CFK_LN_BWD(8, 1)
        CFK_LN_BWD(16, 1)
        CFK_LN_BWD(32, 1)
        CFK_LN_BWD(16, 3)
        CFK_LN_BWD(32, 2)
        CFK_LN_BWD(32, 3)
        CFK_LN_BWD(32, 4)
#undef CFK_LN_BWD
    }
    if (!launched) {
        grid = grid_for(M, d);
        const int smem = kWarps * 2 * static_cast<int>(C) * static_cast<int>(sizeof(float));
        if (smem > 48 * 1024) {
            CFK_TRY(ensure_smem_attr(reinterpret_cast<const void*>(&ln_bwd_generic_kernel<T>),
                                     d.device, smem, "ln_bwd"));
        }
        ln_bwd_generic_kernel<T><<<grid, kThreads, smem, st>>>(xp, gamma, mean, rstd, dyp, dxp,
                                                               partial, M, static_cast<int>(C), eps);
    }
    CFK_TRY(check_launch("ln_bwd"));
    const int blocks = static_cast<int>((2 * C + 31) / 32);
    ln_bwd_reduce_kernel<<<blocks, kReduceWarps * 32, 0, st>>>(partial, grid, static_cast<int>(C),
                                                               dgamma, dbeta);
    return check_launch("ln_bwd_reduce");
}

int check_ln_args(const char* fn, int dtype, int64_t M, int64_t C, float eps) {
    if (dtype != CFK_F16 && dtype != CFK_BF16) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: dtype must be CFK_F16 or CFK_BF16", fn);
    }
    if (M < 0 || C <= 0) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: x must be [M,C] with C > 0 (got M=%lld C=%lld)",
                    fn, static_cast<long long>(M), static_cast<long long>(C));
    }
    // The backward's generic path keeps 2*C floats per warp in shared memory.
    if (C > 3072) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: C=%lld exceeds the supported 3072", fn,
                    static_cast<long long>(C));
    }
    if (!(eps >= 0.f)) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: eps must be >= 0", fn);
    }
    return CFK_OK;
}

} // namespace
} // namespace cfk

using namespace cfk;

extern "C" int cfk_ln_fwd(cfk_stream_t stream, cfk_dtype dtype, const void* x,
                          const float* gamma, const float* beta, void* y, float* mean, float* rstd,
                          int64_t M, int64_t C, float eps) {
    clear_error();
    CFK_TRY(check_ln_args("cfk_ln_fwd", dtype, M, C, eps));
    if (M == 0) {
        return CFK_OK;
    }
    if (!x || !gamma || !beta || !y) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_ln_fwd: null buffer");
    }
    DeviceInfo d;
    CFK_TRY(current_device(&d));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    return dtype == CFK_BF16
               ? ln_fwd_impl<__nv_bfloat16>(st, d, x, gamma, beta, y, mean, rstd, M, C, eps)
               : ln_fwd_impl<__half>(st, d, x, gamma, beta, y, mean, rstd, M, C, eps);
}

extern "C" int cfk_ln_bwd_workspace_size(int64_t M, int64_t C, size_t* bytes) {
    clear_error();
    if (!bytes || M < 0 || C <= 0) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_ln_bwd_workspace_size: bad arguments");
    }
    // One f32 [2C] partial per CTA; the launch uses at most min(rows, 8 per SM) CTAs.
    const int64_t parts = ln_partials(M, C, nullptr);
    *bytes = static_cast<size_t>(parts) * 2 * static_cast<size_t>(C) * sizeof(float);
    return CFK_OK;
}

extern "C" int cfk_ln_bwd(cfk_stream_t stream, cfk_dtype dtype, const void* x,
                          const float* gamma, const float* mean, const float* rstd, const void* dy,
                          void* dx, float* dgamma, float* dbeta, void* workspace,
                          size_t workspace_bytes, int64_t M, int64_t C, float eps) {
    clear_error();
    CFK_TRY(check_ln_args("cfk_ln_bwd", dtype, M, C, eps));
    if (!gamma || !dgamma || !dbeta) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_ln_bwd: null buffer");
    }
    if ((mean == nullptr) != (rstd == nullptr)) {
        return fail(CFK_ERR_INVALID_ARGUMENT,
                    "cfk_ln_bwd: give both mean and rstd, or neither to recompute them");
    }
    DeviceInfo d;
    CFK_TRY(current_device(&d));
    if (d.num_sms * 8 > kMaxPartials) {
        return fail(CFK_ERR_UNSUPPORTED_DEVICE, "cfk_ln_bwd: device has too many SMs");
    }
    size_t need = 0;
    cfk_ln_bwd_workspace_size(M, C, &need);
    if (!workspace || workspace_bytes < need || !aligned16(workspace)) {
        return fail(CFK_ERR_INVALID_ARGUMENT,
                    "cfk_ln_bwd: workspace must be 16-byte aligned and hold %zu bytes (got %zu)",
                    need, workspace_bytes);
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (M == 0) {
        cudaError_t e1 = cudaMemsetAsync(dgamma, 0, C * sizeof(float), st);
        cudaError_t e2 = cudaMemsetAsync(dbeta, 0, C * sizeof(float), st);
        if (e1 != cudaSuccess || e2 != cudaSuccess) {
            return fail(CFK_ERR_LAUNCH, "cfk_ln_bwd: memset failed");
        }
        return CFK_OK;
    }
    if (!x || !dy || !dx) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_ln_bwd: null buffer");
    }
    float* partial = static_cast<float*>(workspace);
    return dtype == CFK_BF16 ? ln_bwd_impl<__nv_bfloat16>(st, d, x, gamma, mean, rstd, dy, dx,
                                                          dgamma, dbeta, partial, M, C, eps)
                             : ln_bwd_impl<__half>(st, d, x, gamma, mean, rstd, dy, dx, dgamma,
                                                   dbeta, partial, M, C, eps);
}

// ------------------------------------------------------------------------------------------
// LayerNorm backward without caller-provided scratch.
//
// Some callers cannot hand the library device memory: an XLA FFI handler receives only the
// buffers its binding declares and must not allocate, so a LayerNorm-backward handler with the
// reference's buffer list (no workspace result) has nowhere to put the per-CTA dgamma/dbeta
// partials; hosts that pre-plan every device allocation are in the same position.  For them
// this variant keeps the partials in a fixed device array that belongs to the library.
// ------------------------------------------------------------------------------------------
namespace cfk {
namespace {

constexpr int kNoAllocMaxC = 1024;    // widest row the static scratch serves
constexpr int kNoAllocMaxParts = 320; // CTAs (partials) of one launch
constexpr size_t kNoAllocFloats = static_cast<size_t>(kNoAllocMaxParts) * 2 * kNoAllocMaxC;

// 2.5 MiB per device that loads the library, held until the process exits.  Shared by every
// call: each launch overwrites the partials it reads, so nothing needs clearing between calls,
// but two calls that overlap on the GPU (different streams, same device) race on it.
static __device__ __align__(256) float g_ln_noalloc_scratch[kNoAllocFloats];

constexpr int kMaxDev = 64;
std::atomic<float*> g_noalloc_ptr[kMaxDev];
std::mutex g_noalloc_mu;

// Device address of the scratch on the current device.  The array's name is only a host-side
// stand-in, so the address comes from cudaGetSymbolAddress, with that device current.  Only a
// successful lookup is kept: a lookup that failed (for example a first call made while a
// stream capture was open) is retried by the next call.
int noalloc_scratch(int dev, float** out) {
    if (dev < 0 || dev >= kMaxDev) {
        return fail(CFK_ERR_INVALID_ARGUMENT,
                    "cfk_ln_bwd_noalloc: device ordinal %d outside the %d devices it serves", dev,
                    kMaxDev);
    }
    float* p = g_noalloc_ptr[dev].load(std::memory_order_acquire);
    if (!p) {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        p = g_noalloc_ptr[dev].load(std::memory_order_relaxed);
        if (!p) {
            void* addr = nullptr;
            const cudaError_t err = cudaGetSymbolAddress(&addr, g_ln_noalloc_scratch);
            if (err != cudaSuccess || !addr) {
                return fail(CFK_ERR_LAUNCH, "cfk_ln_bwd_noalloc: cudaGetSymbolAddress failed: %s",
                            cudaGetErrorString(err));
            }
            p = static_cast<float*>(addr);
            g_noalloc_ptr[dev].store(p, std::memory_order_release);
        }
    }
    *out = p;
    return CFK_OK;
}

template <typename T>
int ln_bwd_noalloc_impl(cudaStream_t st, const DeviceInfo& d, const void* x, const float* gamma,
                        const float* mean, const float* rstd, const void* dy, void* dx,
                        float* dgamma, float* dbeta, float* partial, int64_t M, int64_t C,
                        float eps) {
    VecShape s;
    const T* xp = static_cast<const T*>(x);
    const T* dyp = static_cast<const T*>(dy);
    T* dxp = static_cast<T*>(dx);
    int grid = 0;
    bool launched = false;
    if (vec_shape(C, &s) && aligned16(x) && aligned16(dy) && aligned16(dx)) {
        const int64_t rps = static_cast<int64_t>(32 / s.lpr) * kU;
        grid = std::min(grid_for((M + rps - 1) / rps, d), kNoAllocMaxParts);
#define CFK_LN_BWD_NA(LPR, NV)                                                                     \
    if (!launched && s.lpr == LPR && s.nv == NV) {                                                 \
        ln_bwd_vec_kernel<T, LPR, NV, kU>                                                          \
            <<<grid, kThreads, 0, st>>>(xp, gamma, mean, rstd, dyp, dxp, partial, M, eps);         \
        launched = true;                                                                           \
    }
        CFK_LN_BWD_NA(8, 1)
        CFK_LN_BWD_NA(16, 1)
        CFK_LN_BWD_NA(32, 1)
        CFK_LN_BWD_NA(16, 3)
        CFK_LN_BWD_NA(32, 2)
        CFK_LN_BWD_NA(32, 3)
        CFK_LN_BWD_NA(32, 4)
#undef CFK_LN_BWD_NA
    }
    if (!launched) {
        grid = std::min(grid_for(M, d), kNoAllocMaxParts);
        const int smem = kWarps * 2 * static_cast<int>(C) * static_cast<int>(sizeof(float));
        if (smem > 48 * 1024) {
            CFK_TRY(ensure_smem_attr(reinterpret_cast<const void*>(&ln_bwd_generic_kernel<T>),
                                     d.device, smem, "ln_bwd_noalloc"));
        }
        ln_bwd_generic_kernel<T><<<grid, kThreads, smem, st>>>(xp, gamma, mean, rstd, dyp, dxp,
                                                               partial, M, static_cast<int>(C), eps);
    }
    CFK_TRY(check_launch("ln_bwd_noalloc"));
    const int blocks = static_cast<int>((2 * C + 31) / 32);
    ln_bwd_reduce_kernel<<<blocks, kReduceWarps * 32, 0, st>>>(partial, grid, static_cast<int>(C),
                                                               dgamma, dbeta);
    return check_launch("ln_bwd_noalloc_reduce");
}

} // namespace
} // namespace cfk

extern "C" int cfk_ln_bwd_noalloc(cfk_stream_t stream, cfk_dtype dtype, const void* x,
                                  const float* gamma, const float* mean, const float* rstd,
                                  const void* dy, void* dx, float* dgamma, float* dbeta,
                                  int64_t M, int64_t C, float eps) {
    clear_error();
    CFK_TRY(check_ln_args("cfk_ln_bwd_noalloc", dtype, M, C, eps));
    if (C > kNoAllocMaxC) {
        return fail(CFK_ERR_INVALID_ARGUMENT,
                    "cfk_ln_bwd_noalloc: C=%lld exceeds the %d columns its static scratch serves; "
                    "use cfk_ln_bwd with a workspace",
                    static_cast<long long>(C), kNoAllocMaxC);
    }
    if (!gamma || !dgamma || !dbeta) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_ln_bwd_noalloc: null buffer");
    }
    if ((mean == nullptr) != (rstd == nullptr)) {
        return fail(CFK_ERR_INVALID_ARGUMENT,
                    "cfk_ln_bwd_noalloc: give both mean and rstd, or neither to recompute them");
    }
    DeviceInfo d;
    CFK_TRY(current_device(&d));
    float* partial = nullptr;
    CFK_TRY(noalloc_scratch(d.device, &partial));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (M == 0) {
        cudaError_t e1 = cudaMemsetAsync(dgamma, 0, C * sizeof(float), st);
        cudaError_t e2 = cudaMemsetAsync(dbeta, 0, C * sizeof(float), st);
        if (e1 != cudaSuccess || e2 != cudaSuccess) {
            return fail(CFK_ERR_LAUNCH, "cfk_ln_bwd_noalloc: memset failed");
        }
        return CFK_OK;
    }
    if (!x || !dy || !dx) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "cfk_ln_bwd_noalloc: null buffer");
    }
    return dtype == CFK_BF16
               ? ln_bwd_noalloc_impl<__nv_bfloat16>(st, d, x, gamma, mean, rstd, dy, dx, dgamma,
                                                    dbeta, partial, M, C, eps)
               : ln_bwd_noalloc_impl<__half>(st, d, x, gamma, mean, rstd, dy, dx, dgamma, dbeta,
                                             partial, M, C, eps);
}
