// ffi_handlers.cc -- XLA FFI handlers of the sm_100a kernels (libcfk_xla_sm100.so).
//
// The drop-in surface of the reference's handlers (same symbol names, argument order, ranks,
// attributes and traits), re-bound to accept F16 or BF16 where the reference takes F16:
//
//   VoltaMma        cuda/volta_mma_attn.cu:304-351    q, k, v, bias, kmask -> out
//                                                     attrs scale, block_q, block_k
//   VoltaWmma       cuda/volta_wmma_attn.cu:264-311   (same; the sm_70 twin's name)
//   VoltaLayerNorm  cuda/volta_ops.cu:62-95           x, scale f32, offset f32 -> out; eps
//   VoltaGdp        cuda/volta_ops.cu:210-265         x, wp, bp, wg, bg, mask -> out
//   VoltaGdpWmma    cuda/volta_gdp_wmma.cu:99-140     (same, stream context only)
//
// and new targets with no reference counterpart:
//
//   CfkAttentionFwdRes  as VoltaMma, plus lse f32 [N,H,Sq] as a second result
//   CfkAttentionBwd     q, k, v, bias, kmask, out, lse, dout -> dq, dk, dv, dbias f32 [H,Sq,Sk],
//                       workspace u8 [>= cfk_attn_bwd_workspace_size]; attr scale
//   CfkLayerNormBwd     x, scale f32, dy -> dx, dscale f32, doffset f32, workspace u8; attr eps
//   CfkGdpBwd           x, wp, bp, wg, bg, mask, dout -> dx, dwp, dbp, dwg, dbg (f32),
//                       workspace u8
//
// Every handler validates ranks, shapes and dtypes (mixed F16/BF16 -> InvalidArgument), then
// enqueues on the XLA stream through the C ABI of include/cfk.h: no allocation (scratch comes in
// as a result buffer), no synchronisation, no host work beyond per-device attribute caches, so
// the handlers keep the reference's kCmdBufferCompatible trait.  C-ABI argument errors map to
// InvalidArgument and launch failures to Internal, as in the reference (:297-300, :310-333).
//
// Built only when the XLA FFI headers (jax >= 0.6.2) are available: see build.py.
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "cfk.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace cfk_ffi {

inline ffi::Error from_status(int rc, const char* what) {
    if (rc == CFK_OK) {
        return ffi::Error::Success();
    }
    std::string msg = std::string(what) + ": " + cfk_last_error();
    return rc == CFK_ERR_INVALID_ARGUMENT ? ffi::Error::InvalidArgument(msg)
                                          : ffi::Error::Internal(msg);
}

// F16 or BF16 -> the C ABI dtype code; anything else -> -1.
inline int half_code(ffi::DataType t) {
    if (t == ffi::DataType::F16) {
        return CFK_F16;
    }
    if (t == ffi::DataType::BF16) {
        return CFK_BF16;
    }
    return -1;
}

template <typename B>
bool has_dims(const B& b, std::initializer_list<int64_t> want) {
    auto d = b.dimensions();
    if (d.size() != want.size()) {
        return false;
    }
    size_t i = 0;
    for (int64_t w : want) {
        if (d[i++] != w) {
            return false;
        }
    }
    return true;
}

// The common dtype of 16-bit buffers, or -1 when one is not F16/BF16 or they differ.
inline int common_half_code(std::initializer_list<const ffi::AnyBuffer*> bufs) {
    int code = -2;
    for (const ffi::AnyBuffer* b : bufs) {
        const int c = half_code(b->element_type());
        if (c < 0 || (code != -2 && c != code)) {
            return -1;
        }
        code = c;
    }
    return code;
}

// (D, block_q, block_k) tuples the reference's dispatch tables accept
// (cuda/volta_mma_attn.cu:322-333, cuda/volta_wmma_attn.cu:281-295).  The B200 kernels use
// their own 128 x 128 tiles; the tuple is checked only to keep the reference's error behaviour.
inline bool mma_tuple_ok(int64_t d, int64_t bq, int64_t bk) {
    static const int64_t t[][3] = {{8, 64, 64},  {8, 64, 32},  {8, 32, 32},  {8, 128, 64},
                                   {8, 32, 64},  {32, 64, 64}, {32, 64, 32}, {32, 32, 64},
                                   {32, 32, 32}, {32, 128, 64}, {32, 16, 64}, {16, 64, 64},
                                   {16, 32, 32}, {16, 64, 32}, {64, 64, 64}, {64, 32, 32}};
    for (const auto& e : t) {
        if (e[0] == d && e[1] == bq && e[2] == bk) {
            return true;
        }
    }
    return false;
}

inline bool wmma_tuple_ok(int64_t d, int64_t bq, int64_t bk) {
    static const int64_t t[][3] = {{32, 64, 64}, {32, 64, 32}, {32, 32, 64}, {32, 32, 32},
                                   {32, 128, 64}, {32, 128, 32}, {16, 64, 64}, {16, 32, 32},
                                   {16, 64, 32}, {64, 64, 64}, {64, 32, 32}, {64, 64, 32},
                                   {8, 64, 64},  {8, 64, 32},  {8, 32, 32}};
    for (const auto& e : t) {
        if (e[0] == d && e[1] == bq && e[2] == bk) {
            return true;
        }
    }
    return false;
}

struct AttnDims {
    int64_t N, H, Sq, Sk, D;
    int code;
};

// Validates q, k, v, bias, kmask (and out) and returns the sizes; `err` set on failure.
inline AttnDims attn_dims(const char* fn, const ffi::AnyBuffer& q, const ffi::AnyBuffer& k,
                          const ffi::AnyBuffer& v, const ffi::AnyBuffer& bias,
                          const ffi::Buffer<ffi::DataType::U8>& kmask, const ffi::AnyBuffer& out,
                          ffi::Error* err) {
    AttnDims a{0, 0, 0, 0, 0, -1};
    auto qd = q.dimensions();
    if (qd.size() != 4) {
        *err = ffi::Error::InvalidArgument(std::string(fn) + ": q must be [N,H,S,D]");
        return a;
    }
    a.N = qd[0];
    a.H = qd[1];
    a.Sq = qd[2];
    a.D = qd[3];
    auto kd = k.dimensions();
    a.Sk = kd.size() == 4 ? kd[2] : -1;
    if (!has_dims(k, {a.N, a.H, a.Sk, a.D}) || !has_dims(v, {a.N, a.H, a.Sk, a.D}) ||
        !has_dims(bias, {a.H, a.Sq, a.Sk}) || !has_dims(kmask, {a.N, a.Sk}) ||
        !has_dims(out, {a.N, a.H, a.Sq, a.D})) {
        *err = ffi::Error::InvalidArgument(
            std::string(fn) + ": expected k, v [N,H,Sk,D], bias [H,Sq,Sk], kmask [N,Sk] and "
                              "out [N,H,Sq,D] for q [N,H,Sq,D]");
        return a;
    }
    a.code = common_half_code({&q, &k, &v, &bias, &out});
    if (a.code < 0) {
        *err = ffi::Error::InvalidArgument(
            std::string(fn) + ": q, k, v, bias and out must all be F16 or all BF16");
    }
    return a;
}

ffi::Error AttentionImpl(const char* fn, bool wmma_table, bool check_tuple, cudaStream_t stream,
                         ffi::AnyBuffer q, ffi::AnyBuffer k, ffi::AnyBuffer v, ffi::AnyBuffer bias,
                         ffi::Buffer<ffi::DataType::U8> kmask, ffi::AnyBuffer* out, float* lse,
                         float scale, int64_t block_q, int64_t block_k) {
    ffi::Error err = ffi::Error::Success();
    const AttnDims a = attn_dims(fn, q, k, v, bias, kmask, *out, &err);
    if (a.code < 0) {
        return err;
    }
    if (check_tuple && !(wmma_table ? wmma_tuple_ok(a.D, block_q, block_k)
                                    : mma_tuple_ok(a.D, block_q, block_k))) {
        return ffi::Error::InvalidArgument(std::string(fn) + ": unsupported (D, bq, bk)");
    }
    return from_status(cfk_attn_fwd(stream, static_cast<cfk_dtype>(a.code), q.untyped_data(),
                                    k.untyped_data(), v.untyped_data(), bias.untyped_data(),
                                    kmask.typed_data(), out->untyped_data(), lse, a.N, a.H, a.Sq,
                                    a.Sk, a.D, scale),
                       fn);
}

ffi::Error VoltaMmaImpl(cudaStream_t stream, int32_t device, ffi::AnyBuffer q, ffi::AnyBuffer k,
                        ffi::AnyBuffer v, ffi::AnyBuffer bias,
                        ffi::Buffer<ffi::DataType::U8> kmask, ffi::Result<ffi::AnyBuffer> out,
                        float scale, int64_t block_q, int64_t block_k) {
    (void)device;
    return AttentionImpl("VoltaMma", false, true, stream, q, k, v, bias, kmask, &*out, nullptr,
                         scale, block_q, block_k);
}

ffi::Error VoltaWmmaImpl(cudaStream_t stream, int32_t device, ffi::AnyBuffer q, ffi::AnyBuffer k,
                         ffi::AnyBuffer v, ffi::AnyBuffer bias,
                         ffi::Buffer<ffi::DataType::U8> kmask, ffi::Result<ffi::AnyBuffer> out,
                         float scale, int64_t block_q, int64_t block_k) {
    (void)device;
    return AttentionImpl("VoltaWmma", true, true, stream, q, k, v, bias, kmask, &*out, nullptr,
                         scale, block_q, block_k);
}

ffi::Error AttentionFwdResImpl(cudaStream_t stream, int32_t device, ffi::AnyBuffer q,
                               ffi::AnyBuffer k, ffi::AnyBuffer v, ffi::AnyBuffer bias,
                               ffi::Buffer<ffi::DataType::U8> kmask,
                               ffi::Result<ffi::AnyBuffer> out,
                               ffi::Result<ffi::Buffer<ffi::DataType::F32>> lse, float scale,
                               int64_t block_q, int64_t block_k) {
    (void)device;
    auto qd = q.dimensions();
    if (qd.size() != 4 || !has_dims(*lse, {qd[0], qd[1], qd[2]})) {
        return ffi::Error::InvalidArgument("CfkAttentionFwdRes: lse must be f32 [N,H,Sq]");
    }
    // block_q / block_k are hints only for this target
    return AttentionImpl("CfkAttentionFwdRes", false, false, stream, q, k, v, bias, kmask, &*out,
                         lse->typed_data(), scale, block_q, block_k);
}

ffi::Error AttentionBwdImpl(cudaStream_t stream, ffi::AnyBuffer q, ffi::AnyBuffer k,
                            ffi::AnyBuffer v, ffi::AnyBuffer bias,
                            ffi::Buffer<ffi::DataType::U8> kmask, ffi::AnyBuffer out,
                            ffi::Buffer<ffi::DataType::F32> lse, ffi::AnyBuffer dout,
                            ffi::Result<ffi::AnyBuffer> dq, ffi::Result<ffi::AnyBuffer> dk,
                            ffi::Result<ffi::AnyBuffer> dv,
                            ffi::Result<ffi::Buffer<ffi::DataType::F32>> dbias,
                            ffi::Result<ffi::Buffer<ffi::DataType::U8>> workspace, float scale) {
    const char* fn = "CfkAttentionBwd";
    ffi::Error err = ffi::Error::Success();
    const AttnDims a = attn_dims(fn, q, k, v, bias, kmask, out, &err);
    if (a.code < 0) {
        return err;
    }
    if (!has_dims(lse, {a.N, a.H, a.Sq}) || !has_dims(dout, {a.N, a.H, a.Sq, a.D}) ||
        !has_dims(*dq, {a.N, a.H, a.Sq, a.D}) || !has_dims(*dk, {a.N, a.H, a.Sk, a.D}) ||
        !has_dims(*dv, {a.N, a.H, a.Sk, a.D}) || !has_dims(*dbias, {a.H, a.Sq, a.Sk}) ||
        workspace->dimensions().size() != 1) {
        return ffi::Error::InvalidArgument(
            "CfkAttentionBwd: expected lse [N,H,Sq], dout and dq [N,H,Sq,D], dk and dv "
            "[N,H,Sk,D], dbias [H,Sq,Sk] and a rank-1 workspace");
    }
    if (common_half_code({&q, &dout, &*dq, &*dk, &*dv}) != a.code) {
        return ffi::Error::InvalidArgument(
            "CfkAttentionBwd: dout, dq, dk and dv must have the dtype of q");
    }
    return from_status(
        cfk_attn_bwd(stream, static_cast<cfk_dtype>(a.code), q.untyped_data(), k.untyped_data(),
                     v.untyped_data(), bias.untyped_data(), kmask.typed_data(),
                     out.untyped_data(), lse.typed_data(), dout.untyped_data(),
                     dq->untyped_data(), dk->untyped_data(), dv->untyped_data(),
                     dbias->typed_data(), workspace->typed_data(),
                     static_cast<size_t>(workspace->dimensions()[0]), a.N, a.H, a.Sq, a.Sk, a.D,
                     scale),
        fn);
}

ffi::Error LayerNormImpl(cudaStream_t stream, ffi::AnyBuffer x,
                         ffi::Buffer<ffi::DataType::F32> scale,
                         ffi::Buffer<ffi::DataType::F32> offset, ffi::Result<ffi::AnyBuffer> out,
                         float eps) {
    auto d = x.dimensions();
    if (d.size() != 2) {
        return ffi::Error::InvalidArgument("x must be [M,C]");
    }
    const int64_t M = d[0], C = d[1];
    if (!has_dims(scale, {C}) || !has_dims(offset, {C}) || !has_dims(*out, {M, C})) {
        return ffi::Error::InvalidArgument(
            "VoltaLayerNorm: expected scale, offset [C] and out [M,C]");
    }
    const int code = common_half_code({&x, &*out});
    if (code < 0) {
        return ffi::Error::InvalidArgument("VoltaLayerNorm: x and out must both be F16 or BF16");
    }
    return from_status(cfk_ln_fwd(stream, static_cast<cfk_dtype>(code), x.untyped_data(),
                                  scale.typed_data(), offset.typed_data(), out->untyped_data(),
                                  nullptr, nullptr, M, C, eps),
                       "VoltaLayerNorm");
}

ffi::Error LayerNormBwdImpl(cudaStream_t stream, ffi::AnyBuffer x,
                            ffi::Buffer<ffi::DataType::F32> scale, ffi::AnyBuffer dy,
                            ffi::Result<ffi::AnyBuffer> dx,
                            ffi::Result<ffi::Buffer<ffi::DataType::F32>> dscale,
                            ffi::Result<ffi::Buffer<ffi::DataType::F32>> doffset,
                            ffi::Result<ffi::Buffer<ffi::DataType::U8>> workspace, float eps) {
    auto d = x.dimensions();
    if (d.size() != 2) {
        return ffi::Error::InvalidArgument("CfkLayerNormBwd: x must be [M,C]");
    }
    const int64_t M = d[0], C = d[1];
    if (!has_dims(scale, {C}) || !has_dims(dy, {M, C}) || !has_dims(*dx, {M, C}) ||
        !has_dims(*dscale, {C}) || !has_dims(*doffset, {C}) ||
        workspace->dimensions().size() != 1) {
        return ffi::Error::InvalidArgument(
            "CfkLayerNormBwd: expected scale [C], dy and dx [M,C], dscale and doffset [C] and "
            "a rank-1 workspace");
    }
    const int code = common_half_code({&x, &dy, &*dx});
    if (code < 0) {
        return ffi::Error::InvalidArgument(
            "CfkLayerNormBwd: x, dy and dx must all be F16 or all BF16");
    }
    // mean and rstd are recomputed from x (the forward handler does not return them)
    return from_status(cfk_ln_bwd(stream, static_cast<cfk_dtype>(code), x.untyped_data(),
                                  scale.typed_data(), nullptr, nullptr, dy.untyped_data(),
                                  dx->untyped_data(), dscale->typed_data(), doffset->typed_data(),
                                  workspace->typed_data(),
                                  static_cast<size_t>(workspace->dimensions()[0]), M, C, eps),
                       "CfkLayerNormBwd");
}

struct GdpDims {
    int64_t M, K, N;
    int code;
};

inline GdpDims gdp_dims(const char* fn, const ffi::AnyBuffer& x, const ffi::AnyBuffer& wp,
                        const ffi::AnyBuffer& bp, const ffi::AnyBuffer& wg,
                        const ffi::AnyBuffer& bg, const ffi::AnyBuffer& mask, ffi::Error* err) {
    GdpDims g{0, 0, 0, -1};
    auto xd = x.dimensions();
    if (xd.size() != 2) {
        *err = ffi::Error::InvalidArgument("x must be [M,K]");
        return g;
    }
    g.M = xd[0];
    g.K = xd[1];
    auto wd = wp.dimensions();
    g.N = wd.size() == 2 ? wd[1] : -1;
    if (!has_dims(wp, {g.K, g.N}) || !has_dims(wg, {g.K, g.N}) || !has_dims(bp, {g.N}) ||
        !has_dims(bg, {g.N}) || !has_dims(mask, {g.M})) {
        *err = ffi::Error::InvalidArgument(
            std::string(fn) + ": expected wp, wg [K,N], bp, bg [N] and mask [M] for x [M,K]");
        return g;
    }
    if (g.N % 8) {
        *err = ffi::Error::InvalidArgument("gdp: N must be a multiple of 8");
        return g;
    }
    g.code = common_half_code({&x, &wp, &bp, &wg, &bg, &mask});
    if (g.code < 0) {
        *err = ffi::Error::InvalidArgument(
            std::string(fn) + ": x, wp, bp, wg, bg and mask must all be F16 or all BF16");
    }
    return g;
}

ffi::Error GdpFwd(const char* fn, cudaStream_t stream, ffi::AnyBuffer x, ffi::AnyBuffer wp,
                  ffi::AnyBuffer bp, ffi::AnyBuffer wg, ffi::AnyBuffer bg, ffi::AnyBuffer mask,
                  ffi::AnyBuffer* out) {
    ffi::Error err = ffi::Error::Success();
    const GdpDims g = gdp_dims(fn, x, wp, bp, wg, bg, mask, &err);
    if (g.code < 0) {
        return err;
    }
    if (!has_dims(*out, {g.M, g.N}) || half_code(out->element_type()) != g.code) {
        return ffi::Error::InvalidArgument(std::string(fn) + ": out must be [M,N] of x's dtype");
    }
    return from_status(cfk_gdp_fwd(stream, static_cast<cfk_dtype>(g.code), x.untyped_data(),
                                   wp.untyped_data(), bp.untyped_data(), wg.untyped_data(),
                                   bg.untyped_data(), mask.untyped_data(), out->untyped_data(),
                                   g.M, g.K, g.N),
                       fn);
}

ffi::Error GdpImpl(cudaStream_t stream, int32_t device, ffi::AnyBuffer x, ffi::AnyBuffer wp,
                   ffi::AnyBuffer bp, ffi::AnyBuffer wg, ffi::AnyBuffer bg, ffi::AnyBuffer mask,
                   ffi::Result<ffi::AnyBuffer> out) {
    (void)device;
    return GdpFwd("VoltaGdp", stream, x, wp, bp, wg, bg, mask, &*out);
}

ffi::Error GdpWmmaImpl(cudaStream_t stream, ffi::AnyBuffer x, ffi::AnyBuffer wp,
                       ffi::AnyBuffer bp, ffi::AnyBuffer wg, ffi::AnyBuffer bg,
                       ffi::AnyBuffer mask, ffi::Result<ffi::AnyBuffer> out) {
    return GdpFwd("VoltaGdpWmma", stream, x, wp, bp, wg, bg, mask, &*out);
}

ffi::Error GdpBwdImpl(cudaStream_t stream, ffi::AnyBuffer x, ffi::AnyBuffer wp,
                      ffi::AnyBuffer bp, ffi::AnyBuffer wg, ffi::AnyBuffer bg,
                      ffi::AnyBuffer mask, ffi::AnyBuffer dout, ffi::Result<ffi::AnyBuffer> dx,
                      ffi::Result<ffi::Buffer<ffi::DataType::F32>> dwp,
                      ffi::Result<ffi::Buffer<ffi::DataType::F32>> dbp,
                      ffi::Result<ffi::Buffer<ffi::DataType::F32>> dwg,
                      ffi::Result<ffi::Buffer<ffi::DataType::F32>> dbg,
                      ffi::Result<ffi::Buffer<ffi::DataType::U8>> workspace) {
    const char* fn = "CfkGdpBwd";
    ffi::Error err = ffi::Error::Success();
    const GdpDims g = gdp_dims(fn, x, wp, bp, wg, bg, mask, &err);
    if (g.code < 0) {
        return err;
    }
    if (!has_dims(dout, {g.M, g.N}) || !has_dims(*dx, {g.M, g.K}) ||
        !has_dims(*dwp, {g.K, g.N}) || !has_dims(*dwg, {g.K, g.N}) || !has_dims(*dbp, {g.N}) ||
        !has_dims(*dbg, {g.N}) || workspace->dimensions().size() != 1) {
        return ffi::Error::InvalidArgument(
            "CfkGdpBwd: expected dout [M,N], dx [M,K], dwp and dwg [K,N], dbp and dbg [N] and a "
            "rank-1 workspace");
    }
    if (common_half_code({&x, &dout, &*dx}) != g.code) {
        return ffi::Error::InvalidArgument("CfkGdpBwd: dout and dx must have the dtype of x");
    }
    return from_status(
        cfk_gdp_bwd(stream, static_cast<cfk_dtype>(g.code), x.untyped_data(), wp.untyped_data(),
                    bp.untyped_data(), wg.untyped_data(), bg.untyped_data(), mask.untyped_data(),
                    dout.untyped_data(), dx->untyped_data(), dwp->typed_data(),
                    dbp->typed_data(), dwg->typed_data(), dbg->typed_data(),
                    workspace->typed_data(), static_cast<size_t>(workspace->dimensions()[0]),
                    g.M, g.K, g.N),
        fn);
}

} // namespace cfk_ffi

// ---------------------------------------------------------------------------------------------
// Symbols.  kCmdBufferCompatible: each handler only enqueues kernels (and, for the backward
// handlers, cudaMemsetAsync) on the XLA stream.
// ---------------------------------------------------------------------------------------------
#define CFK_ATTN_FWD_BINDING                                                                       \
    ffi::Ffi::Bind()                                                                               \
        .Ctx<ffi::PlatformStream<cudaStream_t>>()                                                  \
        .Ctx<ffi::DeviceOrdinal>()                                                                 \
        .Arg<ffi::AnyBuffer>()                                                                     \
        .Arg<ffi::AnyBuffer>()                                                                     \
        .Arg<ffi::AnyBuffer>()                                                                     \
        .Arg<ffi::AnyBuffer>()                                                                     \
        .Arg<ffi::Buffer<ffi::DataType::U8>>()                                                     \
        .Ret<ffi::AnyBuffer>()

XLA_FFI_DEFINE_HANDLER_SYMBOL(VoltaMma, cfk_ffi::VoltaMmaImpl,
                              CFK_ATTN_FWD_BINDING.Attr<float>("scale")
                                  .Attr<int64_t>("block_q")
                                  .Attr<int64_t>("block_k"),
                              {ffi::Traits::kCmdBufferCompatible});

XLA_FFI_DEFINE_HANDLER_SYMBOL(VoltaWmma, cfk_ffi::VoltaWmmaImpl,
                              CFK_ATTN_FWD_BINDING.Attr<float>("scale")
                                  .Attr<int64_t>("block_q")
                                  .Attr<int64_t>("block_k"),
                              {ffi::Traits::kCmdBufferCompatible});

XLA_FFI_DEFINE_HANDLER_SYMBOL(CfkAttentionFwdRes, cfk_ffi::AttentionFwdResImpl,
                              CFK_ATTN_FWD_BINDING.Ret<ffi::Buffer<ffi::DataType::F32>>()
                                  .Attr<float>("scale")
                                  .Attr<int64_t>("block_q")
                                  .Attr<int64_t>("block_k"),
                              {ffi::Traits::kCmdBufferCompatible});

XLA_FFI_DEFINE_HANDLER_SYMBOL(CfkAttentionBwd, cfk_ffi::AttentionBwdImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()                      // q
                                  .Arg<ffi::AnyBuffer>()                      // k
                                  .Arg<ffi::AnyBuffer>()                      // v
                                  .Arg<ffi::AnyBuffer>()                      // bias
                                  .Arg<ffi::Buffer<ffi::DataType::U8>>()      // kmask
                                  .Arg<ffi::AnyBuffer>()                      // out
                                  .Arg<ffi::Buffer<ffi::DataType::F32>>()     // lse
                                  .Arg<ffi::AnyBuffer>()                      // dout
                                  .Ret<ffi::AnyBuffer>()                      // dq
                                  .Ret<ffi::AnyBuffer>()                      // dk
                                  .Ret<ffi::AnyBuffer>()                      // dv
                                  .Ret<ffi::Buffer<ffi::DataType::F32>>()     // dbias
                                  .Ret<ffi::Buffer<ffi::DataType::U8>>()      // workspace
                                  .Attr<float>("scale"),
                              {ffi::Traits::kCmdBufferCompatible});

XLA_FFI_DEFINE_HANDLER_SYMBOL(VoltaLayerNorm, cfk_ffi::LayerNormImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::DataType::F32>>()
                                  .Arg<ffi::Buffer<ffi::DataType::F32>>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Attr<float>("eps"),
                              {ffi::Traits::kCmdBufferCompatible});

XLA_FFI_DEFINE_HANDLER_SYMBOL(CfkLayerNormBwd, cfk_ffi::LayerNormBwdImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()                      // x
                                  .Arg<ffi::Buffer<ffi::DataType::F32>>()     // scale
                                  .Arg<ffi::AnyBuffer>()                      // dy
                                  .Ret<ffi::AnyBuffer>()                      // dx
                                  .Ret<ffi::Buffer<ffi::DataType::F32>>()     // dscale
                                  .Ret<ffi::Buffer<ffi::DataType::F32>>()     // doffset
                                  .Ret<ffi::Buffer<ffi::DataType::U8>>()      // workspace
                                  .Attr<float>("eps"),
                              {ffi::Traits::kCmdBufferCompatible});

#define CFK_GDP_ARGS                                                                               \
    .Arg<ffi::AnyBuffer>()       /* x */                                                           \
        .Arg<ffi::AnyBuffer>()   /* wp */                                                          \
        .Arg<ffi::AnyBuffer>()   /* bp */                                                          \
        .Arg<ffi::AnyBuffer>()   /* wg */                                                          \
        .Arg<ffi::AnyBuffer>()   /* bg */                                                          \
        .Arg<ffi::AnyBuffer>()   /* mask */

XLA_FFI_DEFINE_HANDLER_SYMBOL(VoltaGdp, cfk_ffi::GdpImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Ctx<ffi::DeviceOrdinal>() CFK_GDP_ARGS
                                  .Ret<ffi::AnyBuffer>(),
                              {ffi::Traits::kCmdBufferCompatible});

XLA_FFI_DEFINE_HANDLER_SYMBOL(VoltaGdpWmma, cfk_ffi::GdpWmmaImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>() CFK_GDP_ARGS
                                  .Ret<ffi::AnyBuffer>(),
                              {ffi::Traits::kCmdBufferCompatible});

XLA_FFI_DEFINE_HANDLER_SYMBOL(CfkGdpBwd, cfk_ffi::GdpBwdImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>() CFK_GDP_ARGS
                                  .Arg<ffi::AnyBuffer>()                      // dout
                                  .Ret<ffi::AnyBuffer>()                      // dx
                                  .Ret<ffi::Buffer<ffi::DataType::F32>>()     // dwp
                                  .Ret<ffi::Buffer<ffi::DataType::F32>>()     // dbp
                                  .Ret<ffi::Buffer<ffi::DataType::F32>>()     // dwg
                                  .Ret<ffi::Buffer<ffi::DataType::F32>>()     // dbg
                                  .Ret<ffi::Buffer<ffi::DataType::U8>>(),     // workspace
                              {ffi::Traits::kCmdBufferCompatible});
