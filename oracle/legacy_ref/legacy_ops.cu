// Legacy comparator: the reference's LayerNorm (cuda/volta_ops.cu, LayerNormImpl at :62-85)
// and gated dual projection (GdpImpl at :210-252), compiled from the reference source as it
// lies and called through its own handler bodies -- TEST INFRASTRUCTURE (see build.py).
#include "legacy_common.h"

#include "volta_ops.cu"

LEGACY_API int legacy_layer_norm(void* stream, const void* x, const float* gamma,
                                 const float* beta, void* out, int64_t M, int64_t C, float eps,
                                 char* msg, int msg_len) {
    using namespace xla::ffi;
    Buffer<DataType::F16> xb(x, {M, C}), ob(out, {M, C});
    Buffer<DataType::F32> gb(gamma, {C}), bb(beta, {C});
    return legacy_result(LayerNormImpl(static_cast<cudaStream_t>(stream), xb, gb, bb,
                                       Result<Buffer<DataType::F16>>(&ob), eps),
                         msg, msg_len);
}

LEGACY_API int legacy_gdp(void* stream, const void* x, const void* wp, const void* bp,
                          const void* wg, const void* bg, const void* mask, void* out, int64_t M,
                          int64_t K, int64_t N, char* msg, int msg_len) {
    using namespace xla::ffi;
    Buffer<DataType::F16> xb(x, {M, K}), wpb(wp, {K, N}), bpb(bp, {N}), wgb(wg, {K, N}),
        bgb(bg, {N}), mb(mask, {M}), ob(out, {M, N});
    return legacy_result(GdpImpl(static_cast<cudaStream_t>(stream), legacy_device(), xb, wpb, bpb,
                                 wgb, bgb, mb, Result<Buffer<DataType::F16>>(&ob)),
                         msg, msg_len);
}
