// Legacy comparator: the reference's sm_70 gated dual projection (cuda/volta_gdp_wmma.cu,
// GdpWmmaImpl at :99-128), compiled from the reference source as it lies and called through
// its own handler body -- TEST INFRASTRUCTURE (see build.py).
#include "legacy_common.h"

#include "volta_gdp_wmma.cu"

LEGACY_API int legacy_gdp_wmma(void* stream, const void* x, const void* wp, const void* bp,
                               const void* wg, const void* bg, const void* mask, void* out,
                               int64_t M, int64_t K, int64_t N, char* msg, int msg_len) {
    using namespace xla::ffi;
    Buffer<DataType::F16> xb(x, {M, K}), wpb(wp, {K, N}), bpb(bp, {N}), wgb(wg, {K, N}),
        bgb(bg, {N}), mb(mask, {M}), ob(out, {M, N});
    return legacy_result(GdpWmmaImpl(static_cast<cudaStream_t>(stream), xb, wpb, bpb, wgb, bgb,
                                     mb, Result<Buffer<DataType::F16>>(&ob)),
                         msg, msg_len);
}
