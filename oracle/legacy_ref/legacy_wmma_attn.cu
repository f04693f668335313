// Legacy comparator: the reference's sm_70 attention (cuda/volta_wmma_attn.cu, VoltaWmmaImpl
// at :264-296), compiled from the reference source as it lies and called through its own
// handler body -- TEST INFRASTRUCTURE (see build.py).  fp16 only, forward only.
#include "legacy_common.h"

#include "volta_wmma_attn.cu"

LEGACY_API int legacy_volta_wmma(void* stream, const void* q, const void* k, const void* v,
                                 const void* bias, const void* kmask, void* out, int64_t N,
                                 int64_t H, int64_t Sq, int64_t Sk, int64_t D, float scale,
                                 int64_t block_q, int64_t block_k, char* msg, int msg_len) {
    using namespace xla::ffi;
    Buffer<DataType::F16> qb(q, {N, H, Sq, D}), kb(k, {N, H, Sk, D}), vb(v, {N, H, Sk, D});
    Buffer<DataType::F16> bb(bias, {H, Sq, Sk});
    Buffer<DataType::U8> mb(kmask, {N, Sk});
    Buffer<DataType::F16> ob(out, {N, H, Sq, D});
    return legacy_result(VoltaWmmaImpl(static_cast<cudaStream_t>(stream), legacy_device(), qb,
                                       kb, vb, bb, mb, Result<Buffer<DataType::F16>>(&ob), scale,
                                       block_q, block_k),
                         msg, msg_len);
}
