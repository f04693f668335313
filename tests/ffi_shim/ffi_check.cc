// Test driver for the XLA FFI handlers (tests/test_ffi_handlers.py): compiles
// colabfold-legacy-kernels_b200/csrc/ffi_handlers.cc against the stand-in header next to this
// file and exposes one C entry point that runs a named scenario through a handler body.  The
// buffers carry null data pointers, so every scenario ends in the handler's own validation or
// in the C ABI's argument checks; none reaches a device.
#include "ffi_handlers.cc"

#include <cstring>

using namespace xla::ffi;

namespace {

AnyBuffer H(DataType t, std::initializer_list<int64_t> d) { return AnyBuffer(nullptr, t, d); }
template <DataType T>
Buffer<T> B(std::initializer_list<int64_t> d) {
    return Buffer<T>(nullptr, d);
}

Error attn(const char* what, DataType tq, DataType tk, int64_t bq, int64_t bk, bool bad_bias) {
    const int64_t N = 2, Hh = 4, S = 128, D = 32;
    auto q = H(tq, {N, Hh, S, D}), k = H(tk, {N, Hh, S, D}), v = H(tq, {N, Hh, S, D});
    auto bias = bad_bias ? H(tq, {Hh, S, S + 1}) : H(tq, {Hh, S, S});
    auto km = B<DataType::U8>({N, S});
    Result<AnyBuffer> out(H(tq, {N, Hh, S, D}));
    if (std::strcmp(what, "VoltaWmma") == 0) {
        return cfk_ffi::VoltaWmmaImpl(nullptr, 0, q, k, v, bias, km, out, 0.17f, bq, bk);
    }
    if (std::strcmp(what, "CfkAttentionFwdRes") == 0) {
        Result<Buffer<DataType::F32>> lse(B<DataType::F32>({N, Hh, S}));
        return cfk_ffi::AttentionFwdResImpl(nullptr, 0, q, k, v, bias, km, out, lse, 0.17f, bq,
                                            bk);
    }
    return cfk_ffi::VoltaMmaImpl(nullptr, 0, q, k, v, bias, km, out, 0.17f, bq, bk);
}

Error attn_bwd(bool bad_dbias) {
    const int64_t N = 2, Hh = 4, S = 128, D = 32;
    const DataType t = DataType::BF16;
    Result<AnyBuffer> dq(H(t, {N, Hh, S, D})), dk(H(t, {N, Hh, S, D})), dv(H(t, {N, Hh, S, D}));
    Result<Buffer<DataType::F32>> dbias(bad_dbias ? B<DataType::F32>({Hh, S})
                                                  : B<DataType::F32>({Hh, S, S}));
    Result<Buffer<DataType::U8>> ws(B<DataType::U8>({1 << 20}));
    return cfk_ffi::AttentionBwdImpl(nullptr, H(t, {N, Hh, S, D}), H(t, {N, Hh, S, D}),
                                     H(t, {N, Hh, S, D}), H(t, {Hh, S, S}),
                                     B<DataType::U8>({N, S}), H(t, {N, Hh, S, D}),
                                     B<DataType::F32>({N, Hh, S}), H(t, {N, Hh, S, D}), dq, dk,
                                     dv, dbias, ws, 0.17f);
}

Error ln(DataType tx, DataType tout, int64_t rank) {
    auto x = rank == 2 ? H(tx, {64, 128}) : H(tx, {64, 128, 1});
    Result<AnyBuffer> out(H(tout, {64, 128}));
    return cfk_ffi::LayerNormImpl(nullptr, x, B<DataType::F32>({128}), B<DataType::F32>({128}),
                                  out, 1e-5f);
}

Error ln_bwd() {
    const DataType t = DataType::F16;
    Result<AnyBuffer> dx(H(t, {64, 128}));
    Result<Buffer<DataType::F32>> ds(B<DataType::F32>({128})), dof(B<DataType::F32>({128}));
    Result<Buffer<DataType::U8>> ws(B<DataType::U8>({4096}));
    return cfk_ffi::LayerNormBwdImpl(nullptr, H(t, {64, 128}), B<DataType::F32>({128}),
                                     H(t, {64, 128}), dx, ds, dof, ws, 1e-5f);
}

Error gdp(const char* what, int64_t N, DataType tmask) {
    const DataType t = DataType::BF16;
    const int64_t M = 256, K = 128;
    Result<AnyBuffer> out(H(t, {M, N}));
    if (std::strcmp(what, "CfkGdpBwd") == 0) {
        Result<AnyBuffer> dx(H(t, {M, K}));
        Result<Buffer<DataType::F32>> dwp(B<DataType::F32>({K, N})), dbp(B<DataType::F32>({N})),
            dwg(B<DataType::F32>({K, N})), dbg(B<DataType::F32>({N}));
        Result<Buffer<DataType::U8>> ws(B<DataType::U8>({16}));
        return cfk_ffi::GdpBwdImpl(nullptr, H(t, {M, K}), H(t, {K, N}), H(t, {N}), H(t, {K, N}),
                                   H(t, {N}), H(tmask, {M}), H(t, {M, N}), dx, dwp, dbp, dwg, dbg,
                                   ws);
    }
    if (std::strcmp(what, "VoltaGdpWmma") == 0) {
        return cfk_ffi::GdpWmmaImpl(nullptr, H(t, {M, K}), H(t, {K, N}), H(t, {N}),
                                    H(t, {K, N}), H(t, {N}), H(tmask, {M}), out);
    }
    return cfk_ffi::GdpImpl(nullptr, 0, H(t, {M, K}), H(t, {K, N}), H(t, {N}), H(t, {K, N}),
                            H(t, {N}), H(tmask, {M}), out);
}

} // namespace

// Runs scenario `name`; returns the handler's error code (0 success, 1 InvalidArgument,
// 2 Internal) and copies its message.
extern "C" __attribute__((visibility("default"))) int ffi_check(const char* name, char* msg,
                                                                int len) {
    const DataType F16 = DataType::F16, BF16 = DataType::BF16, F32 = DataType::F32;
    Error e = Error::InvalidArgument("unknown scenario");
    const std::string s(name);
    if (s == "mma_ok") e = attn("VoltaMma", BF16, BF16, 64, 64, false);
    else if (s == "mma_f16_ok") e = attn("VoltaMma", F16, F16, 128, 64, false);
    else if (s == "mma_mixed") e = attn("VoltaMma", BF16, F16, 64, 64, false);
    else if (s == "mma_f32") e = attn("VoltaMma", F32, F32, 64, 64, false);
    else if (s == "mma_tuple") e = attn("VoltaMma", BF16, BF16, 64, 128, false);
    else if (s == "wmma_tuple_ok") e = attn("VoltaWmma", BF16, BF16, 128, 32, false);
    else if (s == "mma_tuple_wmma_only") e = attn("VoltaMma", BF16, BF16, 128, 32, false);
    else if (s == "mma_bias_shape") e = attn("VoltaMma", BF16, BF16, 64, 64, true);
    else if (s == "fwdres_any_tuple") e = attn("CfkAttentionFwdRes", BF16, BF16, 7, 9, false);
    else if (s == "attn_bwd_ok") e = attn_bwd(false);
    else if (s == "attn_bwd_dbias_shape") e = attn_bwd(true);
    else if (s == "ln_ok") e = ln(BF16, BF16, 2);
    else if (s == "ln_rank") e = ln(BF16, BF16, 3);
    else if (s == "ln_mixed") e = ln(F16, BF16, 2);
    else if (s == "ln_bwd_ok") e = ln_bwd();
    else if (s == "gdp_ok") e = gdp("VoltaGdp", 64, BF16);
    else if (s == "gdp_n8") e = gdp("VoltaGdp", 60, BF16);
    else if (s == "gdp_mixed") e = gdp("VoltaGdp", 64, F16);
    else if (s == "gdp_wmma_ok") e = gdp("VoltaGdpWmma", 64, BF16);
    else if (s == "gdp_bwd_ok") e = gdp("CfkGdpBwd", 64, BF16);
    std::strncpy(msg, e.message().c_str(), static_cast<size_t>(len - 1));
    msg[len - 1] = '\0';
    return e.code();
}
