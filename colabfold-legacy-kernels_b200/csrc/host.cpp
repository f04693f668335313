// host.cpp -- error reporting, device caches, kernel attributes and TMA descriptors.
//
// The reference caches the opt-in shared-memory limit and the attribute call in unguarded
// statics (cuda/volta_mma_attn.cu:34-57), which races when XLA calls handlers for several
// devices from several threads.  Here every cache is guarded.
#include "host.h"

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <set>
#include <utility>

namespace cfk {

namespace {

thread_local char t_last_error[512] = {0};

constexpr int kMaxDevices = 64;
std::once_flag g_dev_once[kMaxDevices];
DeviceInfo g_dev_info[kMaxDevices];
int g_dev_err[kMaxDevices];

std::mutex g_attr_mu;
std::set<std::pair<const void*, int>> g_attr_done;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
std::once_flag g_encode_once;
EncodeTiledFn g_encode = nullptr;

} // namespace

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
    va_end(ap);
    return code;
}

void clear_error() {
    t_last_error[0] = '\0';
}

int current_device(DeviceInfo* info) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        return fail(CFK_ERR_LAUNCH, "cudaGetDevice: %s", cudaGetErrorString(e));
    }
    if (dev < 0 || dev >= kMaxDevices) {
        return fail(CFK_ERR_UNSUPPORTED_DEVICE, "device ordinal %d out of range", dev);
    }
    // A thread that never made a runtime call that binds a context (a framework's worker
    // thread, e.g. an autograd engine's) has none current, and the driver's tensor-map encoder
    // then fails; cudaSetDevice binds the device's primary context once per thread.
    thread_local bool bound[kMaxDevices] = {};
    if (!bound[dev]) {
        e = cudaSetDevice(dev);
        if (e != cudaSuccess) {
            return fail(CFK_ERR_LAUNCH, "cudaSetDevice(%d): %s", dev, cudaGetErrorString(e));
        }
        bound[dev] = true;
    }
    std::call_once(g_dev_once[dev], [dev]() {
        DeviceInfo d;
        d.device = dev;
        int major = 0, minor = 0;
        cudaError_t r1 = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaError_t r2 = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
        cudaError_t r3 = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev);
        cudaError_t r4 =
            cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        d.cc = major * 10 + minor;
        g_dev_err[dev] = (r1 || r2 || r3 || r4) ? 1 : 0;
        g_dev_info[dev] = d;
    });
    if (g_dev_err[dev]) {
        return fail(CFK_ERR_LAUNCH, "cannot query attributes of device %d", dev);
    }
    *info = g_dev_info[dev];
    if (info->cc != 100) {
        return fail(CFK_ERR_UNSUPPORTED_DEVICE,
                    "device %d is sm_%d; this library holds sm_100a code only", dev, info->cc);
    }
    return CFK_OK;
}

int ensure_smem_attr(const void* kernel, int device, int bytes, const char* name,
                     int launch_regs) {
    std::lock_guard<std::mutex> lock(g_attr_mu);
    auto key = std::make_pair(kernel, device);
    if (g_attr_done.count(key)) {
        return CFK_OK;
    }
    if (launch_regs > 0) {
        // setmaxnreg.inc waits until the block's pool (threads x registers at launch) has the
        // registers: a kernel compiled with fewer than the split assumes must not launch
        cudaFuncAttributes a{};
        cudaError_t e = cudaFuncGetAttributes(&a, kernel);
        if (e != cudaSuccess) {
            return fail(CFK_ERR_LAUNCH, "%s: cudaFuncGetAttributes: %s", name,
                        cudaGetErrorString(e));
        }
        if (a.numRegs != launch_regs) {
            return fail(CFK_ERR_LAUNCH,
                        "%s: built with %d registers per thread; its register split needs %d",
                        name, a.numRegs, launch_regs);
        }
    }
    cudaError_t e =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) {
        return fail(CFK_ERR_LAUNCH, "%s: cudaFuncSetAttribute(%d bytes): %s", name, bytes,
                    cudaGetErrorString(e));
    }
    g_attr_done.insert(key);
    return CFK_OK;
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        return fail(CFK_ERR_LAUNCH, "%s launch: %s", what, cudaGetErrorString(e));
    }
    return CFK_OK;
}

namespace {

// cuTensorMapEncodeTiled of a rank-3 or rank-4 map (dim 0 contiguous)
int encode_tiled(CUtensorMap* map, int rank, const void* base, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes,
                 const char* what, bool f32, Map16 type16 = Map16::kBits) {
    std::call_once(g_encode_once, []() {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            g_encode = reinterpret_cast<EncodeTiledFn>(fn);
        }
    });
    if (!g_encode) {
        return fail(CFK_ERR_LAUNCH, "%s: driver has no cuTensorMapEncodeTiled", what);
    }
    CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE;
    switch (swizzle_bytes) {
    case 0:
        sw = CU_TENSOR_MAP_SWIZZLE_NONE;
        break;
    case 32:
        sw = CU_TENSOR_MAP_SWIZZLE_32B;
        break;
    case 64:
        sw = CU_TENSOR_MAP_SWIZZLE_64B;
        break;
    case 128:
        sw = CU_TENSOR_MAP_SWIZZLE_128B;
        break;
    default:
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: bad swizzle %d", what, swizzle_bytes);
    }
    cuuint64_t gdims[4];
    cuuint64_t gstrides[3];
    cuuint32_t gbox[4];
    cuuint32_t estr[4] = {1, 1, 1, 1};
    for (int i = 0; i < rank; ++i) {
        gdims[i] = dims[i];
        gbox[i] = box[i];
        if (i > 0) {
            gstrides[i - 1] = strides_bytes[i - 1];
        }
    }
    const CUtensorMapDataType dt =
        f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
            : (type16 == Map16::kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                      : (type16 == Map16::kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                               : CU_TENSOR_MAP_DATA_TYPE_UINT16));
    CUresult r = g_encode(map, dt,
                          static_cast<cuuint32_t>(rank), const_cast<void*>(base), gdims, gstrides,
                          gbox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        return fail(CFK_ERR_INVALID_ARGUMENT,
                    "%s: cuTensorMapEncodeTiled failed (%d): dims %llu x %llu x %llu x %llu", what,
                    static_cast<int>(r), static_cast<unsigned long long>(dims[0]),
                    static_cast<unsigned long long>(dims[1]),
                    static_cast<unsigned long long>(dims[2]),
                    static_cast<unsigned long long>(rank > 3 ? dims[3] : 1));
    }
    return CFK_OK;
}

} // namespace

int make_tmap_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                 uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1,
                 uint32_t b2, int swizzle_bytes, const char* what, bool f32) {
    const uint64_t dims[3] = {d0, d1, d2};
    const uint64_t strides[2] = {stride1_bytes, stride2_bytes};
    const uint32_t box[3] = {b0, b1, b2};
    return encode_tiled(map, 3, base, dims, strides, box, swizzle_bytes, what, f32);
}

int view_of(const char* fn, const char* name, const cfk_view* user, int64_t N, int64_t H,
            int64_t S, int64_t D, RowView* out) {
    if (!user) {
        *out = packed_view(N, H, S, D);
        return CFK_OK;
    }
    const int64_t ext[3] = {N, H, S};
    const int64_t str[3] = {user->b, user->h, user->s};
    const char* axis[3] = {"batch", "head", "sequence"};
    for (int i = 0; i < 3; ++i) {
        if (ext[i] > 1 && (str[i] <= 0 || str[i] % 8 != 0 || str[i] >= (1ll << 38))) {
            return fail(CFK_ERR_INVALID_ARGUMENT,
                        "%s: %s %s stride %lld must be a positive multiple of 8 elements", fn,
                        name, axis[i], static_cast<long long>(str[i]));
        }
    }
    // the farthest element must stay addressable: below 2^40 elements (2 TiB of 16-bit data)
    // keeps every offset the kernels form within int64 and within the TMA's address range
    const double last = static_cast<double>(N > 0 ? N - 1 : 0) * static_cast<double>(str[0]) +
                        static_cast<double>(H > 0 ? H - 1 : 0) * static_cast<double>(str[1]) +
                        static_cast<double>(S > 0 ? S - 1 : 0) * static_cast<double>(str[2]) +
                        static_cast<double>(D);
    if (last >= 1099511627776.0) {
        return fail(CFK_ERR_INVALID_ARGUMENT, "%s: %s view reaches past 2^40 elements", fn, name);
    }
    *out = RowView{N, H, S, user->b, user->h, user->s};
    return CFK_OK;
}

int make_tmap_rows(CUtensorMap* map, const void* base, const RowView& v, uint64_t d,
                   uint32_t box_rows, int swizzle_bytes, const char* what, Map16 type) {
    // dims (D, S, H, N); a dimension of extent 1 gets a harmless stride (its index is always 0)
    const uint64_t dims[4] = {d, static_cast<uint64_t>(v.S), static_cast<uint64_t>(v.H),
                              static_cast<uint64_t>(v.N)};
    const uint64_t fallback = 2 * d;
    const uint64_t strides[3] = {v.S > 1 ? 2 * static_cast<uint64_t>(v.s) : fallback,
                                 v.H > 1 ? 2 * static_cast<uint64_t>(v.h) : fallback,
                                 v.N > 1 ? 2 * static_cast<uint64_t>(v.b) : fallback};
    const uint32_t box[4] = {static_cast<uint32_t>(d), box_rows, 1, 1};
    return encode_tiled(map, 4, base, dims, strides, box, swizzle_bytes, what, false, type);
}

} // namespace cfk

extern "C" const char* cfk_last_error(void) {
    return cfk::t_last_error;
}

extern "C" const char* cfk_version(void) {
    return "colabfold-b200-kernels 0.1.0 (sm_100a)";
}
