// status.cu -- the per-device status word that bounded waits write when they give up, the
// per-device wait limit, and a self-test of the give-up path.
#include "host.h"
#include "sm100.cuh"

namespace cfk {
namespace {

// One CTA of one warp that waits on an mbarrier no thread ever arrives on.  The wait runs the
// kernels' own waiting loop (mbar_wait_limit_s) and gives up after `limit_ns` (0: the device's
// configured limit), recording kStatusTimeoutBarrier in the status word; the kernel then
// returns normally.  No TMA, tensor-memory or MMA work is in flight.  `result` (device memory)
// receives 1 if the wait gave up, 2 if it completed (it cannot), 0 if the kernel did not run.
__global__ void wait_timeout_selftest_kernel(unsigned long long limit_ns, uint32_t* result) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t abort_word;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_word = 0;
        fence_mbar_init();
    }
    __syncthreads();
    const unsigned long long limit = limit_ns ? limit_ns : wait_limit_ns();
    const bool ok = mbar_wait_limit_s(smem_u32(&bar), 0, smem_u32(&abort_word), limit);
    __syncwarp();
    if (threadIdx.x == 0) {
        *result = ok ? 2u : 1u;
    }
}

} // namespace
} // namespace cfk

extern "C" int cfk_device_status(uint32_t* code) {
    if (!code) {
        return cfk::fail(CFK_ERR_INVALID_ARGUMENT, "cfk_device_status: null pointer");
    }
    cfk::DeviceInfo info;
    CFK_TRY(cfk::current_device(&info));
    cudaError_t e = cudaMemcpyFromSymbol(code, cfk::g_status_word, sizeof(uint32_t));
    if (e != cudaSuccess) {
        return cfk::fail(CFK_ERR_LAUNCH, "cfk_device_status: %s", cudaGetErrorString(e));
    }
    return CFK_OK;
}

extern "C" int cfk_clear_device_status(void) {
    cfk::DeviceInfo info;
    CFK_TRY(cfk::current_device(&info));
    const uint32_t zero = 0;
    cudaError_t e = cudaMemcpyToSymbol(cfk::g_status_word, &zero, sizeof(uint32_t));
    if (e != cudaSuccess) {
        return cfk::fail(CFK_ERR_LAUNCH, "cfk_clear_device_status: %s", cudaGetErrorString(e));
    }
    return CFK_OK;
}

namespace {
constexpr unsigned long long kMinWaitLimitNs = 100000ull;         // 0.1 ms
constexpr unsigned long long kMaxWaitLimitNs = 600000000000ull;   // 10 minutes
} // namespace

extern "C" int cfk_set_wait_limit_ns(uint64_t ns) {
    cfk::clear_error();
    if (ns < kMinWaitLimitNs || ns > kMaxWaitLimitNs) {
        return cfk::fail(CFK_ERR_INVALID_ARGUMENT,
                         "cfk_set_wait_limit_ns: %llu ns outside [%llu, %llu]",
                         static_cast<unsigned long long>(ns), kMinWaitLimitNs, kMaxWaitLimitNs);
    }
    cfk::DeviceInfo info;
    CFK_TRY(cfk::current_device(&info));
    const unsigned long long v = ns;
    cudaError_t e = cudaMemcpyToSymbol(cfk::g_wait_limit_ns, &v, sizeof(v));
    if (e != cudaSuccess) {
        return cfk::fail(CFK_ERR_LAUNCH, "cfk_set_wait_limit_ns: %s", cudaGetErrorString(e));
    }
    return CFK_OK;
}

extern "C" int cfk_get_wait_limit_ns(uint64_t* ns) {
    cfk::clear_error();
    if (!ns) {
        return cfk::fail(CFK_ERR_INVALID_ARGUMENT, "cfk_get_wait_limit_ns: null pointer");
    }
    cfk::DeviceInfo info;
    CFK_TRY(cfk::current_device(&info));
    unsigned long long v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, cfk::g_wait_limit_ns, sizeof(v));
    if (e != cudaSuccess) {
        return cfk::fail(CFK_ERR_LAUNCH, "cfk_get_wait_limit_ns: %s", cudaGetErrorString(e));
    }
    *ns = v;
    return CFK_OK;
}

extern "C" int cfk_test_wait_timeout(cfk_stream_t stream, uint64_t limit_ns, uint32_t* result) {
    cfk::clear_error();
    if (!result) {
        return cfk::fail(CFK_ERR_INVALID_ARGUMENT, "cfk_test_wait_timeout: null result");
    }
    if (limit_ns != 0 && (limit_ns < kMinWaitLimitNs || limit_ns > 100000000ull)) {
        return cfk::fail(CFK_ERR_INVALID_ARGUMENT,
                         "cfk_test_wait_timeout: limit %llu ns outside [%llu, 1e8] (or 0 for the "
                         "device's limit)",
                         static_cast<unsigned long long>(limit_ns), kMinWaitLimitNs);
    }
    cfk::DeviceInfo info;
    CFK_TRY(cfk::current_device(&info));
    cfk::wait_timeout_selftest_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        limit_ns, result);
    return cfk::check_launch("wait_timeout_selftest");
}
