// status.cu -- the per-device status word that bounded waits write when they give up.
#include "host.h"
#include "sm100.cuh"

namespace cfk {
__device__ uint32_t g_status_word = 0;
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
