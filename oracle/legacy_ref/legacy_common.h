// Shared helpers of the legacy-comparator wrappers -- TEST INFRASTRUCTURE (see build.py).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>

#include "xla/ffi/api/ffi.h"

// Copies the handler's error message (if any) and returns its code (0 = success).
static inline int legacy_result(const xla::ffi::Error& e, char* msg, int msg_len) {
    if (msg && msg_len > 0) {
        std::strncpy(msg, e.message().c_str(), static_cast<size_t>(msg_len - 1));
        msg[msg_len - 1] = '\0';
    }
    return e.code();
}

static inline int legacy_device() {
    int d = 0;
    cudaGetDevice(&d);
    return d;
}

#define LEGACY_API extern "C" __attribute__((visibility("default")))
