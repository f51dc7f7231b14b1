// abi_util.h -- host-side helpers for the C ABI: the per-thread error message,
// CUDA error mapping, tunables read from the environment, device attributes.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <string>

#include "../../include/swann_b200.h"

namespace abi {

inline std::string& last_error() {
    static thread_local std::string msg;
    return msg;
}

inline int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    last_error() = buf;
    return code;
}

inline int cuda_fail(cudaError_t e, const char* what) {
    return fail(SWB_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

inline int cuda_check(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, what);
    return SWB_OK;
}

inline int env_int(const char* name, int dflt) {
    const char* v = std::getenv(name);
    if (!v || !*v) return dflt;
    return std::atoi(v);
}

inline int current_device() {
    int dev = 0;
    cudaGetDevice(&dev);
    return dev;
}

inline int max_smem_optin() {
    static int cache[64] = {0};
    const int dev = current_device();
    if (dev >= 0 && dev < 64 && cache[dev]) return cache[dev];
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) v = 48 * 1024;
    if (dev >= 0 && dev < 64) cache[dev] = v;
    return v;
}

inline int num_sms() {
    static int cache[64] = {0};
    const int dev = current_device();
    if (dev >= 0 && dev < 64 && cache[dev]) return cache[dev];
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) v = 132;
    if (dev >= 0 && dev < 64) cache[dev] = v;
    return v;
}

}  // namespace abi
