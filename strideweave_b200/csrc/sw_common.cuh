// sw_common.cuh - status handling shared by every translation unit of the
// B200 carrier library.  Host entry points return SW_* codes and record a
// per-thread message; device code reports through one error word.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "strideweave_b200.h"

namespace sw {

// Sets the calling thread's last-error message and returns `code`.
int fail(int code, const char* fmt, ...);

// Clears the calling thread's last-error message and returns SW_OK.
int ok();

// Converts a CUDA error into SW_ERR_CUDA with context.
inline int cuda_fail(cudaError_t err, const char* what) {
    return fail(SW_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

// The device-side error word (defined in sw_runtime.cu).  A bounded wait that
// gives up, or a device bound check that trips, stores its SW_* code here and
// returns; the host reads it with sw_device_status().
extern __device__ int g_device_error;

__device__ __forceinline__ void report_device_error(int code) {
    atomicCAS(&g_device_error, 0, code);
}

// Wall-time cap of every device-side wait: far above any legitimate wait
// (microseconds) and far below a watchdog timeout.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

}  // namespace sw

#define SW_CUDA_TRY(expr, what)                         \
    do {                                                \
        cudaError_t err__ = (expr);                     \
        if (err__ != cudaSuccess) return ::sw::cuda_fail(err__, what); \
    } while (0)

#define SW_LAUNCH_CHECK(what)                                   \
    do {                                                        \
        cudaError_t err__ = cudaGetLastError();                 \
        if (err__ != cudaSuccess) return ::sw::cuda_fail(err__, what); \
    } while (0)
