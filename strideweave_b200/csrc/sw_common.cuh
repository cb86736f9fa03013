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

// Programmatic dependent launch: a grid launched with launch_pdl may be
// scheduled while the previous grid on its stream drains.  It calls
// pdl_enter() before touching global memory: that waits for the previous grid
// (and its memory) to complete, then lets the next grid begin launching.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launches `kernel` with programmatic stream serialization.
template <class... KArgs, class... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

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
