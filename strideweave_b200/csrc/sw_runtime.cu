// sw_runtime.cu - device storage, copies, streams and the status plumbing of
// the C ABI (include/strideweave_b200.h).
#include <cstring>

#include "sw_common.cuh"
#include "sw_ptx.cuh"

namespace sw {

namespace {
thread_local std::string t_last_error;

// An mbarrier that nothing arrives on, waited for with the same bounded wait
// the contraction's pipeline uses: the wait gives up after `limit_ns`, records
// SW_ERR_TIMEOUT and the kernel returns.
__global__ void bounded_wait_probe(unsigned long long limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    const uint32_t addr = ptx::smem_addr(&bar);
    if (threadIdx.x == 0) {
        ptx::mbar_init(addr, 1);
        ptx::fence_barrier_init();
        ptx::mbar_wait(addr, 0, limit_ns);
    }
}
}  // namespace

__device__ int g_device_error = 0;

int fail(int code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

int ok() {
    t_last_error.clear();
    return SW_OK;
}

}  // namespace sw

using sw::fail;
using sw::ok;

extern "C" {

const char* sw_last_error(void) { return sw::t_last_error.c_str(); }

int sw_abi_version(void) { return 1; }

int sw_device_count(int* count) {
    if (!count) return fail(SW_ERR_INVALID, "sw_device_count: null output");
    *count = 0;
    cudaError_t err = cudaGetDeviceCount(count);
    if (err == cudaErrorNoDevice || err == cudaErrorInsufficientDriver) {
        cudaGetLastError();
        *count = 0;
        return ok();
    }
    SW_CUDA_TRY(err, "cudaGetDeviceCount");
    return ok();
}

int sw_set_device(int device) {
    SW_CUDA_TRY(cudaSetDevice(device), "cudaSetDevice");
    return ok();
}

int sw_get_device(int* device) {
    if (!device) return fail(SW_ERR_INVALID, "sw_get_device: null output");
    SW_CUDA_TRY(cudaGetDevice(device), "cudaGetDevice");
    return ok();
}

// Carrier storage comes from the device's stream-ordered memory pool on the
// legacy default stream (the stream every carrier operation is ordered on):
// allocation and release neither synchronise the device nor return memory to
// the driver between steps.
static int ensure_pool(int device) {
    static bool configured[64] = {};
    if (device < 0 || device >= 64 || configured[device]) return SW_OK;
    cudaMemPool_t pool;
    SW_CUDA_TRY(cudaDeviceGetDefaultMemPool(&pool, device), "cudaDeviceGetDefaultMemPool");
    uint64_t keep = ~uint64_t(0);
    SW_CUDA_TRY(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep), "pool release threshold");
    configured[device] = true;
    return SW_OK;
}

int sw_alloc(void** ptr, int64_t bytes) {
    if (!ptr) return fail(SW_ERR_INVALID, "sw_alloc: null output");
    *ptr = nullptr;
    if (bytes < 0) return fail(SW_ERR_INVALID, "sw_alloc: negative size %lld", (long long)bytes);
    if (bytes == 0) return ok();
    int dev = 0;
    SW_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
    int rc = ensure_pool(dev);
    if (rc != SW_OK) return rc;
    cudaError_t err = cudaMallocAsync(ptr, (size_t)bytes, (cudaStream_t)0);
    if (err == cudaErrorMemoryAllocation) {
        cudaGetLastError();
        return fail(SW_ERR_NOMEM, "sw_alloc: out of device memory (%lld bytes)", (long long)bytes);
    }
    SW_CUDA_TRY(err, "cudaMallocAsync");
    return ok();
}

int sw_free(void* ptr) {
    if (!ptr) return ok();
    SW_CUDA_TRY(cudaFreeAsync(ptr, (cudaStream_t)0), "cudaFreeAsync");
    return ok();
}

static int copy(void* dst, const void* src, int64_t bytes, cudaMemcpyKind kind,
                void* stream, const char* what) {
    if (bytes < 0) return fail(SW_ERR_INVALID, "%s: negative size", what);
    if (bytes == 0) return ok();
    if (!dst || !src) return fail(SW_ERR_INVALID, "%s: null pointer", what);
    SW_CUDA_TRY(cudaMemcpyAsync(dst, src, (size_t)bytes, kind, (cudaStream_t)stream), what);
    return ok();
}

int sw_memcpy_h2d(void* dst, const void* src, int64_t bytes, void* stream) {
    return copy(dst, src, bytes, cudaMemcpyHostToDevice, stream, "sw_memcpy_h2d");
}

int sw_memcpy_d2h(void* dst, const void* src, int64_t bytes, void* stream) {
    int rc = copy(dst, src, bytes, cudaMemcpyDeviceToHost, stream, "sw_memcpy_d2h");
    if (rc != SW_OK) return rc;
    // A pageable destination is only valid once the copy has landed.
    SW_CUDA_TRY(cudaStreamSynchronize((cudaStream_t)stream), "sw_memcpy_d2h sync");
    return ok();
}

int sw_memcpy_d2h_async(void* dst, const void* src, int64_t bytes, void* stream) {
    // no host synchronisation: the caller waits on the stream (or an event
    // recorded after the copy) before it reads the destination
    return copy(dst, src, bytes, cudaMemcpyDeviceToHost, stream, "sw_memcpy_d2h_async");
}

int sw_memcpy_d2d(void* dst, const void* src, int64_t bytes, void* stream) {
    return copy(dst, src, bytes, cudaMemcpyDeviceToDevice, stream, "sw_memcpy_d2d");
}

int sw_memset(void* dst, int value, int64_t bytes, void* stream) {
    if (bytes < 0) return fail(SW_ERR_INVALID, "sw_memset: negative size");
    if (bytes == 0) return ok();
    SW_CUDA_TRY(cudaMemsetAsync(dst, value, (size_t)bytes, (cudaStream_t)stream), "cudaMemsetAsync");
    return ok();
}

int sw_host_alloc(void** ptr, int64_t bytes) {
    if (!ptr || bytes < 0) return fail(SW_ERR_INVALID, "sw_host_alloc: bad argument");
    *ptr = nullptr;
    if (bytes == 0) return ok();
    SW_CUDA_TRY(cudaMallocHost(ptr, (size_t)bytes), "cudaMallocHost");
    return ok();
}

int sw_host_free(void* ptr) {
    if (!ptr) return ok();
    SW_CUDA_TRY(cudaFreeHost(ptr), "cudaFreeHost");
    return ok();
}

int sw_stream_create(void** stream) {
    if (!stream) return fail(SW_ERR_INVALID, "sw_stream_create: null output");
    cudaStream_t s;
    SW_CUDA_TRY(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
    *stream = (void*)s;
    return ok();
}

int sw_stream_destroy(void* stream) {
    if (!stream) return ok();
    SW_CUDA_TRY(cudaStreamDestroy((cudaStream_t)stream), "cudaStreamDestroy");
    return ok();
}

int sw_stream_synchronize(void* stream) {
    SW_CUDA_TRY(cudaStreamSynchronize((cudaStream_t)stream), "cudaStreamSynchronize");
    return ok();
}

int sw_device_sm_count(int* count) {
    if (!count) return fail(SW_ERR_INVALID, "sw_device_sm_count: null output");
    int dev = 0;
    SW_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
    SW_CUDA_TRY(cudaDeviceGetAttribute(count, cudaDevAttrMultiProcessorCount, dev), "SM count");
    return ok();
}

int sw_event_create(void** event, int timing) {
    if (!event) return fail(SW_ERR_INVALID, "sw_event_create: null output");
    cudaEvent_t e;
    SW_CUDA_TRY(cudaEventCreateWithFlags(&e, timing ? cudaEventDefault : cudaEventDisableTiming), "cudaEventCreate");
    *event = (void*)e;
    return ok();
}

int sw_event_destroy(void* event) {
    if (!event) return ok();
    SW_CUDA_TRY(cudaEventDestroy((cudaEvent_t)event), "cudaEventDestroy");
    return ok();
}

int sw_event_record(void* event, void* stream) {
    if (!event) return fail(SW_ERR_INVALID, "sw_event_record: null event");
    SW_CUDA_TRY(cudaEventRecord((cudaEvent_t)event, (cudaStream_t)stream), "cudaEventRecord");
    return ok();
}

int sw_stream_wait_event(void* stream, void* event) {
    if (!event) return fail(SW_ERR_INVALID, "sw_stream_wait_event: null event");
    SW_CUDA_TRY(cudaStreamWaitEvent((cudaStream_t)stream, (cudaEvent_t)event, 0), "cudaStreamWaitEvent");
    return ok();
}

int sw_event_elapsed_ms(void* start, void* end, float* ms) {
    if (!start || !end || !ms) return fail(SW_ERR_INVALID, "sw_event_elapsed_ms: null argument");
    SW_CUDA_TRY(cudaEventSynchronize((cudaEvent_t)end), "cudaEventSynchronize");
    SW_CUDA_TRY(cudaEventElapsedTime(ms, (cudaEvent_t)start, (cudaEvent_t)end), "cudaEventElapsedTime");
    return ok();
}

int sw_graph_capture_begin(void* stream) {
    if (!stream) return fail(SW_ERR_INVALID, "sw_graph_capture_begin: capture needs a stream from sw_stream_create");
    SW_CUDA_TRY(cudaStreamBeginCapture((cudaStream_t)stream, cudaStreamCaptureModeThreadLocal),
                "cudaStreamBeginCapture");
    return ok();
}

int sw_graph_capture_end(void* stream, void** graph_exec) {
    if (!stream || !graph_exec) return fail(SW_ERR_INVALID, "sw_graph_capture_end: null argument");
    *graph_exec = nullptr;
    cudaGraph_t graph = nullptr;
    SW_CUDA_TRY(cudaStreamEndCapture((cudaStream_t)stream, &graph), "cudaStreamEndCapture");
    cudaGraphExec_t exec = nullptr;
    const cudaError_t err = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    SW_CUDA_TRY(err, "cudaGraphInstantiate");
    *graph_exec = (void*)exec;
    return ok();
}

int sw_graph_launch(void* graph_exec, void* stream) {
    if (!graph_exec) return fail(SW_ERR_INVALID, "sw_graph_launch: null graph");
    SW_CUDA_TRY(cudaGraphLaunch((cudaGraphExec_t)graph_exec, (cudaStream_t)stream), "cudaGraphLaunch");
    return ok();
}

int sw_graph_destroy(void* graph_exec) {
    if (!graph_exec) return ok();
    SW_CUDA_TRY(cudaGraphExecDestroy((cudaGraphExec_t)graph_exec), "cudaGraphExecDestroy");
    return ok();
}

int sw_probe_bounded_wait(int64_t limit_ns, void* stream) {
    if (limit_ns < 0 || limit_ns > 1000000000)
        return fail(SW_ERR_INVALID, "sw_probe_bounded_wait: the limit must lie in [0, 1 s]");
    sw::bounded_wait_probe<<<1, 32, 0, (cudaStream_t)stream>>>((unsigned long long)limit_ns);
    SW_LAUNCH_CHECK("bounded wait probe launch");
    return ok();
}

int sw_device_status(int* status) {
    if (!status) return fail(SW_ERR_INVALID, "sw_device_status: null output");
    SW_CUDA_TRY(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    int value = 0, zero = 0;
    SW_CUDA_TRY(cudaMemcpyFromSymbol(&value, sw::g_device_error, sizeof(int)), "read device status");
    SW_CUDA_TRY(cudaMemcpyToSymbol(sw::g_device_error, &zero, sizeof(int)), "clear device status");
    *status = value;
    return ok();
}

}  // extern "C"
