// sw_peer.cu - the pieces of a K-split contraction that reduces over NVLink
// peer memory instead of a collective library.
//
// Every rank owns a landing buffer of `world` slots, slot p holding rank p's
// Float32 partial of the C rows this rank owns.  The contraction writes each
// of its row blocks straight into the owner's slot (sw_mx_gemm_routed, plain
// peer stores over NVLink, no TMA and no multicast), then signals every owner
// through a flag in the owner's memory; the owner waits for all `world` flags
// of the step and sums its slots in rank order, which makes the result the
// same bit for bit on every run, then tells every writer that its slot is free
// for the next step.
//
//   sw_ipc_alloc / sw_ipc_open / sw_ipc_close / sw_ipc_free - the landing
//       buffer and its flags, shared between the processes of one node
//       (CUDA IPC; each process opens the others' buffers once);
//   sw_peer_wait   - waits, bounded, until `count` flags in this GPU's memory
//       reach a step number (the other ranks write them);
//   sw_peer_signal - after a system-scope fence, writes a step number into a
//       flag in each of `count` peers' memory;
//   sw_sum_slots_f32 - out = slot 0 + slot 1 + ... in that order.
//
// A wait that runs past its limit records SW_ERR_TIMEOUT in the device error
// word and returns: a rank that died turns into a status the host reads, and
// the GPU stays usable.  Each rank runs its kernels on its own GPU; no two
// ranks ever share one.
#include <algorithm>

#include "sw_common.cuh"
#include "sw_ptx.cuh"

namespace sw {
namespace {

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Flags count steps and only grow; "reached" compares modulo 2^32.
__device__ __forceinline__ bool reached(uint32_t flag, uint32_t target) { return int32_t(flag - target) >= 0; }

__global__ void peer_wait_kernel(const uint32_t* flags, int count, uint32_t target, unsigned long long limit_ns) {
    if (threadIdx.x >= count) return;
    const uint32_t* f = flags + threadIdx.x;
    if (reached(ld_acquire_sys(f), target)) return;
    const uint64_t t0 = ptx::globaltimer_ns();
    for (uint32_t i = 1; i < (1u << 30); ++i) {
        if (reached(ld_acquire_sys(f), target)) return;
        if ((i & 63) == 0) {
            if (ptx::globaltimer_ns() - t0 > limit_ns) break;
            __nanosleep(256);
        }
    }
    report_device_error(SW_ERR_TIMEOUT);
}

constexpr int kMaxPeers = 8;

struct PeerFlags {
    uint32_t* flag[kMaxPeers];
};

__global__ void peer_signal_kernel(PeerFlags dst, int count, uint32_t value) {
    // every store the stream issued before this kernel (the contraction's
    // peer writes included) is performed before any flag is seen
    __threadfence_system();
    if (threadIdx.x < count) st_release_sys(dst.flag[threadIdx.x], value);
}

// A block sums tiles of kSumUnroll x 256 vectors: each thread keeps kSumUnroll
// independent 16-byte loads of every slot in flight (a 2-slot sum streams
// 3 bytes of HBM traffic per output byte and needs that depth to reach it).
constexpr int kSumThreads = 256;
constexpr int kSumUnroll = 4;

__global__ void __launch_bounds__(kSumThreads) sum_slots_kernel(const float4* __restrict__ slots, int64_t slot_vec,
                                                                int count, float4* __restrict__ out) {
    pdl_enter();
    constexpr int64_t kTile = int64_t(kSumThreads) * kSumUnroll;
    for (int64_t t0 = int64_t(blockIdx.x) * kTile; t0 < slot_vec; t0 += int64_t(gridDim.x) * kTile) {
        const int64_t i0 = t0 + threadIdx.x;
        float4 acc[kSumUnroll];
        // L2, where the peers' writes land, not L1: every load goes past L1
#pragma unroll
        for (int u = 0; u < kSumUnroll; ++u) {
            const int64_t i = i0 + u * kSumThreads;
            acc[u] = i < slot_vec ? __ldcg(slots + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        for (int s = 1; s < count; ++s) {
            const float4* slot = slots + int64_t(s) * slot_vec;
            float4 v[kSumUnroll];
#pragma unroll
            for (int u = 0; u < kSumUnroll; ++u) {
                const int64_t i = i0 + u * kSumThreads;
                v[u] = i < slot_vec ? __ldcg(slot + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < kSumUnroll; ++u) {
                acc[u].x += v[u].x;
                acc[u].y += v[u].y;
                acc[u].z += v[u].z;
                acc[u].w += v[u].w;
            }
        }
#pragma unroll
        for (int u = 0; u < kSumUnroll; ++u) {
            const int64_t i = i0 + u * kSumThreads;
            if (i < slot_vec) out[i] = acc[u];
        }
    }
}

int sm_count_peer() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        cudaGetLastError();
        sms = 148;
    }
    return sms;
}

}  // namespace
}  // namespace sw

extern "C" int sw_ipc_alloc(void** ptr, int64_t bytes, uint8_t* handle) {
    using namespace sw;
    if (!ptr || !handle || bytes <= 0) return fail(SW_ERR_INVALID, "sw_ipc_alloc: bad argument");
    *ptr = nullptr;
    void* p = nullptr;
    cudaError_t err = cudaMalloc(&p, (size_t)bytes);
    if (err == cudaErrorMemoryAllocation) {
        cudaGetLastError();
        return fail(SW_ERR_NOMEM, "sw_ipc_alloc: out of device memory (%lld bytes)", (long long)bytes);
    }
    SW_CUDA_TRY(err, "cudaMalloc (IPC buffer)");
    cudaIpcMemHandle_t h;
    err = cudaIpcGetMemHandle(&h, p);
    if (err != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(err, "cudaIpcGetMemHandle");
    }
    static_assert(sizeof(h) == SW_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    *ptr = p;
    return ok();
}

extern "C" int sw_ipc_free(void* ptr) {
    if (!ptr) return sw::ok();
    SW_CUDA_TRY(cudaFree(ptr), "cudaFree (IPC buffer)");
    return sw::ok();
}

extern "C" int sw_ipc_open(const uint8_t* handle, void** ptr) {
    using namespace sw;
    if (!handle || !ptr) return fail(SW_ERR_INVALID, "sw_ipc_open: null argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    SW_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    *ptr = p;
    return ok();
}

extern "C" int sw_ipc_close(void* ptr) {
    if (!ptr) return sw::ok();
    SW_CUDA_TRY(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
    return sw::ok();
}

extern "C" int sw_peer_wait(const uint32_t* flags, int count, uint32_t target, int64_t limit_ns, void* stream) {
    using namespace sw;
    if (count < 0 || count > 1024) return fail(SW_ERR_INVALID, "sw_peer_wait: bad flag count %d", count);
    if (count == 0) return ok();
    if (!flags) return fail(SW_ERR_INVALID, "sw_peer_wait: null flags");
    if (limit_ns <= 0 || limit_ns > 10000000000LL)
        return fail(SW_ERR_INVALID, "sw_peer_wait: the limit must lie in (0, 10 s]");
    peer_wait_kernel<<<1, 32 * ((count + 31) / 32), 0, (cudaStream_t)stream>>>(flags, count, target,
                                                                                (unsigned long long)limit_ns);
    SW_LAUNCH_CHECK("sw_peer_wait launch");
    return ok();
}

extern "C" int sw_peer_signal(uint32_t* const* flags, int count, uint32_t value, void* stream) {
    using namespace sw;
    if (count < 0 || count > kMaxPeers) return fail(SW_ERR_INVALID, "sw_peer_signal: at most %d flags", kMaxPeers);
    if (count == 0) return ok();
    if (!flags) return fail(SW_ERR_INVALID, "sw_peer_signal: null flag list");
    PeerFlags f{};
    for (int i = 0; i < count; ++i) {
        if (!flags[i]) return fail(SW_ERR_INVALID, "sw_peer_signal: null flag %d", i);
        f.flag[i] = flags[i];
    }
    peer_signal_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(f, count, value);
    SW_LAUNCH_CHECK("sw_peer_signal launch");
    return ok();
}

extern "C" int sw_sum_slots_f32(const float* slots, int64_t slot_elems, int count, float* out, void* stream) {
    using namespace sw;
    if (slot_elems < 0 || count < 1) return fail(SW_ERR_INVALID, "sw_sum_slots_f32: bad extent");
    if (slot_elems == 0) return ok();
    if (!slots || !out) return fail(SW_ERR_INVALID, "sw_sum_slots_f32: null pointer");
    if (slot_elems % 4 || ((reinterpret_cast<uintptr_t>(slots) | reinterpret_cast<uintptr_t>(out)) & 15))
        return fail(SW_ERR_INVALID, "sw_sum_slots_f32: slots of whole 16-byte vectors, 16-byte aligned");
    const int64_t vecs = slot_elems / 4;
    const int64_t tile = int64_t(kSumThreads) * kSumUnroll;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((vecs + tile - 1) / tile, int64_t(sm_count_peer()) * 8));
    SW_CUDA_TRY(launch_pdl(sum_slots_kernel, grid, kSumThreads, 0, (cudaStream_t)stream,
                           reinterpret_cast<const float4*>(slots), vecs, count, reinterpret_cast<float4*>(out)),
                "sum_slots launch");
    SW_LAUNCH_CHECK("sw_sum_slots_f32 launch");
    return ok();
}
