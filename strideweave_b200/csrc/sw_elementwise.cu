// sw_elementwise.cu - the elementwise work around the contractions of an MLP
// training step: GELU and its gradient, the SGD update, and mean squared
// error with its gradient.  Contiguous Float32 buffers; 16-byte vectors when
// the pointers allow.
#include <algorithm>

#include "sw_common.cuh"
#include "sw_gelu.cuh"

namespace sw {
namespace {

template <int OP>
__device__ __forceinline__ float apply(float a, float b, float alpha) {
    if (OP == SW_EW_GELU) return gelu(a);
    if (OP == SW_EW_GELU_GRAD) return b * gelu_grad(a);
    return fmaf(alpha, b, a);
}

template <int OP>
__global__ void __launch_bounds__(256) ew_kernel(int64_t n, const float* __restrict__ a, const float* __restrict__ b,
                                                 float* out, float alpha, bool vec) {
    pdl_enter();
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    const int64_t t0 = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (vec) {
        const int64_t nv = n / 4;
        for (int64_t i = t0; i < nv; i += stride) {
            const float4 x = reinterpret_cast<const float4*>(a)[i];
            float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
            if (OP != SW_EW_GELU) y = reinterpret_cast<const float4*>(b)[i];
            float4 r;
            r.x = apply<OP>(x.x, y.x, alpha);
            r.y = apply<OP>(x.y, y.y, alpha);
            r.z = apply<OP>(x.z, y.z, alpha);
            r.w = apply<OP>(x.w, y.w, alpha);
            reinterpret_cast<float4*>(out)[i] = r;
        }
        for (int64_t i = nv * 4 + t0; i < n; i += stride) out[i] = apply<OP>(a[i], OP == SW_EW_GELU ? 0.f : b[i], alpha);
    } else {
        for (int64_t i = t0; i < n; i += stride) out[i] = apply<OP>(a[i], OP == SW_EW_GELU ? 0.f : b[i], alpha);
    }
}

__global__ void __launch_bounds__(256) mse_loss_kernel(int64_t n, const float* __restrict__ p,
                                                       const float* __restrict__ t, float* loss, float inv_n) {
    float acc = 0.0f;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const float d = p[i] - t[i];
        acc = fmaf(d, d, acc);
    }
    for (int s = 16; s > 0; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
    __shared__ float part[8];
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        float b = 0.0f;
        for (int w = 0; w < 8; ++w) b += part[w];
        atomicAdd(loss, b * inv_n);
    }
}

__global__ void __launch_bounds__(256) mse_grad_kernel(int64_t n, const float* __restrict__ p,
                                                       const float* __restrict__ t, const float* __restrict__ up,
                                                       float* __restrict__ g, float two_over_n) {
    pdl_enter();
    const float s = (up ? up[0] : 1.0f) * two_over_n;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        g[i] = s * (p[i] - t[i]);
}

// Loss and gradient in one pass (no upstream gradient: the loss is the root):
// d = p - t once per element, grad = two_over_n * d, loss += sum d^2 / n.
// The gradient is the same expression as mse_grad_kernel's; the loss sums in
// another order (an atomic sum over blocks either way).  16-byte vectors when
// `vec`.
__global__ void __launch_bounds__(256) mse_fused_kernel(int64_t n, const float* __restrict__ p,
                                                        const float* __restrict__ t, float* loss,
                                                        float* __restrict__ g, float inv_n, float two_over_n,
                                                        bool vec) {
    float acc = 0.0f;
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    const int64_t t0 = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    int64_t tail = 0;
    if (vec) {
        const int64_t nv = n / 4;
        for (int64_t i = t0; i < nv; i += stride) {
            const float4 a = reinterpret_cast<const float4*>(p)[i];
            const float4 b = reinterpret_cast<const float4*>(t)[i];
            const float d0 = a.x - b.x, d1 = a.y - b.y, d2 = a.z - b.z, d3 = a.w - b.w;
            acc = fmaf(d0, d0, acc);
            acc = fmaf(d1, d1, acc);
            acc = fmaf(d2, d2, acc);
            acc = fmaf(d3, d3, acc);
            reinterpret_cast<float4*>(g)[i] = make_float4(two_over_n * d0, two_over_n * d1, two_over_n * d2,
                                                          two_over_n * d3);
        }
        tail = nv * 4;
    }
    for (int64_t i = tail + t0; i < n; i += stride) {
        const float d = p[i] - t[i];
        acc = fmaf(d, d, acc);
        g[i] = two_over_n * d;
    }
    for (int sh = 16; sh > 0; sh >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, sh);
    __shared__ float part[8];
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        float b = 0.0f;
        for (int w = 0; w < 8; ++w) b += part[w];
        atomicAdd(loss, b * inv_n);
    }
}

int grid_of(int64_t n) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, int64_t(sms) * 8));
}

}  // namespace
}  // namespace sw

extern "C" int sw_elementwise_f32(int op, int64_t n, const float* a, const float* b, float* out, float alpha,
                                  void* stream) {
    using namespace sw;
    if (op < SW_EW_GELU || op > SW_EW_AXPY) return fail(SW_ERR_INVALID, "sw_elementwise_f32: unknown op %d", op);
    if (n < 0) return fail(SW_ERR_INVALID, "sw_elementwise_f32: negative size");
    if (n == 0) return ok();
    if (!a || !out || (op != SW_EW_GELU && !b)) return fail(SW_ERR_INVALID, "sw_elementwise_f32: null pointer");
    const bool vec = ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(out) |
                       (op != SW_EW_GELU ? reinterpret_cast<uintptr_t>(b) : 0)) & 15) == 0;
    cudaStream_t s = (cudaStream_t)stream;
    const int grid = grid_of(vec ? n / 4 + 1 : n);
    auto kernel = op == SW_EW_GELU        ? ew_kernel<SW_EW_GELU>
                  : op == SW_EW_GELU_GRAD ? ew_kernel<SW_EW_GELU_GRAD>
                                          : ew_kernel<SW_EW_AXPY>;
    SW_CUDA_TRY(launch_pdl(kernel, grid, 256, 0, s, n, a, b, out, alpha, vec), "sw_elementwise_f32 launch");
    SW_LAUNCH_CHECK("sw_elementwise_f32 launch");
    return ok();
}

extern "C" int sw_mse_f32(int64_t n, const float* pred, const float* target, float* loss, const float* upstream,
                          float* grad, void* stream) {
    using namespace sw;
    if (n <= 0) return fail(SW_ERR_INVALID, "sw_mse_f32: the mean of an empty set");
    if (!pred || !target || (!loss && !grad)) return fail(SW_ERR_INVALID, "sw_mse_f32: null pointer");
    cudaStream_t s = (cudaStream_t)stream;
    const int grid = grid_of(n);
    if (loss && grad && !upstream) {
        // the training step's case: one pass writes the gradient and sums the loss
        const bool vec = ((reinterpret_cast<uintptr_t>(pred) | reinterpret_cast<uintptr_t>(target) |
                           reinterpret_cast<uintptr_t>(grad)) & 15) == 0;
        SW_CUDA_TRY(cudaMemsetAsync(loss, 0, sizeof(float), s), "mse loss reset");
        mse_fused_kernel<<<vec ? grid_of(n / 4 + 1) : grid, 256, 0, s>>>(n, pred, target, loss, grad,
                                                                        1.0f / float(n), 2.0f / float(n), vec);
        SW_LAUNCH_CHECK("sw_mse_f32 launch");
        return ok();
    }
    if (loss) {
        SW_CUDA_TRY(cudaMemsetAsync(loss, 0, sizeof(float), s), "mse loss reset");
        mse_loss_kernel<<<grid, 256, 0, s>>>(n, pred, target, loss, 1.0f / float(n));
        SW_LAUNCH_CHECK("sw_mse_f32 loss launch");
    }
    if (grad) {
        SW_CUDA_TRY(launch_pdl(mse_grad_kernel, grid, 256, 0, s, n, pred, target, upstream, grad, 2.0f / float(n)),
                    "mse grad launch");
        SW_LAUNCH_CHECK("sw_mse_f32 grad launch");
    }
    return ok();
}
