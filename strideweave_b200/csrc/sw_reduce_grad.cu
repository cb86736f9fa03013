// sw_reduce_grad.cu - vector-Jacobian products of the layout-aware reductions
// (reduce_sum and reduce_max), written into the gradient's own placement.
//
// The rules are the reference CPU carrier's:
//   reduce_sum (src/strideweave/carriers/cpu/native/ops/reduce_sum.cpp:120-150):
//     every element of fibre i receives grad_out[i];
//   reduce_max (src/strideweave/carriers/cpu/native/_cpu_reduction.hpp:155-182):
//     the maximum is recomputed with the forward rule, the gradient is split
//     evenly between the elements equal to it (grad_out[i] / winners, a
//     binary32 division), the others get 0, and a NaN maximum gives NaN to
//     the whole fibre.
// One warp per kept ordinal; lanes stride the fibre.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "sw_common.cuh"

namespace sw {
namespace {

struct Leaves {
    int rank;
    int64_t shape[SW_MAX_LEAVES];
    int64_t stride[SW_MAX_LEAVES];
};

struct GradPlan {
    int kind;
    int64_t n_kept, n_red;
    int64_t x_offset, x_size, g_offset, g_size;
    Leaves xk, xr, gk, gr;
    int swz_rank;
    int swz_bits[SW_MAX_SWIZZLE], swz_base[SW_MAX_SWIZZLE], swz_shift[SW_MAX_SWIZZLE];
    int dswz_rank;  // the destination's carrier swizzle (view copies only)
    int dswz_bits[SW_MAX_SWIZZLE], dswz_base[SW_MAX_SWIZZLE], dswz_shift[SW_MAX_SWIZZLE];
};

__device__ __forceinline__ int64_t swizzle_stages(int rank, const int* bits, const int* base, const int* shift,
                                                  int64_t r) {
    for (int s = 0; s < rank; ++s) {
        const int64_t mask = (int64_t(1) << bits[s]) - 1;
        if (shift[s] > 0) r ^= ((r >> (base[s] + shift[s])) & mask) << base[s];
        else r ^= ((r >> base[s]) & mask) << (base[s] - shift[s]);
    }
    return r;
}

__device__ __forceinline__ int64_t decompose(const Leaves& l, int64_t i) {
    int64_t off = 0;
    for (int d = 0; d < l.rank; ++d) {
        off += (i % l.shape[d]) * l.stride[d];
        i /= l.shape[d];
    }
    return off;
}

__device__ __forceinline__ int64_t swz(const GradPlan& p, int64_t r) {
    return swizzle_stages(p.swz_rank, p.swz_bits, p.swz_base, p.swz_shift, r);
}

__device__ __forceinline__ float max_rule(float a, float b) {
    if (isnan(a)) return a;
    if (isnan(b)) return b;
    if (a == b && a == 0.0f) return 0.0f;
    return a > b ? a : b;
}

__device__ __forceinline__ float read_x(const float* x, const GradPlan& p, int64_t row, int64_t j) {
    const int64_t f = swz(p, row + decompose(p.xr, j));
    if (f < 0 || f >= p.x_size) {
        report_device_error(SW_ERR_INVALID);
        return 0.0f;
    }
    return x[f];
}

__global__ void __launch_bounds__(256) reduce_grad_kernel(const float* __restrict__ x,
                                                          const float* __restrict__ gout, float* __restrict__ gin,
                                                          GradPlan p) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t i = warp; i < p.n_kept; i += nwarps) {
        const float g = gout[i];
        const int64_t grow = p.g_offset + decompose(p.gk, i);
        if (p.kind == SW_REDUCE_SUM) {
            for (int64_t j = lane; j < p.n_red; j += 32) gin[grow + decompose(p.gr, j)] = g;
            continue;
        }
        const int64_t xrow = p.x_offset + decompose(p.xk, i);
        // exact maximum: the max rule is associative and commutative once the
        // first NaN is chosen by ordinal
        float m = -INFINITY;
        int64_t first_nan = INT64_MAX;
        for (int64_t j = lane; j < p.n_red; j += 32) {
            const float v = read_x(x, p, xrow, j);
            if (isnan(v)) {
                if (j < first_nan) first_nan = j;
            } else {
                m = max_rule(m, v);
            }
        }
        for (int s = 16; s > 0; s >>= 1) {
            m = max_rule(m, __shfl_xor_sync(0xffffffffu, m, s));
            first_nan = min(first_nan, (int64_t)__shfl_xor_sync(0xffffffffu, (long long)first_nan, s));
        }
        const bool nan_max = first_nan != INT64_MAX;
        long long winners = 0;
        if (!nan_max) {
            for (int64_t j = lane; j < p.n_red; j += 32) winners += (read_x(x, p, xrow, j) == m);
            for (int s = 16; s > 0; s >>= 1) winners += __shfl_xor_sync(0xffffffffu, winners, s);
        }
        const float each = nan_max ? __uint_as_float(0x7FC00000u) : __fdiv_rn(g, float(winners));
        for (int64_t j = lane; j < p.n_red; j += 32) {
            float out;
            if (nan_max) out = each;
            else out = read_x(x, p, xrow, j) == m ? each : 0.0f;
            gin[grow + decompose(p.gr, j)] = out;
        }
    }
}

__global__ void __launch_bounds__(256) copy_view_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                                        GradPlan p) {
    const int64_t total = p.n_kept * p.n_red;
    for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
         t += int64_t(gridDim.x) * blockDim.x) {
        const int64_t i = t / p.n_red, j = t % p.n_red;
        const int64_t f = swz(p, p.x_offset + decompose(p.xk, i) + decompose(p.xr, j));
        const int64_t g = swizzle_stages(p.dswz_rank, p.dswz_bits, p.dswz_base, p.dswz_shift,
                                         p.g_offset + decompose(p.gk, i) + decompose(p.gr, j));
        if (f < 0 || f >= p.x_size || g < 0 || g >= p.g_size) {
            report_device_error(SW_ERR_INVALID);
            continue;
        }
        dst[g] = src[f];
    }
}

int copy_leaves(Leaves& l, int rank, const int64_t* shape, const int64_t* stride, int64_t& numel) {
    if (rank < 0 || rank > SW_MAX_LEAVES) return fail(SW_ERR_INVALID, "sw_reduce_backward_f32: leaf rank out of range");
    l.rank = rank;
    numel = 1;
    for (int d = 0; d < rank; ++d) {
        if (shape[d] < 0) return fail(SW_ERR_INVALID, "sw_reduce_backward_f32: negative extent");
        l.shape[d] = shape[d];
        l.stride[d] = stride[d];
        numel *= shape[d];
    }
    return SW_OK;
}

}  // namespace
}  // namespace sw

extern "C" int sw_reduce_backward_f32(const sw_reduce_plan* plan, const float* x, int64_t x_size,
                                      const float* grad_out, float* grad_in, const sw_reduce_plan* grad_plan,
                                      int64_t grad_size, void* stream) {
    using namespace sw;
    if (!plan || !grad_plan || !grad_out || !grad_in)
        return fail(SW_ERR_INVALID, "sw_reduce_backward_f32: null argument");
    if (plan->kind != SW_REDUCE_SUM && plan->kind != SW_REDUCE_MAX)
        return fail(SW_ERR_INVALID, "sw_reduce_backward_f32: only reduce_sum and reduce_max have a gradient");
    if (plan->kind == SW_REDUCE_MAX && !x) return fail(SW_ERR_INVALID, "sw_reduce_backward_f32: max needs x");
    GradPlan p;
    std::memset(&p, 0, sizeof(p));
    p.kind = plan->kind;
    int64_t nk, nr, gnk, gnr;
    int rc;
    if ((rc = copy_leaves(p.xk, plan->kept_rank, plan->kept_shape, plan->kept_stride, nk)) != SW_OK) return rc;
    if ((rc = copy_leaves(p.xr, plan->reduced_rank, plan->reduced_shape, plan->reduced_stride, nr)) != SW_OK) return rc;
    if ((rc = copy_leaves(p.gk, grad_plan->kept_rank, grad_plan->kept_shape, grad_plan->kept_stride, gnk)) != SW_OK)
        return rc;
    if ((rc = copy_leaves(p.gr, grad_plan->reduced_rank, grad_plan->reduced_shape, grad_plan->reduced_stride, gnr)) !=
        SW_OK)
        return rc;
    if (nk != gnk || nr != gnr) return fail(SW_ERR_INVALID, "sw_reduce_backward_f32: gradient shape mismatch");
    p.n_kept = nk;
    p.n_red = nr;
    p.x_offset = plan->offset;
    p.x_size = x_size;
    p.g_offset = grad_plan->offset;
    p.g_size = grad_size;
    p.swz_rank = plan->swizzle_rank;
    if (p.swz_rank < 0 || p.swz_rank > SW_MAX_SWIZZLE) return fail(SW_ERR_INVALID, "sw_reduce_backward_f32: swizzle rank");
    for (int s = 0; s < p.swz_rank; ++s) {
        p.swz_bits[s] = plan->swizzle_bits[s];
        p.swz_base[s] = plan->swizzle_base[s];
        p.swz_shift[s] = plan->swizzle_shift[s];
    }
    // every gradient address must lie inside grad_in
    int64_t lo = p.g_offset, hi = p.g_offset;
    for (const Leaves* l : {&p.gk, &p.gr})
        for (int d = 0; d < l->rank; ++d) {
            const int64_t span = (l->shape[d] - 1) * l->stride[d];
            if (l->shape[d] == 0) continue;
            if (span < 0) lo += span; else hi += span;
        }
    if (nk > 0 && nr > 0 && (lo < 0 || hi >= grad_size))
        return fail(SW_ERR_INVALID, "sw_reduce_backward_f32: gradient placement outside its carrier");
    if (nk == 0 || nr == 0) return ok();
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t blocks = std::min<int64_t>((nk + 7) / 8, int64_t(sms) * 8);
    reduce_grad_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(x, grad_out, grad_in, p);
    SW_LAUNCH_CHECK("sw_reduce_backward_f32 launch");
    return ok();
}

extern "C" int sw_copy_view_f32(const sw_reduce_plan* src_plan, const float* src, int64_t src_size,
                                const sw_reduce_plan* dst_plan, float* dst, int64_t dst_size, void* stream) {
    using namespace sw;
    if (!src_plan || !dst_plan || !src || !dst) return fail(SW_ERR_INVALID, "sw_copy_view_f32: null argument");
    GradPlan p;
    std::memset(&p, 0, sizeof(p));
    int64_t nk, nr, gnk, gnr;
    int rc;
    if ((rc = copy_leaves(p.xk, src_plan->kept_rank, src_plan->kept_shape, src_plan->kept_stride, nk)) != SW_OK)
        return rc;
    if ((rc = copy_leaves(p.xr, src_plan->reduced_rank, src_plan->reduced_shape, src_plan->reduced_stride, nr)) !=
        SW_OK)
        return rc;
    if ((rc = copy_leaves(p.gk, dst_plan->kept_rank, dst_plan->kept_shape, dst_plan->kept_stride, gnk)) != SW_OK)
        return rc;
    if ((rc = copy_leaves(p.gr, dst_plan->reduced_rank, dst_plan->reduced_shape, dst_plan->reduced_stride, gnr)) !=
        SW_OK)
        return rc;
    if (nk != gnk || nr != gnr) return fail(SW_ERR_INVALID, "sw_copy_view_f32: mode sizes differ");
    p.n_kept = nk;
    p.n_red = nr;
    p.x_offset = src_plan->offset;
    p.x_size = src_size;
    p.g_offset = dst_plan->offset;
    p.g_size = dst_size;
    p.swz_rank = src_plan->swizzle_rank;
    if (p.swz_rank < 0 || p.swz_rank > SW_MAX_SWIZZLE) return fail(SW_ERR_INVALID, "sw_copy_view_f32: swizzle rank");
    for (int s = 0; s < p.swz_rank; ++s) {
        p.swz_bits[s] = src_plan->swizzle_bits[s];
        p.swz_base[s] = src_plan->swizzle_base[s];
        p.swz_shift[s] = src_plan->swizzle_shift[s];
    }
    p.dswz_rank = dst_plan->swizzle_rank;
    if (p.dswz_rank < 0 || p.dswz_rank > SW_MAX_SWIZZLE)
        return fail(SW_ERR_INVALID, "sw_copy_view_f32: destination swizzle rank");
    for (int s = 0; s < p.dswz_rank; ++s) {
        p.dswz_bits[s] = dst_plan->swizzle_bits[s];
        p.dswz_base[s] = dst_plan->swizzle_base[s];
        p.dswz_shift[s] = dst_plan->swizzle_shift[s];
    }
    for (const sw_reduce_plan* q : {src_plan, dst_plan})
        for (int s = 0; s < q->swizzle_rank; ++s)  // the constraints of SwizzleStage (core/swizzle.py:44-60)
            if (q->swizzle_bits[s] <= 0 || q->swizzle_base[s] < 0 || q->swizzle_shift[s] == 0 ||
                std::abs(q->swizzle_shift[s]) < q->swizzle_bits[s] ||
                q->swizzle_bits[s] + q->swizzle_base[s] + std::abs(q->swizzle_shift[s]) > 62)
                return fail(SW_ERR_INVALID, "sw_copy_view_f32: invalid swizzle stage %d", s);
    if (nk == 0 || nr == 0) return ok();
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t blocks = std::min<int64_t>((nk * nr + 255) / 256, int64_t(sms) * 16);
    copy_view_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(src, dst, p);
    SW_LAUNCH_CHECK("sw_copy_view_f32 launch");
    return ok();
}
