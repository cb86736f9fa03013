// sw_binary.cu - strided binary elementwise Float32 maps.
//
// out[o(i)] = a[a(i)] (op) b[b(i)] for every logical index i of a view whose
// leaves (first leaf fastest) the three operands share, each with its own
// strides (0 on a broadcast leaf) and offset.  This is the reference's binary
// elementwise walk (cpu_binary_elementwise_forward,
// src/strideweave/carriers/cpu/native/_cpu_binary.hpp:85-130: one shared key
// over the aligned operands' leaves) as one grid-stride kernel.
#include <algorithm>

#include "sw_common.cuh"

namespace sw {
namespace {

constexpr int kMaxBinaryLeaves = 16;

struct BinaryPlan {
    int rank;
    int64_t n;
    int64_t shape[kMaxBinaryLeaves];
    int64_t sa[kMaxBinaryLeaves], sb[kMaxBinaryLeaves], so[kMaxBinaryLeaves];
    int64_t oa, ob, oo;
};

// x^p as the reference's std::pow(float, float): the squares of an MSE loss
// (p = 2) and p = 1 are the correctly rounded products; other exponents go
// through the device powf.
__device__ __forceinline__ float pow_f32(float x, float p) {
    if (p == 2.0f) return __fmul_rn(x, x);
    if (p == 1.0f) return x;
    return powf(x, p);
}

template <int OP>
__device__ __forceinline__ float apply(float x, float y, float s) {
    if (OP == SW_MAP_ADD) return __fadd_rn(x, y);
    if (OP == SW_MAP_SUB) return __fsub_rn(x, y);
    if (OP == SW_MAP_MUL) return __fmul_rn(x, y);
    if (OP == SW_MAP_SCALE) return __fmul_rn(x, s);
    if (OP == SW_MAP_POW) return pow_f32(x, s);
    // SW_MAP_POW_GRAD: the reference's g * p * std::pow(x, p - 1), left to right
    return __fmul_rn(__fmul_rn(x, s), pow_f32(y, s - 1.0f));
}

template <int OP>
__global__ void __launch_bounds__(256) binary_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                                     float* __restrict__ out, BinaryPlan p, float s) {
    constexpr bool kUnary = OP == SW_MAP_SCALE || OP == SW_MAP_POW;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < p.n; i += int64_t(gridDim.x) * blockDim.x) {
        int64_t t = i, fa = p.oa, fb = p.ob, fo = p.oo;
        for (int d = 0; d < p.rank; ++d) {
            const int64_t c = t % p.shape[d];
            t /= p.shape[d];
            fa += c * p.sa[d];
            fb += c * p.sb[d];
            fo += c * p.so[d];
        }
        out[fo] = apply<OP>(a[fa], kUnary ? 0.0f : b[fb], s);
    }
}

// [lo, hi] of the addresses a view reaches.
void span_of(const BinaryPlan& p, const int64_t* stride, int64_t offset, int64_t& lo, int64_t& hi) {
    lo = hi = offset;
    for (int d = 0; d < p.rank; ++d) {
        const int64_t reach = (p.shape[d] - 1) * stride[d];
        if (reach < 0) lo += reach;
        else hi += reach;
    }
}

}  // namespace
}  // namespace sw

namespace sw {
namespace {

int map_impl(const char* who, int op, int rank, const int64_t* shape, const float* a, int64_t a_offset,
             const int64_t* a_stride, int64_t a_size, const float* b, int64_t b_offset, const int64_t* b_stride,
             int64_t b_size, float* out, int64_t out_offset, const int64_t* out_stride, int64_t out_size, float scalar,
             void* stream) {
    if (op < SW_MAP_ADD || op > SW_MAP_POW_GRAD) return fail(SW_ERR_INVALID, "%s: unknown op %d", who, op);
    const bool unary = op == SW_MAP_SCALE || op == SW_MAP_POW;
    if (rank < 0 || rank > kMaxBinaryLeaves)
        return fail(SW_ERR_UNSUPPORTED, "%s: %d leaves (at most %d)", who, rank, kMaxBinaryLeaves);
    if (rank > 0 && (!shape || !a_stride || !out_stride || (!unary && !b_stride)))
        return fail(SW_ERR_INVALID, "%s: null shape or stride array", who);
    BinaryPlan p;
    p.rank = rank;
    p.n = 1;
    for (int d = 0; d < rank; ++d) {
        if (shape[d] < 0) return fail(SW_ERR_INVALID, "%s: negative extent", who);
        p.shape[d] = shape[d];
        p.sa[d] = a_stride[d];
        p.sb[d] = unary ? 0 : b_stride[d];
        p.so[d] = out_stride[d];
        p.n *= shape[d];
    }
    if (p.n == 0) return ok();
    if (!a || (!unary && !b) || !out) return fail(SW_ERR_INVALID, "%s: null pointer", who);
    p.oa = a_offset;
    p.ob = unary ? 0 : b_offset;
    p.oo = out_offset;
    int64_t lo, hi;
    span_of(p, p.sa, p.oa, lo, hi);
    if (lo < 0 || hi >= a_size) return fail(SW_ERR_INVALID, "%s: lhs view outside its carrier", who);
    if (!unary) {
        span_of(p, p.sb, p.ob, lo, hi);
        if (lo < 0 || hi >= b_size) return fail(SW_ERR_INVALID, "%s: rhs view outside its carrier", who);
    }
    span_of(p, p.so, p.oo, lo, hi);
    if (lo < 0 || hi >= out_size) return fail(SW_ERR_INVALID, "%s: output view outside its carrier", who);
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const unsigned blocks = (unsigned)std::min<int64_t>((p.n + 255) / 256, int64_t(sms) * 8);
    cudaStream_t s = (cudaStream_t)stream;
    switch (op) {
        case SW_MAP_ADD: binary_kernel<SW_MAP_ADD><<<blocks, 256, 0, s>>>(a, b, out, p, scalar); break;
        case SW_MAP_SUB: binary_kernel<SW_MAP_SUB><<<blocks, 256, 0, s>>>(a, b, out, p, scalar); break;
        case SW_MAP_MUL: binary_kernel<SW_MAP_MUL><<<blocks, 256, 0, s>>>(a, b, out, p, scalar); break;
        case SW_MAP_SCALE: binary_kernel<SW_MAP_SCALE><<<blocks, 256, 0, s>>>(a, a, out, p, scalar); break;
        case SW_MAP_POW: binary_kernel<SW_MAP_POW><<<blocks, 256, 0, s>>>(a, a, out, p, scalar); break;
        default: binary_kernel<SW_MAP_POW_GRAD><<<blocks, 256, 0, s>>>(a, b, out, p, scalar); break;
    }
    SW_LAUNCH_CHECK("elementwise view map launch");
    return ok();
}

}  // namespace
}  // namespace sw

extern "C" int sw_binary_f32(int op, int rank, const int64_t* shape, const float* a, int64_t a_offset,
                             const int64_t* a_stride, int64_t a_size, const float* b, int64_t b_offset,
                             const int64_t* b_stride, int64_t b_size, float* out, int64_t out_offset,
                             const int64_t* out_stride, int64_t out_size, void* stream) {
    if (op != SW_BIN_MUL) return sw::fail(SW_ERR_INVALID, "sw_binary_f32: unknown op %d", op);
    return sw::map_impl("sw_binary_f32", SW_MAP_MUL, rank, shape, a, a_offset, a_stride, a_size, b, b_offset,
                        b_stride, b_size, out, out_offset, out_stride, out_size, 0.0f, stream);
}

extern "C" int sw_map_f32(int op, int rank, const int64_t* shape, const float* a, int64_t a_offset,
                          const int64_t* a_stride, int64_t a_size, const float* b, int64_t b_offset,
                          const int64_t* b_stride, int64_t b_size, float* out, int64_t out_offset,
                          const int64_t* out_stride, int64_t out_size, float scalar, void* stream) {
    return sw::map_impl("sw_map_f32", op, rank, shape, a, a_offset, a_stride, a_size, b, b_offset, b_stride, b_size,
                        out, out_offset, out_stride, out_size, scalar, stream);
}
