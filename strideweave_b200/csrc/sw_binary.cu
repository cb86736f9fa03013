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

template <int OP>
__global__ void __launch_bounds__(256) binary_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                                     float* __restrict__ out, BinaryPlan p) {
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < p.n; i += int64_t(gridDim.x) * blockDim.x) {
        int64_t t = i, fa = p.oa, fb = p.ob, fo = p.oo;
        for (int d = 0; d < p.rank; ++d) {
            const int64_t c = t % p.shape[d];
            t /= p.shape[d];
            fa += c * p.sa[d];
            fb += c * p.sb[d];
            fo += c * p.so[d];
        }
        if (OP == SW_BIN_MUL) out[fo] = __fmul_rn(a[fa], b[fb]);
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

extern "C" int sw_binary_f32(int op, int rank, const int64_t* shape, const float* a, int64_t a_offset,
                             const int64_t* a_stride, int64_t a_size, const float* b, int64_t b_offset,
                             const int64_t* b_stride, int64_t b_size, float* out, int64_t out_offset,
                             const int64_t* out_stride, int64_t out_size, void* stream) {
    using namespace sw;
    if (op != SW_BIN_MUL) return fail(SW_ERR_INVALID, "sw_binary_f32: unknown op %d", op);
    if (rank < 0 || rank > kMaxBinaryLeaves)
        return fail(SW_ERR_UNSUPPORTED, "sw_binary_f32: %d leaves (at most %d)", rank, kMaxBinaryLeaves);
    BinaryPlan p;
    p.rank = rank;
    p.n = 1;
    for (int d = 0; d < rank; ++d) {
        if (shape[d] < 0) return fail(SW_ERR_INVALID, "sw_binary_f32: negative extent");
        p.shape[d] = shape[d];
        p.sa[d] = a_stride[d];
        p.sb[d] = b_stride[d];
        p.so[d] = out_stride[d];
        p.n *= shape[d];
    }
    if (p.n == 0) return ok();
    if (!a || !b || !out) return fail(SW_ERR_INVALID, "sw_binary_f32: null pointer");
    p.oa = a_offset;
    p.ob = b_offset;
    p.oo = out_offset;
    int64_t lo, hi;
    span_of(p, p.sa, p.oa, lo, hi);
    if (lo < 0 || hi >= a_size) return fail(SW_ERR_INVALID, "sw_binary_f32: lhs view outside its carrier");
    span_of(p, p.sb, p.ob, lo, hi);
    if (lo < 0 || hi >= b_size) return fail(SW_ERR_INVALID, "sw_binary_f32: rhs view outside its carrier");
    span_of(p, p.so, p.oo, lo, hi);
    if (lo < 0 || hi >= out_size) return fail(SW_ERR_INVALID, "sw_binary_f32: output view outside its carrier");
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t blocks = std::min<int64_t>((p.n + 255) / 256, int64_t(sms) * 8);
    binary_kernel<SW_BIN_MUL><<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(a, b, out, p);
    SW_LAUNCH_CHECK("sw_binary_f32 launch");
    return ok();
}
