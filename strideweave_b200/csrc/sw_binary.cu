// sw_binary.cu - strided binary elementwise Float32 maps.
//
// out[o(i)] = a[a(i)] (op) b[b(i)] for every logical index i of a view whose
// leaves (first leaf fastest) the three operands share, each with its own
// strides (0 on a broadcast leaf) and offset.  This is the reference's binary
// elementwise walk (cpu_binary_elementwise_forward,
// src/strideweave/carriers/cpu/native/_cpu_binary.hpp:85-130: one shared key
// over the aligned operands' leaves) as one grid-stride kernel.
#include <algorithm>
#include <cstdlib>
#include <utility>

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

// Row walk of a normalised plan (leaves sorted by output stride, contiguous
// leaves merged): leaf 0 is the row, the other leaves number the rows.  A CTA
// takes kRowsPer rows at a time (grid-stride over row groups), decomposing
// each row index once, and its threads walk the rows together, so every
// thread keeps kRowsPer loads in flight.  With kVec the walk moves four
// elements at a time as 16-byte vectors (leaf 0 unit-stride in a and out,
// unit or zero stride in b, row length a multiple of 4, every row start
// 16-byte aligned).
constexpr int kRowsPer = 4;

template <int OP, bool kVec>
__global__ void __launch_bounds__(256) map_rows_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                                       float* __restrict__ out, BinaryPlan p, int64_t rows, float s) {
    constexpr bool kUnary = OP == SW_MAP_SCALE || OP == SW_MAP_POW;
    const int64_t n0 = p.shape[0];
    for (int64_t row0 = int64_t(blockIdx.y) * kRowsPer; row0 < rows; row0 += int64_t(gridDim.y) * kRowsPer) {
        int64_t fa[kRowsPer], fb[kRowsPer], fo[kRowsPer];
        bool live[kRowsPer];
#pragma unroll
        for (int u = 0; u < kRowsPer; ++u) {
            live[u] = row0 + u < rows;
            int64_t t = live[u] ? row0 + u : 0;
            fa[u] = p.oa;
            fb[u] = p.ob;
            fo[u] = p.oo;
            for (int d = 1; d < p.rank; ++d) {
                const int64_t c = t % p.shape[d];
                t /= p.shape[d];
                fa[u] += c * p.sa[d];
                fb[u] += c * p.sb[d];
                fo[u] += c * p.so[d];
            }
        }
        if (kVec) {
            const int64_t nv = n0 >> 2;
            for (int64_t v = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; v < nv;
                 v += int64_t(gridDim.x) * blockDim.x) {
                float4 x[kRowsPer], y[kRowsPer];
#pragma unroll
                for (int u = 0; u < kRowsPer; ++u) {
                    if (!live[u]) continue;
                    x[u] = *reinterpret_cast<const float4*>(a + fa[u] + 4 * v);
                    if (kUnary) {
                        y[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                    } else if (p.sb[0] == 0) {
                        const float bb = b[fb[u]];
                        y[u] = make_float4(bb, bb, bb, bb);
                    } else {
                        y[u] = *reinterpret_cast<const float4*>(b + fb[u] + 4 * v);
                    }
                }
#pragma unroll
                for (int u = 0; u < kRowsPer; ++u) {
                    if (!live[u]) continue;
                    float4 r;
                    r.x = apply<OP>(x[u].x, y[u].x, s);
                    r.y = apply<OP>(x[u].y, y[u].y, s);
                    r.z = apply<OP>(x[u].z, y[u].z, s);
                    r.w = apply<OP>(x[u].w, y[u].w, s);
                    *reinterpret_cast<float4*>(out + fo[u] + 4 * v) = r;
                }
            }
        } else {
            for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n0;
                 i += int64_t(gridDim.x) * blockDim.x) {
                float x[kRowsPer], y[kRowsPer];
#pragma unroll
                for (int u = 0; u < kRowsPer; ++u) {
                    if (!live[u]) continue;
                    x[u] = a[fa[u] + i * p.sa[0]];
                    y[u] = kUnary ? 0.0f : b[fb[u] + i * p.sb[0]];
                }
#pragma unroll
                for (int u = 0; u < kRowsPer; ++u)
                    if (live[u]) out[fo[u] + i * p.so[0]] = apply<OP>(x[u], y[u], s);
            }
        }
    }
}

// Drops unit leaves, orders the rest by output stride (then a's), and merges
// a leaf into the one below it where every operand continues contiguously.
// The map is elementwise over a shared index space, so any leaf order gives
// the same results; this one makes consecutive threads write consecutive
// addresses.
void normalise(BinaryPlan& p) {
    int r = 0;
    for (int d = 0; d < p.rank; ++d) {
        if (p.shape[d] == 1) continue;
        p.shape[r] = p.shape[d];
        p.sa[r] = p.sa[d];
        p.sb[r] = p.sb[d];
        p.so[r] = p.so[d];
        ++r;
    }
    p.rank = r;
    for (int i = 1; i < p.rank; ++i)  // insertion sort, stable
        for (int j = i; j > 0; --j) {
            const auto key = [&](int k) { return std::make_pair(std::llabs(p.so[k]), std::llabs(p.sa[k])); };
            if (!(key(j) < key(j - 1))) break;
            std::swap(p.shape[j], p.shape[j - 1]);
            std::swap(p.sa[j], p.sa[j - 1]);
            std::swap(p.sb[j], p.sb[j - 1]);
            std::swap(p.so[j], p.so[j - 1]);
        }
    int m = 0;
    for (int d = 1; d < p.rank; ++d) {
        if (p.sa[d] == p.sa[m] * p.shape[m] && p.sb[d] == p.sb[m] * p.shape[m] &&
            p.so[d] == p.so[m] * p.shape[m]) {
            p.shape[m] *= p.shape[d];
            continue;
        }
        ++m;
        p.shape[m] = p.shape[d];
        p.sa[m] = p.sa[d];
        p.sb[m] = p.sb[d];
        p.so[m] = p.so[d];
    }
    if (p.rank > 0) p.rank = m + 1;
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
    cudaStream_t s = (cudaStream_t)stream;
    normalise(p);
    if (p.rank >= 1 && p.shape[0] >= 256) {
        // rows of at least one CTA's width: the row walk
        const int64_t rows = p.n / p.shape[0];
        const bool b_ok = unary || p.sb[0] == 1 || p.sb[0] == 0;
        bool vec = p.sa[0] == 1 && p.so[0] == 1 && b_ok && p.shape[0] % 4 == 0;
        if (vec) {  // every row start 16-byte aligned
            const auto aligned = [&](const float* base, int64_t off, const int64_t* st, bool check) {
                if (!check) return true;
                if ((reinterpret_cast<uintptr_t>(base + off) & 15) != 0) return false;
                for (int d = 1; d < p.rank; ++d)
                    if (st[d] % 4 != 0) return false;
                return true;
            };
            vec = aligned(a, p.oa, p.sa, true) && aligned(out, p.oo, p.so, true) &&
                  aligned(b, p.ob, p.sb, !unary && p.sb[0] == 1);
        }
        const int64_t per_row = vec ? p.shape[0] / 4 : p.shape[0];
        const int64_t bx = std::min<int64_t>((per_row + 255) / 256, int64_t(sms) * 8);
        const int64_t groups = (rows + kRowsPer - 1) / kRowsPer;
        const int64_t by = std::min<int64_t>({groups, std::max<int64_t>(1, int64_t(sms) * 8 / bx), 65535});
        const dim3 grid((unsigned)bx, (unsigned)by);
#define SW_MAP_ROWS(OPV)                                                                            \
    (vec ? map_rows_kernel<OPV, true><<<grid, 256, 0, s>>>(a, unary ? a : b, out, p, rows, scalar) \
         : map_rows_kernel<OPV, false><<<grid, 256, 0, s>>>(a, unary ? a : b, out, p, rows, scalar))
        switch (op) {
            case SW_MAP_ADD: SW_MAP_ROWS(SW_MAP_ADD); break;
            case SW_MAP_SUB: SW_MAP_ROWS(SW_MAP_SUB); break;
            case SW_MAP_MUL: SW_MAP_ROWS(SW_MAP_MUL); break;
            case SW_MAP_SCALE: SW_MAP_ROWS(SW_MAP_SCALE); break;
            case SW_MAP_POW: SW_MAP_ROWS(SW_MAP_POW); break;
            default: SW_MAP_ROWS(SW_MAP_POW_GRAD); break;
        }
#undef SW_MAP_ROWS
        SW_LAUNCH_CHECK("elementwise view map launch");
        return ok();
    }
    const unsigned blocks = (unsigned)std::min<int64_t>((p.n + 255) / 256, int64_t(sms) * 8);
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
