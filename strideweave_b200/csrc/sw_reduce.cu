// sw_reduce.cu - layout-aware Float32 reductions (sum, max, argmax) over the
// second mode of a two-mode view, for any hierarchical strides and an optional
// carrier-level XOR swizzle.
//
// Semantics follow the reference CPU carrier exactly where it pins them:
//   max    (src/strideweave/carriers/cpu/native/_cpu_reduction.hpp:21-32): the
//          first NaN in logical order wins with its payload; two zeros of any
//          sign give +0; otherwise the larger value.  This rule is associative
//          and commutative once NaNs carry their ordinal, so a tree over any
//          partition of the fibre reproduces the sequential fold bit for bit.
//   argmax (_cpu_reduction.hpp:76-93): NaN beats every number, the first NaN
//          wins, otherwise the first ordinal holding the largest value
//          (-0 == +0).  Ordered by (is-NaN, value, -ordinal), so again any
//          tree order gives the sequential answer.
//   sum    (ops/reduce_sum.cpp:12-28): Float32 accumulation; the tree order
//          differs from the sequential one, within the path's tolerance.
//
// Kernels (chosen on the host from the lowered plan):
//   rows_vec  - the reduced mode has a unit-stride leaf: one warp per kept
//               ordinal streams 16-byte vectors along it.
//   cols_vec  - the kept mode has a unit-stride leaf: each thread owns four
//               adjacent kept ordinals; the fibre is split over the 8 warps
//               of a CTA and over the CTAs of a thread-block cluster, whose
//               partials meet in distributed shared memory (no scratch
//               memory, no second launch).
//   rows_affine - the reduced mode walks memory affinely per lane (one
//               unit-stride run, or equal runs at a fixed stride): one warp
//               per kept ordinal, pointer increments only, no index math.
//   cols_affine - the kept mode is unit-stride and the reduced mode is one
//               leaf: CTAs own 128 kept ordinals and a slice of the fibre;
//               slices meet in a small scratch buffer (at most SMs x 3 x 128
//               partials), folded by the last CTA of each column block.
//   cols_narrow - the same walk when there are kept ordinals enough for a
//               CTA of 32 per SM: each CTA reads 128-byte row pieces of the
//               whole fibre and folds in shared memory; no scratch memory.
//   gather   - anything else: one warp per kept ordinal, scalar loads.
#include <cooperative_groups.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <type_traits>
#include <vector>

#include "sw_common.cuh"

namespace cg = cooperative_groups;

namespace sw {
namespace {

struct LeafSet {
    int rank;
    int64_t shape[SW_MAX_LEAVES];
    int64_t stride[SW_MAX_LEAVES];
    int64_t weight[SW_MAX_LEAVES];  // logical ordinal weight (colexicographic)
};

struct Swz {
    int rank;
    int bits[SW_MAX_SWIZZLE];
    int base[SW_MAX_SWIZZLE];
    int shift[SW_MAX_SWIZZLE];
};

struct DevPlan {
    int64_t offset;
    int64_t x_size;
    int64_t n_kept;
    int64_t n_red;
    LeafSet kept;
    LeafSet red;
    Swz swz;
};

__device__ __forceinline__ int64_t swizzle(const Swz& s, int64_t r) {
#pragma unroll
    for (int i = 0; i < SW_MAX_SWIZZLE; ++i) {
        if (i < s.rank) {
            const int64_t mask = (int64_t(1) << s.bits[i]) - 1;
            if (s.shift[i] > 0) {
                r ^= ((r >> (s.base[i] + s.shift[i])) & mask) << s.base[i];
            } else {
                r ^= ((r >> s.base[i]) & mask) << (s.base[i] - s.shift[i]);
            }
        }
    }
    return r;
}

// Offset of kept ordinal i (decomposed first-leaf-fastest over the kept leaves
// in their logical order).
__device__ __forceinline__ int64_t kept_offset(const LeafSet& k, int64_t i) {
    int64_t off = 0;
    for (int l = 0; l < k.rank; ++l) {
        const int64_t c = i % k.shape[l];
        i /= k.shape[l];
        off += c * k.stride[l];
    }
    return off;
}

// ---- reduction states ------------------------------------------------------

enum class Kind { kSum, kMax, kArgmax };

struct SumOp {
    static constexpr Kind kKind = Kind::kSum;
    struct S { float v; };
    static __device__ __forceinline__ S identity() { return {0.0f}; }
    static __device__ __forceinline__ void add(S& s, float v, int64_t) { s.v += v; }
    static __device__ __forceinline__ void merge(S& a, const S& b) { a.v += b.v; }
    static __device__ __forceinline__ S shfl(const S& s, int lane_mask) {
        return {__shfl_xor_sync(0xffffffffu, s.v, lane_mask)};
    }
};

// reduce_sum with accumulator_dtype=Float64: Float32 elements summed in
// binary64, the result rounded once (_cpu_accumulation.hpp:38-41).  Only the
// general gather walk instantiates it.
struct SumOp64 {
    struct S { double v; };
    static __device__ __forceinline__ S identity() { return {0.0}; }
    static __device__ __forceinline__ void add(S& s, float v, int64_t) { s.v = __dadd_rn(s.v, double(v)); }
    static __device__ __forceinline__ void merge(S& a, const S& b) { a.v = __dadd_rn(a.v, b.v); }
    static __device__ __forceinline__ S shfl(const S& s, int lane_mask) {
        return {__shfl_xor_sync(0xffffffffu, s.v, lane_mask)};
    }
};

struct MaxOp {
    static constexpr Kind kKind = Kind::kMax;
    struct S { float v; int64_t j; };  // j only orders NaNs
    static __device__ __forceinline__ S identity() { return {-INFINITY, INT64_MAX}; }
    static __device__ __forceinline__ void add(S& s, float v, int64_t j) { merge(s, S{v, j}); }
    static __device__ __forceinline__ void merge(S& a, const S& b) {
        const bool na = isnan(a.v), nb = isnan(b.v);
        if (na || nb) {
            if (nb && (!na || b.j < a.j)) a = b;
            return;
        }
        if (a.v == b.v && a.v == 0.0f) {
            a.v = 0.0f;  // two zeros of any sign give +0
            return;
        }
        if (b.v > a.v) a = b;
    }
    static __device__ __forceinline__ S shfl(const S& s, int m) {
        return {__shfl_xor_sync(0xffffffffu, s.v, m),
                (int64_t)__shfl_xor_sync(0xffffffffu, (long long)s.j, m)};
    }
};

struct ArgmaxOp {
    static constexpr Kind kKind = Kind::kArgmax;
    struct S { float v; int64_t j; };
    static __device__ __forceinline__ S identity() { return {-INFINITY, INT64_MAX}; }
    static __device__ __forceinline__ void add(S& s, float v, int64_t j) { merge(s, S{v, j}); }
    static __device__ __forceinline__ void merge(S& a, const S& b) {
        const bool na = isnan(a.v), nb = isnan(b.v);
        bool take;
        if (na != nb) take = nb;
        else if (na) take = b.j < a.j;
        else take = b.v > a.v || (b.v == a.v && b.j < a.j);
        if (take) a = b;
    }
    static __device__ __forceinline__ S shfl(const S& s, int m) {
        return {__shfl_xor_sync(0xffffffffu, s.v, m),
                (int64_t)__shfl_xor_sync(0xffffffffu, (long long)s.j, m)};
    }
};

template <class Op>
__device__ __forceinline__ void store_result(void* out, int64_t i, const typename Op::S& s);

template <>
__device__ __forceinline__ void store_result<SumOp>(void* out, int64_t i, const SumOp::S& s) {
    static_cast<float*>(out)[i] = s.v;
}
template <>
__device__ __forceinline__ void store_result<SumOp64>(void* out, int64_t i, const SumOp64::S& s) {
    static_cast<float*>(out)[i] = __double2float_rn(s.v);
}
template <>
__device__ __forceinline__ void store_result<MaxOp>(void* out, int64_t i, const MaxOp::S& s) {
    static_cast<float*>(out)[i] = s.v;
}
template <>
__device__ __forceinline__ void store_result<ArgmaxOp>(void* out, int64_t i, const ArgmaxOp::S& s) {
    static_cast<int32_t*>(out)[i] = (int32_t)s.j;
}

template <class Op>
__device__ __forceinline__ typename Op::S warp_reduce(typename Op::S s) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) Op::merge(s, Op::shfl(s, m));
    return s;
}

__device__ __forceinline__ float4 load_stream4(const float* p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ float load_stream1(const float* p) {
    float v;
    asm volatile("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}

// Odometer over the reduced leaves 1..rank-1 (leaf 0 is walked separately).
struct OuterCursor {
    int64_t key[SW_MAX_LEAVES];
    int64_t off;   // flat offset contribution
    int64_t ord;   // logical ordinal contribution
};

__device__ __forceinline__ void cursor_set(OuterCursor& c, const LeafSet& r, int64_t o) {
    c.off = 0;
    c.ord = 0;
    for (int l = 1; l < r.rank; ++l) {
        c.key[l] = o % r.shape[l];
        o /= r.shape[l];
        c.off += c.key[l] * r.stride[l];
        c.ord += c.key[l] * r.weight[l];
    }
}

__device__ __forceinline__ void cursor_step(OuterCursor& c, const LeafSet& r) {
    for (int l = 1; l < r.rank; ++l) {
        c.key[l] += 1;
        c.off += r.stride[l];
        c.ord += r.weight[l];
        if (c.key[l] < r.shape[l]) return;
        c.off -= r.stride[l] * r.shape[l];
        c.ord -= r.weight[l] * r.shape[l];
        c.key[l] = 0;
    }
}

// ---- rows_vec ----------------------------------------------------------------
// Reduced leaf 0 has stride 1 and a length divisible by 4; every other stride,
// the offset and the swizzle keep 16-byte vectors intact (checked on the host).
template <class Op>
__global__ void __launch_bounds__(256) reduce_rows_vec(const float* __restrict__ x, DevPlan p, void* out) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    const int64_t nv0 = p.red.shape[0] >> 2;          // vectors per leaf-0 run
    const int64_t nvec = p.n_red >> 2;                // vectors per fibre
    constexpr int U = 8;
    for (int64_t i = warp; i < p.n_kept; i += nwarps) {
        const int64_t row = p.offset + kept_offset(p.kept, i);
        typename Op::S acc[4] = {Op::identity(), Op::identity(), Op::identity(), Op::identity()};
        int64_t q = lane;
        int64_t v0 = q % nv0;
        OuterCursor cur;
        cursor_set(cur, p.red, q / nv0);
        while (q < nvec) {
            float4 val[U];
            int64_t ord[U];
            bool live[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                live[u] = q < nvec;
                if (live[u]) {
                    const int64_t f = swizzle(p.swz, row + v0 * 4 + cur.off);
                    val[u] = load_stream4(x + f);
                    ord[u] = v0 * 4 * p.red.weight[0] + cur.ord;
                    q += 32;
                    v0 += 32;
                    while (v0 >= nv0) {
                        v0 -= nv0;
                        cursor_step(cur, p.red);
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (live[u]) {
                    const int64_t w = p.red.weight[0];
                    Op::add(acc[0], val[u].x, ord[u]);
                    Op::add(acc[1], val[u].y, ord[u] + w);
                    Op::add(acc[2], val[u].z, ord[u] + 2 * w);
                    Op::add(acc[3], val[u].w, ord[u] + 3 * w);
                }
            }
        }
        Op::merge(acc[0], acc[1]);
        Op::merge(acc[2], acc[3]);
        Op::merge(acc[0], acc[2]);
        typename Op::S r = warp_reduce<Op>(acc[0]);
        if (lane == 0) store_result<Op>(out, i, r);
    }
}

// ---- cols_vec ----------------------------------------------------------------
// Kept leaf 0 has stride 1 and a length divisible by 4.  Block = 256 threads:
// 32 lanes x 4 kept ordinals = 128 kept ordinals per CTA, 8 warps split the
// fibre; `gridDim.y` CTAs of one cluster split it further.
constexpr int kColsThreads = 256;
constexpr int kColsWarps = kColsThreads / 32;

template <class Op>
__global__ void __launch_bounds__(kColsThreads) reduce_cols_vec(const float* __restrict__ x, DevPlan p, void* out) {
    __shared__ typename Op::S part[kColsWarps][32][4];
    cg::cluster_group cluster = cg::this_cluster();
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int splits = (int)cluster.num_blocks();
    const int split = (int)cluster.block_rank();
    const int64_t kv = int64_t(blockIdx.x) * 32 + lane;     // kept vector index
    const int64_t nkv = p.n_kept >> 2;
    const bool live_col = kv < nkv;
    int64_t col = 0;
    if (live_col) col = p.offset + kept_offset(p.kept, kv * 4);
    typename Op::S acc[4] = {Op::identity(), Op::identity(), Op::identity(), Op::identity()};
    // Fibre slice of this (split, warp).
    const int64_t per = (p.n_red + splits - 1) / splits;
    const int64_t j0 = per * split;
    const int64_t j1 = min(p.n_red, j0 + per);
    if (live_col && j0 < j1) {
        // Reduced leaves walked as one odometer; this thread takes every
        // kColsWarps-th ordinal of its split.
        int64_t j = j0 + warp;
        int64_t key[SW_MAX_LEAVES];
        int64_t off = 0, ord = 0;
        {
            int64_t t = j;
            for (int l = 0; l < p.red.rank; ++l) {
                key[l] = t % p.red.shape[l];
                t /= p.red.shape[l];
                off += key[l] * p.red.stride[l];
                ord += key[l] * p.red.weight[l];
            }
        }
        constexpr int U = 4;
        while (j < j1) {
            float4 val[U];
            int64_t o[U];
            bool live[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                live[u] = j < j1;
                if (live[u]) {
                    val[u] = load_stream4(x + swizzle(p.swz, col + off));
                    o[u] = ord;
                    j += kColsWarps;
                    // advance the odometer by kColsWarps ordinals
                    for (int s = 0; s < kColsWarps; ++s) {
                        for (int l = 0; l < p.red.rank; ++l) {
                            key[l] += 1;
                            off += p.red.stride[l];
                            ord += p.red.weight[l];
                            if (key[l] < p.red.shape[l]) break;
                            off -= p.red.stride[l] * p.red.shape[l];
                            ord -= p.red.weight[l] * p.red.shape[l];
                            key[l] = 0;
                        }
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (live[u]) {
                    Op::add(acc[0], val[u].x, o[u]);
                    Op::add(acc[1], val[u].y, o[u]);
                    Op::add(acc[2], val[u].z, o[u]);
                    Op::add(acc[3], val[u].w, o[u]);
                }
            }
        }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) part[warp][lane][e] = acc[e];
    __syncthreads();
    // Fold the 8 warps into warp 0's slot.
    if (warp == 0) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            typename Op::S s = part[0][lane][e];
            for (int w = 1; w < kColsWarps; ++w) Op::merge(s, part[w][lane][e]);
            part[0][lane][e] = s;
        }
    }
    cluster.sync();
    // Rank 0 folds every CTA's partial through distributed shared memory.
    if (split == 0 && warp == 0 && live_col) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            typename Op::S s = part[0][lane][e];
            for (int r = 1; r < splits; ++r) {
                typename Op::S(*peer)[32][4] = cluster.map_shared_rank(part, r);
                Op::merge(s, peer[0][lane][e]);
            }
            store_result<Op>(out, kv * 4 + e, s);
        }
    }
    cluster.sync();  // peers keep their shared memory alive until rank 0 read it
}

// ---- affine walks -------------------------------------------------------------
// When a lane's (or a thread's) share of a fibre is an arithmetic progression
// of 16-byte vectors, step t reads start + t * delta.  When the carrier's
// swizzle only rewrites bits below the lowest set bit of delta, the swizzle
// commutes with the step and is applied once, to the start: the loop is a
// pointer increment and a load.  The loop runs a cheap fold that is exact
// whenever the lane saw only finite values (and, for max, a non-zero result);
// otherwise the lane walks its share again with the exact merge.  Lanes then
// combine with the exact merge, so results stay bit-exact.

__device__ __forceinline__ float max_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

// Fast fold of four independent component streams, each visited in
// increasing ordinal order.
template <class Op, class Ord>
struct FastFold {
    float v[4];
    Ord j[4];
    float nanp;  // max.NaN of every value seen (argmax): NaN iff a NaN was seen
    // j[e] holds the step index of the current winner; the ordinal is
    // rebuilt once, in component().
    __device__ __forceinline__ void init(const float4& q) {
        const float c[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            v[e] = c[e];
            j[e] = 0;
        }
        nanp = max_nan(max_nan(c[0], c[1]), max_nan(c[2], c[3]));
    }
    __device__ __forceinline__ void step(const float4& q, int t) {
        const float c[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            if (Op::kKind == Kind::kSum) {
                v[e] += c[e];
            } else if (Op::kKind == Kind::kMax) {
                v[e] = max_nan(v[e], c[e]);  // a NaN sticks and forces the exact walk
            } else if (c[e] > v[e]) {
                v[e] = c[e];
                j[e] = Ord(t);
            }
        }
        if (Op::kKind == Kind::kArgmax) nanp = max_nan(nanp, max_nan(max_nan(c[0], c[1]), max_nan(c[2], c[3])));
    }
    __device__ __forceinline__ bool needs_exact() const {
        if (Op::kKind == Kind::kSum) return false;
        if (Op::kKind == Kind::kArgmax) return isnan(nanp);
        bool bad = false;
#pragma unroll
        for (int e = 0; e < 4; ++e) bad |= isnan(v[e]) || v[e] == 0.0f;
        return bad;
    }
    __device__ __forceinline__ typename Op::S component(int e, Ord ord0, Ord dord, Ord w0) const {
        typename Op::S t;
        if constexpr (Op::kKind == Kind::kSum) {
            t.v = v[e];
        } else {
            t.v = v[e];
            t.j = Op::kKind == Kind::kMax ? INT64_MAX
                                          : int64_t(ord0) + int64_t(j[e]) * int64_t(dord) + int64_t(e) * int64_t(w0);
        }
        return t;
    }
};

template <bool kSwz>
__device__ __forceinline__ int64_t phys(const Swz& s, int64_t f) {
    if constexpr (kSwz) return swizzle(s, f);
    else return f;
}

// A progression of `iters` vectors: flat offset off0 + t*doff, first component
// ordinal ord0 + t*dord, components w0 ordinals apart.
template <class Ord>
struct LaneWalk {
    int64_t off0, doff;
    Ord ord0, dord, w0;
    int iters;
};

// Exact fold of a progression (used when the fast fold cannot vouch).
template <class Op, bool kSwz, class Ord>
__device__ __forceinline__ void exact_walk(const float* __restrict__ x, const Swz& swz, int64_t base,
                                        const LaneWalk<Ord>& w, typename Op::S (&acc)[4], bool columns) {
    for (int t = 0; t < w.iters; ++t) {
        const float4 q = load_stream4(x + phys<kSwz>(swz, base + w.off0 + int64_t(t) * w.doff));
        const int64_t o = int64_t(w.ord0) + int64_t(t) * int64_t(w.dord);
        const int64_t d = columns ? 0 : int64_t(w.w0);
        Op::add(acc[0], q.x, o);
        Op::add(acc[1], q.y, o + d);
        Op::add(acc[2], q.z, o + 2 * d);
        Op::add(acc[3], q.w, o + 3 * d);
    }
}

// Fast fold of a progression whose physical addresses are affine (the
// swizzle, if any, commutes with doff).  U loads in flight per batch.
template <class Op, class Ord, int U>
__device__ __forceinline__ bool fast_walk(const float* ptr, int64_t doff, int iters, FastFold<Op, Ord>& f) {
    if constexpr (Op::kKind == Kind::kArgmax) {
        // A batch of U vectors is folded per component with max.NaN first
        // (one instruction an element); only a component whose batch maximum
        // beats its running maximum - rare once the walk is under way - is
        // searched for the first step holding that maximum.  That is the
        // sequential rule (larger wins, the earlier of equal values stays,
        // -0 == +0); a NaN anywhere makes its batch maximum NaN, which never
        // compares greater and marks the walk for the exact re-walk.
        for (int t0 = 0; t0 < iters; t0 += U) {
            float4 val[U];
#pragma unroll
            for (int u = 0; u < U; ++u)
                val[u] = t0 + u < iters ? load_stream4(ptr + int64_t(t0 + u) * doff)
                                        : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
            if (t0 == 0) f.init(val[0]);
            float m[4] = {val[0].x, val[0].y, val[0].z, val[0].w};
#pragma unroll
            for (int u = 1; u < U; ++u) {
                m[0] = max_nan(m[0], val[u].x);
                m[1] = max_nan(m[1], val[u].y);
                m[2] = max_nan(m[2], val[u].z);
                m[3] = max_nan(m[3], val[u].w);
            }
            f.nanp = max_nan(f.nanp, max_nan(max_nan(m[0], m[1]), max_nan(m[2], m[3])));
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if (m[e] > f.v[e]) {
                    int first = U - 1;
#pragma unroll
                    for (int u = U - 1; u >= 0; --u) {
                        const float c = e == 0 ? val[u].x : e == 1 ? val[u].y : e == 2 ? val[u].z : val[u].w;
                        if (c == m[e]) first = u;
                    }
                    f.v[e] = m[e];
                    f.j[e] = Ord(t0 + first);
                }
            }
        }
        return !f.needs_exact();
    }
    for (int t0 = 0; t0 < iters; t0 += U) {
        float4 val[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (t0 + u < iters) val[u] = load_stream4(ptr + int64_t(t0 + u) * doff);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (t0 + u < iters) {
                if (t0 + u == 0) f.init(val[u]);
                else f.step(val[u], t0 + u);
            }
        }
    }
    return !f.needs_exact();
}

// Row walk shared by all lanes: the reduced mode is a unit-stride run of
// `run` elements (run % 4 == 0) repeated `nruns` times at stride `rstride`
// (ordinal weight `rweight`); leaf ordinal weight of the run is `w0`.
struct RowWalk {
    int64_t run, nruns, rstride, rweight, w0;
};

constexpr int kRowsAffThreads = 256;
constexpr int kRowsAffWarps = kRowsAffThreads / 32;

// One warp reduces whole rows: warp w owns the contiguous kept ordinals
// [w * rpw, (w + 1) * rpw).  The host sizes the grid so that every warp is
// resident at once and all carry the same number of rows: no tail wave.
// Loads in flight per lane (and the resident CTAs per SM the kernel is
// compiled for) of the row walk, per operation.  Argmax, whose fold issues
// more instructions per element, holds eight 16-byte loads per lane at four
// CTAs per SM (measured, tiled + swizzled / row-major: 5.47 / 5.74 TB/s,
// against 5.27 / 5.65 with four loads; 4.92 / 5.42 with eight loads at three
// CTAs per SM; 5.16 / 5.42 with six).
#ifndef SW_ROWS_U_ARGMAX
#define SW_ROWS_U_ARGMAX 8
#endif
#ifndef SW_ROWS_MINB_ARGMAX
#define SW_ROWS_MINB_ARGMAX 4
#endif
template <class Op>
struct RowsWalkCfg { static constexpr int kU = 4, kMinBlocks = 4; };
template <>
struct RowsWalkCfg<ArgmaxOp> { static constexpr int kU = SW_ROWS_U_ARGMAX, kMinBlocks = SW_ROWS_MINB_ARGMAX; };

template <class Op, bool kSwz, class Ord>
__global__ void __launch_bounds__(kRowsAffThreads, RowsWalkCfg<Op>::kMinBlocks) reduce_rows_affine(const float* __restrict__ x, DevPlan p,
                                                                         RowWalk rw, int64_t rpw, void* out) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nv0 = rw.run >> 2;
    LaneWalk<Ord> w;
    w.w0 = Ord(rw.w0);
    if (nv0 >= 32) {  // one run, 32 vectors per step
        w.off0 = int64_t(lane) * 4;
        w.ord0 = Ord(lane * 4) * w.w0;
        w.doff = 128;
        w.dord = Ord(128) * w.w0;
        w.iters = int(nv0 / 32);
    } else {  // 32 / nv0 runs per step
        const int64_t per = 32 / nv0;
        w.off0 = (lane % nv0) * 4 + (lane / nv0) * rw.rstride;
        w.ord0 = Ord((lane % nv0) * 4 * rw.w0 + (lane / nv0) * rw.rweight);
        w.doff = per * rw.rstride;
        w.dord = Ord(per * rw.rweight);
        w.iters = int(rw.nruns / per);
    }
    const int64_t r0 = warp * rpw;
    const int64_t r1 = min(p.n_kept, r0 + rpw);
    for (int64_t i = r0; i < r1; ++i) {
        const int64_t row = p.offset + kept_offset(p.kept, i);
        typename Op::S r = Op::identity();
        FastFold<Op, Ord> f;
        const float* ptr = x + phys<kSwz>(p.swz, row + w.off0);
        if (fast_walk<Op, Ord, RowsWalkCfg<Op>::kU>(ptr, w.doff, w.iters, f)) {
#pragma unroll
            for (int e = 0; e < 4; ++e) Op::merge(r, f.component(e, w.ord0, w.dord, w.w0));
        } else {
            typename Op::S acc[4] = {Op::identity(), Op::identity(), Op::identity(), Op::identity()};
            exact_walk<Op, kSwz, Ord>(x, p.swz, row, w, acc, false);
#pragma unroll
            for (int e = 0; e < 4; ++e) Op::merge(r, acc[e]);
        }
        r = warp_reduce<Op>(r);
        if (lane == 0) store_result<Op>(out, i, r);
    }
}

constexpr int kColsAffThreads = 256;
constexpr int kColsAffWarps = kColsAffThreads / 32;
constexpr int64_t kMaxColSlices = 256;  // slices of a split column walk
constexpr int kColsAffPerSm = 3;        // resident CTAs per SM (80 registers a thread)
constexpr int kMaxClusterSlices = 8;    // slices that meet in one portable cluster

// Column walk: kept leaf 0 is unit-stride; the reduced mode is one leaf
// (extent n_red, stride `stride`, ordinal weight `weight`).  CTA (bx, by)
// owns 128 kept ordinals (32 lanes x 4) and slice `by` of the gridDim.y
// slices of the fibre; its 8 warps split the slice.  With more than one
// slice every CTA leaves its 128 partials in scratch memory ([slice][kept]),
// and the last CTA of the column block to finish folds them in slice order.
// A counter per column block says which CTA is last; that CTA puts it back
// to zero, so the counters are zero between launches.  No CTA waits for
// another: the early ones simply exit.
template <class Op>
__device__ __forceinline__ typename Op::S load_partial(const typename Op::S* p);
template <>
__device__ __forceinline__ SumOp::S load_partial<SumOp>(const SumOp::S* p) {
    return {__ldcg(&p->v)};
}
template <>
__device__ __forceinline__ MaxOp::S load_partial<MaxOp>(const MaxOp::S* p) {
    return {__ldcg(&p->v), (int64_t)__ldcg(reinterpret_cast<const long long*>(&p->j))};
}
template <>
__device__ __forceinline__ ArgmaxOp::S load_partial<ArgmaxOp>(const ArgmaxOp::S* p) {
    return {__ldcg(&p->v), (int64_t)__ldcg(reinterpret_cast<const long long*>(&p->j))};
}

// The column walk's partials, in shared memory and in scratch, in the
// narrowest form that holds them: on a 32-bit-ordinal walk, max and argmax
// keep their ordinal in 32 bits (8 bytes a partial instead of 16).  The
// identity's "no ordinal" INT64_MAX maps to INT32_MAX, which no 32-bit walk
// reaches (its ordinals stay below 2^30).
template <class Op, class Ord>
struct Packed {
    using T = typename Op::S;
    static __device__ __forceinline__ T pack(const typename Op::S& s) { return s; }
    static __device__ __forceinline__ typename Op::S unpack(const T& t) { return t; }
    static __device__ __forceinline__ T load(const T* p) { return load_partial<Op>(p); }
};
struct Packed8 {
    float v;
    int32_t j;
};
template <class Op>
struct PackedOrd32 {
    using T = Packed8;
    static __device__ __forceinline__ T pack(const typename Op::S& s) {
        return {s.v, s.j >= int64_t(INT32_MAX) ? INT32_MAX : int32_t(s.j)};
    }
    static __device__ __forceinline__ typename Op::S unpack(const T& t) {
        return {t.v, t.j == INT32_MAX ? INT64_MAX : int64_t(t.j)};
    }
    static __device__ __forceinline__ T load(const T* p) {
        const unsigned long long bits = __ldcg(reinterpret_cast<const unsigned long long*>(p));
        return T{__uint_as_float(uint32_t(bits)), int32_t(uint32_t(bits >> 32))};
    }
};
template <>
struct Packed<MaxOp, int32_t> : PackedOrd32<MaxOp> {};
template <>
struct Packed<ArgmaxOp, int32_t> : PackedOrd32<ArgmaxOp> {};

// kCluster: the slices of a column block are the CTAs of one thread-block
// cluster (gridDim.y = cluster size, at most 8) and meet in distributed shared
// memory; otherwise they leave partials in scratch and the last CTA of the
// column block (an atomic ticket) folds them.
template <class Op, bool kSwz, class Ord, bool kCluster>
__global__ void __launch_bounds__(kColsAffThreads, kColsAffPerSm) reduce_cols_affine(const float* __restrict__ x, DevPlan p,
                                                                         int64_t stride, int64_t weight, void* out,
                                                                         typename Packed<Op, Ord>::T* partials,
                                                                         unsigned* counters) {
    using P = Packed<Op, Ord>;
    __shared__ typename P::T part[kColsAffWarps][32][4];
    __shared__ unsigned s_last;
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int splits = (int)gridDim.y;
    const int split = (int)blockIdx.y;
    const int64_t kv = int64_t(blockIdx.x) * 32 + lane;
    const bool live_col = kv < (p.n_kept >> 2);
    const int64_t col = live_col ? p.offset + kept_offset(p.kept, kv * 4) : 0;
    const int64_t per = (p.n_red + splits - 1) / splits;
    const int64_t j0 = per * split + warp;
    const int64_t j1 = min(p.n_red, per * (split + 1));
    typename Op::S acc[4] = {Op::identity(), Op::identity(), Op::identity(), Op::identity()};
    if (live_col && j0 < j1) {
        LaneWalk<Ord> w;
        w.off0 = j0 * stride;
        w.doff = int64_t(kColsAffWarps) * stride;
        w.ord0 = Ord(j0 * weight);
        w.dord = Ord(kColsAffWarps * weight);
        w.w0 = 0;  // the four components are four columns at the same ordinal
        w.iters = int((j1 - j0 + kColsAffWarps - 1) / kColsAffWarps);
        FastFold<Op, Ord> f;
        const float* ptr = x + phys<kSwz>(p.swz, col + w.off0);
        // eight 16-byte loads in flight per lane (argmax included: the
        // 80-register budget of three CTAs per SM holds its ordinals)
        constexpr int kU = 8;
        if (fast_walk<Op, Ord, kU>(ptr, w.doff, w.iters, f)) {
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[e] = f.component(e, w.ord0, w.dord, Ord(0));
        } else {
            exact_walk<Op, kSwz, Ord>(x, p.swz, col, w, acc, true);
        }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) part[warp][lane][e] = P::pack(acc[e]);
    __syncthreads();
    // warps 0..3 fold component `warp` (kept ordinal kv*4 + warp) of the 8 warps' partials
    typename Op::S v = Op::identity();
    const int64_t kept_i = kv * 4 + warp;
    if (warp < 4) {
        v = P::unpack(part[0][lane][warp]);
#pragma unroll
        for (int w = 1; w < kColsAffWarps; ++w) Op::merge(v, P::unpack(part[w][lane][warp]));
    }
    if (splits == 1) {
        if (warp < 4 && live_col) store_result<Op>(out, kept_i, v);
        return;
    }
    if constexpr (kCluster) {
        // slice `split` is cluster rank `split` (cluster dims 1 x splits);
        // rank 0 folds the slices in order, reading its peers' shared memory
        cg::cluster_group cluster = cg::this_cluster();
        if (warp < 4) part[0][lane][warp] = P::pack(v);  // only this thread read that slot
        cluster.sync();
        if (split == 0 && warp < 4 && live_col) {
            typename Op::S r = P::unpack(part[0][lane][warp]);
            for (int q = 1; q < splits; ++q) {
                const typename P::T* peer = cluster.map_shared_rank(&part[0][0][0], q);
                Op::merge(r, P::unpack(peer[lane * 4 + warp]));
            }
            store_result<Op>(out, kept_i, r);
        }
        cluster.sync();  // the peers' shared memory stays alive until rank 0 has read it
        return;
    }
    if (warp < 4 && live_col) partials[int64_t(split) * p.n_kept + kept_i] = P::pack(v);
    __threadfence();  // this CTA's partials are visible before its ticket is
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&counters[blockIdx.x], 1u) == unsigned(splits - 1) ? 1u : 0u;
    __syncthreads();
    if (!s_last) return;
    __threadfence();  // every other slice's partials are visible from here on
    if (warp < 4 && live_col) {
        // a batch of independent loads in flight before each round of merges:
        // the usual slice counts (about SMs x 4 / column blocks) take one round trip
        constexpr int kB = sizeof(typename P::T) > 4 ? 10 : 16;
        typename Op::S r = Op::identity();
        for (int s0 = 0; s0 < splits; s0 += kB) {
            typename P::T q[kB];
#pragma unroll
            for (int u = 0; u < kB; ++u)
                if (s0 + u < splits) q[u] = P::load(partials + int64_t(s0 + u) * p.n_kept + kept_i);
#pragma unroll
            for (int u = 0; u < kB; ++u)
                if (s0 + u < splits) Op::merge(r, P::unpack(q[u]));
        }
        store_result<Op>(out, kept_i, r);
    }
    if (threadIdx.x == 0) counters[blockIdx.x] = 0;
}

// Narrow column walk: the kept mode is unit-stride and the reduced mode is one
// leaf, as for cols_affine, but a CTA owns only kCols kept ordinals and the
// whole fibre.  Lane l reads 16 bytes at column (l % (kCols / 4)) * 4 of row
// l / (kCols / 4) of its warp's row group, so one warp instruction covers
// 128 / kCols rows of kCols * 4 bytes, and the 8 warps interleave the row
// groups.  With enough kept ordinals to give every SM a CTA nothing crosses
// CTAs: no slice partials, no ticket, no fold after the last load.  The CTA
// folds its row streams in shared memory; the fold is the exact merge, so max
// and argmax stay bit-exact whatever the stream order.
//
// Per operation: kept columns per CTA, the resident CTAs per SM the kernel is
// compiled for, and 16-byte loads in flight per lane (0: the operation keeps
// the split walk).  Measured on the 8192 x 4096 transposed walk (GB/s, one
// B200): argmax 5220 / 5697 / 5749 at 8 / 12 / 16 loads (32 columns, two CTAs
// per SM) against 5078 split; max 5440 at 32 columns and eight loads, 5621 at
// 16 columns with four CTAs per SM (one wave of 512 CTAs), 4470 with three
// (two waves), against 5319 split; sum 5367 at eight loads against 5741 split
// (the split walk's cluster fold), slower with more.
template <class Op>
struct NarrowCfg;
template <>
struct NarrowCfg<SumOp> { static constexpr int kCols = 32, kMinBlocks = 2, kU = 0; };
template <>
struct NarrowCfg<MaxOp> { static constexpr int kCols = 16, kMinBlocks = 4, kU = 8; };
template <>
struct NarrowCfg<ArgmaxOp> { static constexpr int kCols = 32, kMinBlocks = 2, kU = 16; };
#ifndef SW_COLS_NARROW_MIN_PER_SM
#define SW_COLS_NARROW_MIN_PER_SM 1  // narrow walk once it has this many CTAs per SM
#endif
constexpr int kNarrowThreads = 256;

template <class Op, bool kSwz, class Ord>
__global__ void __launch_bounds__(kNarrowThreads, NarrowCfg<Op>::kMinBlocks) reduce_cols_narrow(const float* __restrict__ x, DevPlan p,
                                                                         int64_t stride, int64_t weight, void* out) {
    using P = Packed<Op, Ord>;
    constexpr int kNarrowCols = NarrowCfg<Op>::kCols;
    constexpr int kLanesPerRow = kNarrowCols / 4;
    constexpr int kRowsPerWarp = 32 / kLanesPerRow;
    constexpr int kStreams = (kNarrowThreads / 32) * kRowsPerWarp;  // row streams of a CTA
    constexpr int kGroups = kNarrowThreads / kNarrowCols;          // fold groups, 4 streams each
    static_assert(kStreams == 4 * kGroups, "each fold group takes four row streams");
    __shared__ typename P::T part[kStreams][kNarrowCols];
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int cv = lane % kLanesPerRow;
    const int stream_id = warp * kRowsPerWarp + lane / kLanesPerRow;  // rows stream_id + t * kStreams
    const int64_t kv = int64_t(blockIdx.x) * kLanesPerRow + cv;
    const bool live = kv < (p.n_kept >> 2);
    typename Op::S acc[4] = {Op::identity(), Op::identity(), Op::identity(), Op::identity()};
    if (live && stream_id < p.n_red) {
        const int64_t col = p.offset + kept_offset(p.kept, kv * 4);
        LaneWalk<Ord> w;
        w.off0 = int64_t(stream_id) * stride;
        w.doff = int64_t(kStreams) * stride;
        w.ord0 = Ord(int64_t(stream_id) * weight);
        w.dord = Ord(int64_t(kStreams) * weight);
        w.w0 = 0;  // the four components are four columns at the same ordinal
        w.iters = int((p.n_red - stream_id + kStreams - 1) / kStreams);
        FastFold<Op, Ord> f;
        const float* ptr = x + phys<kSwz>(p.swz, col + w.off0);
        constexpr int kU = NarrowCfg<Op>::kU > 0 ? NarrowCfg<Op>::kU : 8;
        if (fast_walk<Op, Ord, kU>(ptr, w.doff, w.iters, f)) {
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[e] = f.component(e, w.ord0, w.dord, Ord(0));
        } else {
            exact_walk<Op, kSwz, Ord>(x, p.swz, col, w, acc, true);
        }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) part[stream_id][cv * 4 + e] = P::pack(acc[e]);
    __syncthreads();
    // thread (g, c) folds streams 4g .. 4g + 3 of column c, then thread c folds the groups
    const int c = threadIdx.x % kNarrowCols;
    const int g = threadIdx.x / kNarrowCols;
    typename Op::S v = P::unpack(part[4 * g][c]);
#pragma unroll
    for (int s = 1; s < 4; ++s) Op::merge(v, P::unpack(part[4 * g + s][c]));
    __syncthreads();
    part[g][c] = P::pack(v);
    __syncthreads();
    const int64_t kept_i = int64_t(blockIdx.x) * kNarrowCols + threadIdx.x;
    if (threadIdx.x < kNarrowCols && kept_i < p.n_kept) {
        typename Op::S r = P::unpack(part[0][threadIdx.x]);
#pragma unroll
        for (int q = 1; q < kGroups; ++q) Op::merge(r, P::unpack(part[q][threadIdx.x]));
        store_result<Op>(out, kept_i, r);
    }
}

// ---- gather ------------------------------------------------------------------
template <class Op>
__global__ void __launch_bounds__(256) reduce_gather(const float* __restrict__ x, DevPlan p, void* out) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t i = warp; i < p.n_kept; i += nwarps) {
        const int64_t row = p.offset + kept_offset(p.kept, i);
        typename Op::S acc = Op::identity();
        for (int64_t j = lane; j < p.n_red; j += 32) {
            int64_t t = j, off = 0, ord = 0;
            for (int l = 0; l < p.red.rank; ++l) {
                const int64_t c = t % p.red.shape[l];
                t /= p.red.shape[l];
                off += c * p.red.stride[l];
                ord += c * p.red.weight[l];
            }
            const int64_t f = swizzle(p.swz, row + off);
            if (f < 0 || f >= p.x_size) {
                report_device_error(SW_ERR_INVALID);
                continue;
            }
            Op::add(acc, load_stream1(x + f), ord);
        }
        acc = warp_reduce<Op>(acc);
        if (lane == 0) store_result<Op>(out, i, acc);
    }
}

// ---- host-side lowering --------------------------------------------------------

int sm_count() {
    static int count = -1;
    if (count < 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
            cudaGetLastError();
            count = 148;
        }
    }
    return count;
}

// Drops unit leaves, records logical weights, merges leaves that walk memory
// contiguously and keep logical order (weight[l+1] == shape[l]*weight[l]).
void lower_leaves(int rank, const int64_t* shape, const int64_t* stride, LeafSet& out, int64_t& numel) {
    out.rank = 0;
    numel = 1;
    int64_t weight = 1;
    for (int l = 0; l < rank; ++l) {
        if (shape[l] != 1) {
            int r = out.rank;
            if (r > 0 && out.stride[r - 1] * out.shape[r - 1] == stride[l] &&
                out.weight[r - 1] * out.shape[r - 1] == weight) {
                out.shape[r - 1] *= shape[l];
            } else {
                out.shape[r] = shape[l];
                out.stride[r] = stride[l];
                out.weight[r] = weight;
                out.rank = r + 1;
            }
        }
        weight *= shape[l];
        numel *= shape[l];
    }
}

// Moves leaf `l` to position 0 (traversal order only; weights keep the
// logical ordinal).
void leaf_to_front(LeafSet& s, int l) {
    if (l <= 0) return;
    LeafSet t = s;
    s.shape[0] = t.shape[l];
    s.stride[0] = t.stride[l];
    s.weight[0] = t.weight[l];
    int w = 1;
    for (int i = 0; i < t.rank; ++i) {
        if (i == l) continue;
        s.shape[w] = t.shape[i];
        s.stride[w] = t.stride[i];
        s.weight[w] = t.weight[i];
        ++w;
    }
}

int unit_leaf(const LeafSet& s) {
    for (int l = 0; l < s.rank; ++l)
        if (s.stride[l] == 1 && s.shape[l] % 4 == 0) return l;
    return -1;
}

bool strides_mult4(const LeafSet& s, int skip) {
    for (int l = 0; l < s.rank; ++l)
        if (l != skip && s.stride[l] % 4 != 0) return false;
    return true;
}

// A swizzle keeps 4-element vectors intact when no stage reads or writes
// bits 0..1 of the flat index.
bool swizzle_keeps_vec4(const Swz& s) {
    for (int i = 0; i < s.rank; ++i) {
        const int tgt = s.shift[i] > 0 ? s.base[i] : s.base[i] - s.shift[i];
        const int src = s.shift[i] > 0 ? s.base[i] + s.shift[i] : s.base[i];
        if (tgt < 2 || src < 2) return false;
    }
    return true;
}

// Whether swizzle(f + k*step) == swizzle(f) + k*step for all f, k: true when
// every bit a stage reads or writes lies below the lowest set bit of step.
bool swizzle_commutes(const Swz& s, int64_t step) {
    if (s.rank == 0) return true;
    if (step == 0) return false;
    int64_t a = step < 0 ? -step : step;
    int low = 0;
    while (((a >> low) & 1) == 0) ++low;
    for (int i = 0; i < s.rank; ++i) {
        const int tgt = s.shift[i] > 0 ? s.base[i] : s.base[i] - s.shift[i];
        const int src = s.shift[i] > 0 ? s.base[i] + s.shift[i] : s.base[i];
        if (std::max(tgt, src) + s.bits[i] - 1 >= low) return false;
    }
    return true;
}

// Highest bit a swizzle may set.
int swizzle_top_bit(const Swz& s) {
    int top = -1;
    for (int i = 0; i < s.rank; ++i) {
        const int tgt = s.shift[i] > 0 ? s.base[i] : s.base[i] - s.shift[i];
        top = std::max(top, tgt + s.bits[i] - 1);
    }
    return top;
}

// Where the split column walk takes its scratch from: the library's
// per-(device, stream) buffer (base == nullptr), or a fixed region the caller
// of the entry point chose (base, bytes) whose counters are cleared per launch.
struct ScratchSource {
    void* base = nullptr;
    size_t bytes = 0;
};

// Scratch memory of the split column walk: one buffer per (device, stream),
// so the launches of one stream use it in order.  It comes from the device's
// stream-ordered pool on first use (and is regrown, the old buffer released
// after the stream's earlier work, when a launch needs more); its counters
// are zeroed on the same stream and are zero again after every launch.
struct ScratchSlot {
    int dev;
    cudaStream_t stream;
    void* ptr;
    size_t bytes;
};
std::mutex g_scratch_mu;
std::vector<ScratchSlot>& scratch_slots() {
    static std::vector<ScratchSlot> slots;
    return slots;
}

int reduce_scratch(size_t need, cudaStream_t stream, void** out) {
    int dev = 0;
    SW_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    ScratchSlot* slot = nullptr;
    for (auto& e : scratch_slots())
        if (e.dev == dev && e.stream == stream) slot = &e;
    if (slot && slot->bytes >= need) {
        *out = slot->ptr;
        return SW_OK;
    }
    const size_t bytes = (need + (size_t(1) << 20) - 1) & ~((size_t(1) << 20) - 1);  // whole MiB
    void* ptr = nullptr;
    cudaError_t err = cudaMallocAsync(&ptr, bytes, stream);
    if (err == cudaErrorMemoryAllocation) {
        cudaGetLastError();
        return fail(SW_ERR_NOMEM, "sw_reduce_f32: out of device memory for %zu bytes of scratch", bytes);
    }
    SW_CUDA_TRY(err, "cudaMallocAsync (reduction scratch)");
    SW_CUDA_TRY(cudaMemsetAsync(ptr, 0, bytes, stream), "zeroing reduction scratch");
    if (slot) {
        SW_CUDA_TRY(cudaFreeAsync(slot->ptr, stream), "cudaFreeAsync (reduction scratch)");
        slot->ptr = ptr;
        slot->bytes = bytes;
    } else {
        scratch_slots().push_back({dev, stream, ptr, bytes});
    }
    *out = ptr;
    return SW_OK;
}

struct Launch {
    int kernel = 2;  // 0 rows_vec, 1 cols_vec, 2 gather, 3 rows_affine, 4 cols_affine, 5 cols_narrow
    int splits = 1;
    int wpr = 1;     // warps per row of rows_affine
    RowWalk rw{};
    int64_t cstride = 0, cweight = 0;
};

template <class Op, bool kSwz, class Ord>
int launch_affine(const float* x, const DevPlan& p, const Launch& L, void* out, cudaStream_t stream,
                  const ScratchSource& src) {
    if (L.kernel == 3) {
        // every warp resident at once, each with the same number of rows
        static int per_sm = 0;  // one query per kernel instantiation
        if (per_sm == 0) {
            int q = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&q, reduce_rows_affine<Op, kSwz, Ord>,
                                                              kRowsAffThreads, 0) != cudaSuccess || q < 1) {
                cudaGetLastError();
                q = 1;
            }
            per_sm = q;
        }
        const int64_t capacity = int64_t(sm_count()) * per_sm * kRowsAffWarps;
        const int64_t rpw = (p.n_kept + capacity - 1) / capacity;
        const int64_t warps = (p.n_kept + rpw - 1) / rpw;
        const int64_t blocks = (warps + kRowsAffWarps - 1) / kRowsAffWarps;
        const cudaError_t err = launch_pdl(reduce_rows_affine<Op, kSwz, Ord>, dim3((unsigned)blocks),
                                           dim3(kRowsAffThreads), 0, stream, x, p, L.rw, rpw, out);
        if (err != cudaSuccess) return cuda_fail(err, "reduce_rows_affine launch");
        return SW_OK;
    }
    if (L.kernel == 5 && NarrowCfg<Op>::kU > 0) {
        const int64_t blocks = (p.n_kept + NarrowCfg<Op>::kCols - 1) / NarrowCfg<Op>::kCols;
        const cudaError_t err = launch_pdl(reduce_cols_narrow<Op, kSwz, Ord>, dim3((unsigned)blocks),
                                           dim3(kNarrowThreads), 0, stream, x, p, L.cstride, L.cweight, out);
        if (err != cudaSuccess) return cuda_fail(err, "reduce_cols_narrow launch");
        return SW_OK;
    }
    const int64_t col_blocks = (p.n_kept / 4 + 31) / 32;
    // Sums fold their slices in a cluster (measured 2% faster on the 8192 x
    // 4096 transposed walk); max and argmax keep the scratch fold, which
    // measured 1% faster for their 8-byte (value, ordinal) partials.
    if (std::is_same<Op, SumOp>::value && L.splits >= 2 && L.splits <= kMaxClusterSlices) {
        // the slices of a column block form one portable cluster: no scratch
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)col_blocks, (unsigned)L.splits, 1);
        cfg.blockDim = dim3(kColsAffThreads, 1, 1);
        cfg.stream = stream;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = (unsigned)L.splits;
        attr[0].val.clusterDim.z = 1;
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 2;
        using PT = typename Packed<Op, Ord>::T;
        const cudaError_t err = cudaLaunchKernelEx(&cfg, reduce_cols_affine<Op, kSwz, Ord, true>, x, p, L.cstride,
                                                   L.cweight, out, static_cast<PT*>(nullptr),
                                                   static_cast<unsigned*>(nullptr));
        if (err != cudaSuccess) return cuda_fail(err, "reduce_cols_affine (cluster) launch");
        return SW_OK;
    }
    // split column walk past one cluster: more than one slice needs scratch for the partials
    using PT = typename Packed<Op, Ord>::T;
    PT* partials = nullptr;
    unsigned* counters = nullptr;
    if (L.splits > 1) {
        const size_t cbytes = (size_t(col_blocks) * sizeof(unsigned) + 255) & ~size_t(255);
        const size_t need = cbytes + size_t(L.splits) * size_t(p.n_kept) * sizeof(PT);
        void* base = nullptr;
        if (src.base) {
            if (need > src.bytes)
                return fail(SW_ERR_UNSUPPORTED,
                            "sw_reduce_f32_noalloc: this reduction needs %zu bytes of scratch; the static scratch "
                            "holds %zu",
                            need, src.bytes);
            base = src.base;
            // the region keeps the previous call's contents: clear the counters
            SW_CUDA_TRY(cudaMemsetAsync(base, 0, cbytes, stream), "clearing the static scratch counters");
        } else {
            const int rc = reduce_scratch(need, stream, &base);
            if (rc != SW_OK) return rc;
        }
        counters = static_cast<unsigned*>(base);
        partials = reinterpret_cast<PT*>(static_cast<char*>(base) + cbytes);
    }
    const cudaError_t err = launch_pdl(reduce_cols_affine<Op, kSwz, Ord, false>, dim3((unsigned)col_blocks, (unsigned)L.splits),
                                       dim3(kColsAffThreads), 0, stream, x, p, L.cstride, L.cweight, out, partials,
                                       counters);
    if (err != cudaSuccess) return cuda_fail(err, "reduce_cols_affine launch");
    return SW_OK;
}

template <class Op, class Ord>
int launch_affine_swz(const float* x, const DevPlan& p, const Launch& L, void* out, cudaStream_t stream,
                      const ScratchSource& src) {
    return p.swz.rank > 0 ? launch_affine<Op, true, Ord>(x, p, L, out, stream, src)
                          : launch_affine<Op, false, Ord>(x, p, L, out, stream, src);
}

template <class Op>
int launch_for(const float* x, const DevPlan& p, const Launch& L, void* out, cudaStream_t stream,
               const ScratchSource& src) {
    if (L.kernel >= 3) {
        // 32-bit ordinals whenever every ordinal of the fibre fits
        int rc = p.n_red < (int64_t(1) << 30) ? launch_affine_swz<Op, int32_t>(x, p, L, out, stream, src)
                                              : launch_affine_swz<Op, int64_t>(x, p, L, out, stream, src);
        if (rc != SW_OK) return rc;
    } else if (L.kernel == 0) {
        const int64_t blocks = std::min<int64_t>((p.n_kept + 7) / 8, int64_t(sm_count()) * 8);
        reduce_rows_vec<Op><<<(unsigned)std::max<int64_t>(blocks, 1), 256, 0, stream>>>(x, p, out);
    } else if (L.kernel == 1) {
        cudaLaunchConfig_t cfg = {};
        const int64_t kept_vecs = p.n_kept / 4;
        cfg.gridDim = dim3((unsigned)((kept_vecs + 31) / 32), (unsigned)L.splits, 1);
        cfg.blockDim = dim3(kColsThreads, 1, 1);
        cfg.dynamicSmemBytes = 0;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = (unsigned)L.splits;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaError_t err = cudaLaunchKernelEx(&cfg, reduce_cols_vec<Op>, x, p, out);
        if (err != cudaSuccess) return cuda_fail(err, "reduce_cols_vec launch");
    } else {
        int64_t blocks = std::min<int64_t>((p.n_kept + 7) / 8, int64_t(sm_count()) * 8);
        reduce_gather<Op><<<(unsigned)std::max<int64_t>(blocks, 1), 256, 0, stream>>>(x, p, out);
    }
    SW_LAUNCH_CHECK("reduction launch");
    return SW_OK;
}

// Chooses the kernel for a lowered plan (see the file header).
Launch choose(DevPlan& p, int kind, bool aligned) {
    Launch L;
    const int ru = unit_leaf(p.red);
    const int ku = unit_leaf(p.kept);
    if (aligned && ru >= 0 && strides_mult4(p.red, ru) && strides_mult4(p.kept, -1)) {
        // rows: try the affine walk first
        const int64_t run = p.red.shape[ru];
        const int64_t nv0 = run / 4;
        const int others = p.red.rank - 1;
        int ol = -1;
        for (int l = 0; l < p.red.rank; ++l)
            if (l != ru) ol = l;
        bool affine = false;
        RowWalk rw{run, 1, 0, 0, p.red.weight[ru]};
        if (others == 0 && nv0 % 32 == 0) {
            affine = true;
        } else if (others == 1 && 32 % nv0 == 0 && p.red.shape[ol] % (32 / nv0) == 0) {
            rw.nruns = p.red.shape[ol];
            rw.rstride = p.red.stride[ol];
            rw.rweight = p.red.weight[ol];
            // argmax folds each lane in increasing ordinal order
            affine = kind != SW_REDUCE_ARGMAX || rw.rweight >= run * rw.w0;
        }
        // the lane step must commute with the swizzle
        const int64_t step = nv0 >= 32 ? 128 : (32 / nv0) * rw.rstride;
        if (affine && swizzle_commutes(p.swz, step)) {
            L.kernel = 3;
            L.rw = rw;
            return L;
        }
        leaf_to_front(p.red, ru);
        L.kernel = 0;
        return L;
    }
    if (aligned && ku == 0 && p.n_kept % 4 == 0 && strides_mult4(p.kept, 0) && strides_mult4(p.red, -1)) {
        const int64_t col_blocks = (p.n_kept / 4 + 31) / 32;
        // every CTA resident at once (kColsAffPerSm per SM): no second, partial wave
        const int64_t want = std::max<int64_t>(1, int64_t(sm_count()) * kColsAffPerSm / col_blocks);
        int ncols = 0, nu = 0;  // the operation's narrow-walk width and load depth
        if (kind == SW_REDUCE_SUM) { ncols = NarrowCfg<SumOp>::kCols; nu = NarrowCfg<SumOp>::kU; }
        if (kind == SW_REDUCE_MAX) { ncols = NarrowCfg<MaxOp>::kCols; nu = NarrowCfg<MaxOp>::kU; }
        if (kind == SW_REDUCE_ARGMAX) { ncols = NarrowCfg<ArgmaxOp>::kCols; nu = NarrowCfg<ArgmaxOp>::kU; }
        const int64_t narrow_streams = nu > 0 ? (kNarrowThreads / 32) * (32 / (ncols / 4)) : 0;
        if (nu > 0 && p.red.rank == 1 && p.n_kept >= int64_t(sm_count()) * SW_COLS_NARROW_MIN_PER_SM * ncols &&
            swizzle_commutes(p.swz, narrow_streams * p.red.stride[0])) {
            // a CTA of ncols kept ordinals for every SM: whole fibres per CTA
            L.kernel = 5;
            L.cstride = p.red.stride[0];
            L.cweight = p.red.weight[0];
            return L;
        }
        if (p.red.rank == 1 && swizzle_commutes(p.swz, int64_t(kColsAffWarps) * p.red.stride[0])) {
            // slices meet in scratch memory: no cap from the cluster size.  About
            // 2.6 CTAs per SM streams fastest for every operation (measured on
            // the 8192 x 4096 transposed walk, 64 column blocks: 6 slices; with
            // 16-byte max / argmax partials max preferred 5)
            const double per_sm = 2.6;
            const int64_t target = std::max<int64_t>(1, std::llround(double(sm_count()) * per_sm / double(col_blocks)));
            L.kernel = 4;
            L.splits = (int)std::max<int64_t>(1, std::min<int64_t>({std::min(target, std::max<int64_t>(want, 1)),
                                                                      kMaxColSlices, p.n_red}));
            L.cstride = p.red.stride[0];
            L.cweight = p.red.weight[0];
        } else {
            // slices meet in distributed shared memory: at most one portable cluster
            L.kernel = 1;
            L.splits = (int)std::max<int64_t>(1, std::min<int64_t>({want, 8, p.n_red}));
        }
        return L;
    }
    return L;
}

}  // namespace
}  // namespace sw

namespace sw {
namespace {

// Validates and lowers a plan, then launches; `src` says where the split
// column walk takes its scratch from.
int reduce_entry(const sw_reduce_plan* plan, const float* x, int64_t x_size, void* out, void* stream,
                 const ScratchSource& src) {
    if (!plan || !out) return fail(SW_ERR_INVALID, "sw_reduce_f32: null plan or output");
    if (plan->kind < SW_REDUCE_SUM || plan->kind > SW_REDUCE_SUM_F64)
        return fail(SW_ERR_INVALID, "sw_reduce_f32: unknown reduction kind %d", plan->kind);
    if (plan->kept_rank < 0 || plan->kept_rank > SW_MAX_LEAVES || plan->reduced_rank < 0 ||
        plan->reduced_rank > SW_MAX_LEAVES || plan->swizzle_rank < 0 || plan->swizzle_rank > SW_MAX_SWIZZLE)
        return fail(SW_ERR_INVALID, "sw_reduce_f32: leaf or swizzle rank out of range");
    DevPlan p;
    std::memset(&p, 0, sizeof(p));
    p.offset = plan->offset;
    p.x_size = x_size;
    for (int l = 0; l < plan->kept_rank; ++l)
        if (plan->kept_shape[l] < 0) return fail(SW_ERR_INVALID, "sw_reduce_f32: negative extent");
    for (int l = 0; l < plan->reduced_rank; ++l)
        if (plan->reduced_shape[l] < 0) return fail(SW_ERR_INVALID, "sw_reduce_f32: negative extent");
    lower_leaves(plan->kept_rank, plan->kept_shape, plan->kept_stride, p.kept, p.n_kept);
    lower_leaves(plan->reduced_rank, plan->reduced_shape, plan->reduced_stride, p.red, p.n_red);
    p.swz.rank = plan->swizzle_rank;
    for (int i = 0; i < plan->swizzle_rank; ++i) {
        p.swz.bits[i] = plan->swizzle_bits[i];
        p.swz.base[i] = plan->swizzle_base[i];
        p.swz.shift[i] = plan->swizzle_shift[i];
        // the constraints of SwizzleStage (src/strideweave/core/swizzle.py:44-60)
        if (p.swz.bits[i] <= 0 || p.swz.base[i] < 0 || p.swz.shift[i] == 0 ||
            std::abs(p.swz.shift[i]) < p.swz.bits[i] || p.swz.bits[i] + p.swz.base[i] + std::abs(p.swz.shift[i]) > 62)
            return fail(SW_ERR_INVALID, "sw_reduce_f32: invalid swizzle stage %d", i);
    }
    if (p.n_kept == 0) return ok();
    if (p.n_red == 0) {
        if (plan->kind != SW_REDUCE_SUM && plan->kind != SW_REDUCE_SUM_F64)
            return fail(SW_ERR_INVALID, "reduction fibers must be non-empty");
        SW_CUDA_TRY(cudaMemsetAsync(out, 0, size_t(p.n_kept) * 4, (cudaStream_t)stream), "zero sum");
        return ok();
    }
    if (!x) return fail(SW_ERR_INVALID, "sw_reduce_f32: null input");
    // Address range of the view (before the swizzle).
    int64_t lo = p.offset, hi = p.offset;
    for (int l = 0; l < p.kept.rank; ++l) {
        const int64_t span = (p.kept.shape[l] - 1) * p.kept.stride[l];
        if (span < 0) lo += span; else hi += span;
    }
    for (int l = 0; l < p.red.rank; ++l) {
        const int64_t span = (p.red.shape[l] - 1) * p.red.stride[l];
        if (span < 0) lo += span; else hi += span;
    }
    if (lo < 0 || hi >= x_size)
        return fail(SW_ERR_INVALID, "sw_reduce_f32: view addresses [%lld, %lld] outside carrier of %lld elements",
                    (long long)lo, (long long)hi, (long long)x_size);
    if (p.swz.rank > 0) {
        // The swizzle only rewrites bits up to `top`: every address stays in the
        // enclosing aligned 2^(top+1) window, which must lie inside the carrier.
        const int top = swizzle_top_bit(p.swz);
        const int64_t win = int64_t(1) << (top + 1);
        const int64_t hi_window = (hi / win + 1) * win - 1;
        if (hi_window >= x_size)
            return fail(SW_ERR_INVALID, "sw_reduce_f32: swizzle may address past the carrier end");
    }
    cudaStream_t s = (cudaStream_t)stream;
    if (plan->kind == SW_REDUCE_SUM_F64) {
        // the widened sum walks any layout with the general gather kernel
        const int64_t blocks = std::min<int64_t>((p.n_kept + 7) / 8, int64_t(sm_count()) * 8);
        reduce_gather<SumOp64><<<(unsigned)std::max<int64_t>(blocks, 1), 256, 0, s>>>(x, p, out);
        SW_LAUNCH_CHECK("reduction launch");
        return ok();
    }
    const bool aligned = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (p.offset % 4 == 0) &&
                         swizzle_keeps_vec4(p.swz);
    const Launch L = choose(p, plan->kind, aligned);
    int rc;
    switch (plan->kind) {
        case SW_REDUCE_SUM: rc = launch_for<SumOp>(x, p, L, out, s, src); break;
        case SW_REDUCE_MAX: rc = launch_for<MaxOp>(x, p, L, out, s, src); break;
        default: rc = launch_for<ArgmaxOp>(x, p, L, out, s, src); break;
    }
    if (rc != SW_OK) return rc;
    return ok();
}

}  // namespace
}  // namespace sw

extern "C" int sw_reduce_f32(const sw_reduce_plan* plan, const float* x, int64_t x_size,
                             void* out, void* stream) {
    return sw::reduce_entry(plan, x, x_size, out, stream, sw::ScratchSource{});
}

// ---- a reduction that allocates nothing -----------------------------------------
//
// sw_reduce_f32 may reserve a small scratch buffer from the device's memory pool
// the first time a stream runs a split column walk.  Some callers cannot let a
// library allocate: an engine that has already divided all of the device's
// memory among its own pools, or a process whose device-memory budget is fixed
// and audited allocation by allocation.  sw_reduce_f32_noalloc serves them with
// the split walk's scratch in a fixed array compiled into this library.

namespace {

// Every GPU that loads the library holds these 2 MiB until the process exits.
// A split column walk needs at most SMs x 4 x 128 partials of 16 bytes plus its
// counters, so this covers every plan on devices with up to 255 SMs.
constexpr size_t kStaticScratchBytes = size_t(2) << 20;
constexpr int kMaxDevices = 64;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// The device address of g_static_scratch on the current device.  In host code
// the array's name stands for a host-side shadow, never a device address, so
// it is looked up once per device with that device current.  The cached
// address belongs to the device's primary context; a device reset, which
// creates a new context, is not supported by this entry point.
int static_scratch(void** out) {
    static std::mutex mu;
    static void* addr[kMaxDevices] = {};
    int dev = 0;
    SW_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices)
        return sw::fail(SW_ERR_UNSUPPORTED, "sw_reduce_f32_noalloc: device ordinal %d above %d", dev, kMaxDevices - 1);
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        SW_CUDA_TRY(cudaGetSymbolAddress(&p, g_static_scratch), "cudaGetSymbolAddress (static reduction scratch)");
        addr[dev] = p;
    }
    *out = addr[dev];
    return SW_OK;
}

}  // namespace

extern "C" int sw_reduce_f32_noalloc(const sw_reduce_plan* plan, const float* x, int64_t x_size, void* out,
                                     void* stream) {
    void* base = nullptr;
    const int rc = static_scratch(&base);
    if (rc != SW_OK) return rc;
    sw::ScratchSource src;
    src.base = base;
    src.bytes = kStaticScratchBytes;
    return sw::reduce_entry(plan, x, x_size, out, stream, src);
}
