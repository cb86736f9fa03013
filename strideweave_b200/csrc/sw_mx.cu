// sw_mx.cu - OCP MX v1.0 quantise / dequantise (MXFP8_E4M3 and MXFP4 E2M1
// payload planes plus E8M0 per-32 scale planes).
//
// Conversion rules (identical to the CPU restatement used by the tests):
//   block   = 32 consecutive elements along the quantised axis (a trailing
//             partial block uses the elements that exist);
//   e       = floor(log2(amax)) - emax_elem (8 for E4M3, 2 for E2M1), clamped
//             to >= -127; scale byte = e + 127;
//   amax==0 -> scale 0x00, each zero keeps its sign;
//   NaN/Inf -> scale 0xFF (NaN), payload codes 0;
//   element = RNE(V * 2^-e) saturated to the largest finite element.
// V * 2^-e is exact in binary32 whenever the result can round to a non-zero
// element, so cvt.rn.satfinite on the product gives the exact rounding.
//
// There is no reference kernel: the reference registers MXFP8_E4M3 / MXFP4 as
// descriptors only (src/strideweave/carriers/_dtype/builtins.py:39-52).
#include <algorithm>
#include <cstring>

#include "sw_common.cuh"
#include "sw_gelu.cuh"
#include "sw_ptx.cuh"

namespace sw {
namespace {

// floor(log2) of a finite non-zero |x| bit pattern.
__device__ __forceinline__ int floor_log2_bits(uint32_t a) {
    const uint32_t ex = a >> 23;
    if (ex != 0) return int(ex) - 127;
    return (31 - __clz(a & 0x7FFFFF)) - 149;
}

template <int FMT>
__device__ __forceinline__ int emax_elem() { return FMT == SW_MX_E4M3 ? 8 : 2; }

// Shared exponent and scale byte of a block from max |bits| over it.
template <int FMT>
__device__ __forceinline__ void block_scale(uint32_t amax_bits, uint8_t& scale, float& inv, bool& special) {
    special = amax_bits >= 0x7F800000u;
    int e;
    if (amax_bits == 0) e = -127;
    else e = max(floor_log2_bits(amax_bits) - emax_elem<FMT>(), -127);
    scale = special ? uint8_t(0xFF) : uint8_t(e + 127);
    inv = __uint_as_float(uint32_t(127 - e) << 23);  // 2^-e, normal for e in [-127, 125]
}

__device__ __forceinline__ uint32_t e4m3x4(float a, float b, float c, float d) {
    uint32_t out;
    asm("{\n.reg .b16 lo, hi;\n"
        "cvt.rn.satfinite.e4m3x2.f32 lo, %2, %1;\n"
        "cvt.rn.satfinite.e4m3x2.f32 hi, %4, %3;\n"
        "mov.b32 %0, {lo, hi};\n}"
        : "=r"(out) : "f"(a), "f"(b), "f"(c), "f"(d));
    return out;
}

__device__ __forceinline__ uint32_t e2m1x8(const float* v) {
    uint32_t out;
    asm("{\n.reg .b8 b0, b1, b2, b3;\n"
        "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n"
        "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n"
        "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n"
        "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n"
        "mov.b32 %0, {b0, b1, b2, b3};\n}"
        : "=r"(out)
        : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
    return out;
}

__host__ __device__ __forceinline__ int64_t scale_offset(int layout, int64_t r, int64_t kb, int64_t kblocks,
                                                          int64_t ld) {
    if (layout == SW_SCALES_TC128) {
        const int64_t katoms = (kblocks + 3) / 4;
        return (r / 128) * katoms * 512 + (kb / 4) * 512 + (r % 32) * 16 + ((r / 32) % 4) * 4 + (kb % 4);
    }
    return r * ld + kb;
}

__device__ __forceinline__ float max_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

__device__ __forceinline__ float max_nan_abs(float m, float v) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(m), "f"(fabsf(v)));
    return r;
}

// Byte offset of block (r, kb) in a scale plane, split into a per-row base and a
// per-block step so that a walk along a row adds instead of recomputing.
__device__ __forceinline__ int64_t scale_row_base(int layout, int64_t r, int64_t kblocks, int64_t ld) {
    if (layout == SW_SCALES_TC128) return (r >> 7) * ((kblocks + 3) >> 2) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4;
    return r * ld;
}
__device__ __forceinline__ int64_t scale_block_step(int layout, int64_t kb) {
    return layout == SW_SCALES_TC128 ? (kb >> 2) * 512 + (kb & 3) : kb;
}

// ---- quantise: blocks along a unit-stride axis --------------------------------
// A warp walks a segment of up to 2048 elements of one row, 256 (eight blocks)
// per step: four lanes per block, eight elements per lane (two 16-byte loads).
// Row and scale addresses are set up once per segment and then advanced.
constexpr int64_t kQuantSegment = 2048;

template <int FMT>
__global__ void __launch_bounds__(256) quantize_rows(const float* __restrict__ x, int64_t rows, int64_t cols,
                                                     int64_t ldx, uint8_t* __restrict__ payload, int64_t ldp,
                                                     uint8_t* __restrict__ scales, int layout, int64_t lds) {
    pdl_enter();
    const int64_t kblocks = (cols + 31) / 32;
    const int64_t segs = (cols + kQuantSegment - 1) / kQuantSegment;
    const int64_t units = rows * segs;
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t u = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; u < units; u += nwarps) {
        int64_t r, sg;
        if (units <= int64_t(0x7FFFFFFF)) {
            const uint32_t uu = uint32_t(u), g = uint32_t(segs);
            const uint32_t q = uu / g;
            r = q;
            sg = uu - q * g;
        } else {
            r = u / segs;
            sg = u - r * segs;
        }
        const int64_t e_begin = sg * kQuantSegment;
        const int64_t e_end = min(cols, e_begin + kQuantSegment);
        const float* src = x + r * ldx + e_begin + lane * 8;
        uint8_t* dst = payload + r * ldp + (FMT == SW_MX_E4M3 ? e_begin + lane * 8 : (e_begin + lane * 8) / 2);
        const int64_t srow = scale_row_base(layout, r, kblocks, lds);
        const bool row_aligned = ((reinterpret_cast<uintptr_t>(x + r * ldx) & 15) == 0);
        for (int64_t e0 = e_begin; e0 < e_end; e0 += 256, src += 256, dst += (FMT == SW_MX_E4M3 ? 256 : 128)) {
            const int64_t c0 = e0 + lane * 8;
            const int64_t kb = (e0 >> 5) + (lane >> 2);
            float v[8];
            const bool full = row_aligned && e0 + 256 <= e_end;
            if (full) {
                const float4 a = __ldcs(reinterpret_cast<const float4*>(src));
                const float4 b = __ldcs(reinterpret_cast<const float4*>(src) + 1);
                v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
                v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = c0 + i < cols ? src[i] : 0.0f;
            }
            float m = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) m = max_nan_abs(m, v[i]);
            m = max_nan(m, __shfl_xor_sync(0xffffffffu, m, 1));
            m = max_nan(m, __shfl_xor_sync(0xffffffffu, m, 2));
            if (kb >= kblocks) continue;
            uint8_t sc;
            float inv;
            bool special;
            block_scale<FMT>(__float_as_uint(m), sc, inv, special);
            if ((lane & 3) == 0) scales[srow + scale_block_step(layout, kb)] = sc;
            uint32_t w0, w1;
            if (!special) {
                float q[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) q[i] = __fmul_rn(v[i], inv);
                if (FMT == SW_MX_E4M3) {
                    w0 = e4m3x4(q[0], q[1], q[2], q[3]);
                    w1 = e4m3x4(q[4], q[5], q[6], q[7]);
                } else {
                    w0 = e2m1x8(q);
                    w1 = 0;
                }
            } else {
                w0 = w1 = 0;  // a NaN/Inf block: scale 0xFF, payload codes 0
            }
            if (FMT == SW_MX_E4M3) {
                if (full && ((reinterpret_cast<uintptr_t>(dst) & 7) == 0)) {
                    *reinterpret_cast<uint2*>(dst) = make_uint2(w0, w1);
                } else {
                    for (int i = 0; i < 8 && c0 + i < cols; ++i) dst[i] = uint8_t(((i < 4 ? w0 : w1) >> (8 * (i & 3))) & 0xFF);
                }
            } else {
                if (full && ((reinterpret_cast<uintptr_t>(dst) & 3) == 0)) {
                    *reinterpret_cast<uint32_t*>(dst) = w0;
                } else {
                    // ragged tail: keep the nibbles beyond `cols` as they were
                    for (int i = 0; i < 8 && c0 + i < cols; i += 2) {
                        const uint8_t byte = uint8_t((w0 >> (4 * i)) & 0xFF);
                        if (c0 + i + 1 < cols) dst[i / 2] = byte;
                        else dst[i / 2] = uint8_t((dst[i / 2] & 0xF0) | (byte & 0x0F));
                    }
                }
            }
        }
    }
}

// ---- quantise: generic strides (one thread per 32-block) -----------------------
// Threads of a warp take consecutive rows, so a unit row stride (blocks along a
// strided axis, e.g. a transposed operand) reads 128-byte lines.
template <int FMT>
__global__ void __launch_bounds__(256) quantize_strided(const float* __restrict__ x, int64_t rows, int64_t cols,
                                                        int64_t ldr, int64_t ldc, uint8_t* __restrict__ payload,
                                                        int64_t ldp, uint8_t* __restrict__ scales, int layout,
                                                        int64_t lds) {
    pdl_enter();
    const int64_t kblocks = (cols + 31) / 32;
    const int64_t total = rows * kblocks;
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < total; t += stride) {
        const int64_t r = t % rows;
        const int64_t kb = t / rows;
        const int64_t c0 = kb * 32;
        const int len = int((cols - c0) < 32 ? (cols - c0) : 32);
        float v[32];
        uint32_t amax = 0;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            v[i] = i < len ? __ldcs(x + r * ldr + (c0 + i) * ldc) : 0.0f;
            amax = max(amax, __float_as_uint(v[i]) & 0x7FFFFFFFu);
        }
        uint8_t sc;
        float inv;
        bool special;
        block_scale<FMT>(amax, sc, inv, special);
        scales[scale_offset(layout, r, kb, kblocks, lds)] = sc;
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = special ? 0.0f : __fmul_rn(v[i], inv);
        if (FMT == SW_MX_E4M3) {
            uint8_t* dst = payload + r * ldp + c0;
            uint32_t w[8];
#pragma unroll
            for (int g = 0; g < 8; ++g) w[g] = e4m3x4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
            if (len == 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
                reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
                reinterpret_cast<uint4*>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
            } else {
                for (int c = 0; c < len; ++c) dst[c] = uint8_t((w[c / 4] >> (8 * (c % 4))) & 0xFF);
            }
        } else {
            uint8_t* dst = payload + r * ldp + c0 / 2;
            uint32_t w[4];
#pragma unroll
            for (int g = 0; g < 4; ++g) w[g] = e2m1x8(v + 8 * g);
            if (len == 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
                *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
            } else {
                for (int c = 0; c < len; c += 2) {
                    const uint8_t byte = uint8_t((w[c / 8] >> (4 * (c % 8))) & 0xFF);
                    if (c + 1 < len) dst[c / 2] = byte;
                    else dst[c / 2] = uint8_t((dst[c / 2] & 0xF0) | (byte & 0x0F));
                }
            }
        }
    }
}

// 16-byte global -> shared copies that complete asynchronously (cp.async).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ---- quantise: blocks along a strided axis with unit row stride ---------------
// (a K x N operand quantised along K, i.e. the blocks of each of N rows run down
// a column).  A CTA stages a 32 (block) x 128 (row) tile through shared memory
// with 16-byte loads along the contiguous rows, then each of its 128 threads
// quantises one row's block from the tile in two passes over shared memory
// (the amax, then scale-and-pack), so only the packed words live in
// registers and eight CTAs fit on an SM.  Needs rows % 4 == 0, a 16-byte
// aligned source and a column pitch that is a multiple of 4 elements.
constexpr int kTileRows = 128;

template <int FMT>
__global__ void __launch_bounds__(kTileRows, 8) quantize_cols_tiled(const float* __restrict__ x, int64_t rows,
                                                                 int64_t cols, int64_t ldc,
                                                                 uint8_t* __restrict__ payload, int64_t ldp,
                                                                 uint8_t* __restrict__ scales, int layout,
                                                                 int64_t lds) {
    __shared__ __align__(16) float tile[32][kTileRows + 4];
    pdl_enter();
    const int64_t kblocks = (cols + 31) / 32;
    const int64_t rtiles = (rows + kTileRows - 1) / kTileRows;
    const int64_t ntiles = rtiles * kblocks;
    const int t = threadIdx.x;
    for (int64_t tt = blockIdx.x; tt < ntiles; tt += gridDim.x) {
        const int64_t kb = tt / rtiles;
        const int64_t r0 = (tt - kb * rtiles) * kTileRows;
        const int64_t c0 = kb * 32;
        const int len = int((cols - c0) < 32 ? (cols - c0) : 32);
        const int rc = (t & 31) * 4;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int kr = (t >> 5) + 4 * i;
            float4 q = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (kr < len && r0 + rc < rows)
                q = __ldcs(reinterpret_cast<const float4*>(x + (c0 + kr) * ldc + r0 + rc));
            *reinterpret_cast<float4*>(&tile[kr][rc]) = q;
        }
        __syncthreads();
        const int64_t r = r0 + t;
        if (r < rows) {
            // pass 1: the block's amax from the tile; pass 2: re-read, scale and pack
            float m = 0.0f;
#pragma unroll
            for (int i = 0; i < 32; ++i) m = max_nan_abs(m, tile[i][t]);
            uint8_t sc;
            float inv;
            bool special;
            block_scale<FMT>(__float_as_uint(m), sc, inv, special);
            scales[scale_offset(layout, r, kb, kblocks, lds)] = sc;
            if (special) inv = 0.0f;  // payload codes 0 below
            if (FMT == SW_MX_E4M3) {
                uint32_t w[8];
#pragma unroll
                for (int g = 0; g < 8; ++g)
                    w[g] = special ? 0u
                                   : e4m3x4(__fmul_rn(tile[4 * g][t], inv), __fmul_rn(tile[4 * g + 1][t], inv),
                                            __fmul_rn(tile[4 * g + 2][t], inv), __fmul_rn(tile[4 * g + 3][t], inv));
                uint8_t* dst = payload + r * ldp + kb * 32;
                if (len == 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
                    reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
                    reinterpret_cast<uint4*>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
                } else {
#pragma unroll
                    for (int c = 0; c < 32; ++c)
                        if (c < len) dst[c] = uint8_t((w[c / 4] >> (8 * (c % 4))) & 0xFF);
                }
            } else {
                uint32_t w[4];
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    float q[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) q[e] = __fmul_rn(tile[8 * g + e][t], inv);
                    w[g] = special ? 0u : e2m1x8(q);
                }
                uint8_t* dst = payload + r * ldp + kb * 16;
                if (len == 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
                    *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
                } else {
#pragma unroll
                    for (int c = 0; c < 32; c += 2) {
                        if (c >= len) continue;
                        const uint8_t byte = uint8_t((w[c / 8] >> (4 * (c % 8))) & 0xFF);
                        if (c + 1 < len) dst[c / 2] = byte;
                        else dst[c / 2] = uint8_t((dst[c / 2] & 0xF0) | (byte & 0x0F));
                    }
                }
            }
        }
        __syncthreads();  // the next tile overwrites the staging
    }
}

// ---- quantise both ways, with the GELU (or its gradient) applied on the way in --
// One read of S[rows, cols] (unit stride along cols, row pitch ld) gives the
// MX planes blocked along cols ("row planes", the operand [rows, cols]) and the
// planes blocked along rows ("column planes", the operand [cols, rows]) - the
// two operands an MLP layer's forward and weight-gradient contractions take
// from one activation.  S is x, gelu(x), or x * gelu'(h) with h the
// pre-activation and x the upstream gradient: the same functions, with the same
// operand order, as the elementwise kernels, so the planes are bit-identical to
// those of the unfused sequence.
// A CTA stages 32 x 128 tiles in which each 32-element row block is padded to
// 36 floats: float4 reads along a row block (the row planes) and scalar reads
// down a column (the column planes) are then both free of bank conflicts.  Two
// stages: cp.async brings the CTA's next tile (and its h tile) while the
// current one is transformed in place and quantised.
constexpr int kDualRows = 32;
constexpr int kDualCols = 128;
constexpr int kDualPitch = 4 * 36;  // floats per staged row

template <int XF>
__device__ __forceinline__ float4 dual_transform(float4 x, float4 h) {
    if (XF == SW_XF_GELU) return make_float4(gelu(x.x), gelu(x.y), gelu(x.z), gelu(x.w));
    if (XF == SW_XF_GELU_GRAD)
        return make_float4(x.x * gelu_grad(h.x), x.y * gelu_grad(h.y), x.z * gelu_grad(h.z), x.w * gelu_grad(h.w));
    return x;
}


constexpr int kDualTileFloats = kDualRows * kDualPitch;

// One block's packed payload: 16-byte stores where the destination allows.
__device__ __forceinline__ void dual_store32(uint8_t* dst, const uint32_t (&w)[8]) {
    if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
        reinterpret_cast<uint4*>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
    } else {
        for (int c = 0; c < 32; ++c) dst[c] = uint8_t((w[c / 4] >> (8 * (c % 4))) & 0xFF);
    }
}
__device__ __forceinline__ void dual_store16(uint8_t* dst, const uint32_t (&w)[4]) {
    if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
        for (int c = 0; c < 16; ++c) dst[c] = uint8_t((w[c / 4] >> (8 * (c % 4))) & 0xFF);
    }
}

template <int XF>
constexpr int dual_min_blocks() { return XF == SW_XF_GELU_GRAD ? 3 : 6; }

template <int FMT, int XF>
__global__ void __launch_bounds__(kDualCols, dual_min_blocks<XF>())
    quantize_dual(const float* __restrict__ x, const float* __restrict__ h, int64_t rows, int64_t cols, int64_t ld,
                  uint8_t* __restrict__ pr, int64_t ldpr, uint8_t* __restrict__ sr, int lr, int64_t ldsr,
                  uint8_t* __restrict__ pc, int64_t ldpc, uint8_t* __restrict__ sc, int lc, int64_t ldsc) {
    extern __shared__ __align__(16) float dsm[];
    // stage s: x tile at dsm + s * kDualTileFloats, h tile (GELU') after both x tiles
    pdl_enter();
    const int t = threadIdx.x;
    const int64_t ctiles = cols / kDualCols;
    const int64_t ntiles = (rows / kDualRows) * ctiles;
    const int c4 = t & 31;
    const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(dsm));
    auto issue = [&](int64_t tt, int stage) {
        const int64_t i0 = (tt / ctiles) * kDualRows;
        const int64_t j0 = (tt - (tt / ctiles) * ctiles) * kDualCols;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int r = (t >> 5) + 4 * k;
            const int64_t off = (i0 + r) * ld + j0 + 4 * c4;
            const int so = stage * kDualTileFloats + r * kDualPitch + (c4 >> 3) * 36 + (c4 & 7) * 4;
            cp_async16(sbase + 4u * so, x + off);
            if (XF == SW_XF_GELU_GRAD) cp_async16(sbase + 4u * (2 * kDualTileFloats + so), h + off);
        }
    };
    int stage = 0;
    if (int64_t(blockIdx.x) < ntiles) issue(blockIdx.x, 0);
    cp_async_commit();
    for (int64_t tt = blockIdx.x; tt < ntiles; tt += gridDim.x, stage ^= 1) {
        const int64_t i0 = (tt / ctiles) * kDualRows;
        const int64_t j0 = (tt - (tt / ctiles) * ctiles) * kDualCols;
        if (tt + gridDim.x < ntiles) issue(tt + gridDim.x, stage ^ 1);
        cp_async_commit();
        cp_async_wait<1>();  // this thread's copies of tile tt have landed
        float* tile = dsm + stage * kDualTileFloats;
        if (XF != SW_XF_NONE) {
            const float* htile = dsm + (2 + stage) * kDualTileFloats;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int r = (t >> 5) + 4 * k;
                const int so = r * kDualPitch + (c4 >> 3) * 36 + (c4 & 7) * 4;
                float4* q = reinterpret_cast<float4*>(tile + so);
                const float4 v = *q;
                const float4 hv = XF == SW_XF_GELU_GRAD ? *reinterpret_cast<const float4*>(htile + so) : v;
                *q = dual_transform<XF>(v, hv);
            }
        }
        __syncthreads();
        if (pr) {
            const int row = t >> 2, blk = t & 3;
            const float4* src = reinterpret_cast<const float4*>(&tile[row * kDualPitch + blk * 36]);
            float m = 0.0f;
#pragma unroll
            for (int g = 0; g < 8; ++g) {
                const float4 v = src[g];
                m = max_nan_abs(max_nan_abs(max_nan_abs(max_nan_abs(m, v.x), v.y), v.z), v.w);
            }
            uint8_t scb;
            float inv;
            bool special;
            block_scale<FMT>(__float_as_uint(m), scb, inv, special);
            const int64_t r = i0 + row, kb = (j0 >> 5) + blk;
            sr[scale_offset(lr, r, kb, cols >> 5, ldsr)] = scb;
            if (FMT == SW_MX_E4M3) {
                uint32_t w[8];
#pragma unroll
                for (int g = 0; g < 8; ++g) {
                    const float4 v = src[g];
                    w[g] = special ? 0u
                                   : e4m3x4(__fmul_rn(v.x, inv), __fmul_rn(v.y, inv), __fmul_rn(v.z, inv),
                                            __fmul_rn(v.w, inv));
                }
                dual_store32(pr + r * ldpr + kb * 32, w);
            } else {
                uint32_t w[4];
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    const float4 a = src[2 * g], b = src[2 * g + 1];
                    const float q[8] = {__fmul_rn(a.x, inv), __fmul_rn(a.y, inv), __fmul_rn(a.z, inv),
                                        __fmul_rn(a.w, inv), __fmul_rn(b.x, inv), __fmul_rn(b.y, inv),
                                        __fmul_rn(b.z, inv), __fmul_rn(b.w, inv)};
                    w[g] = special ? 0u : e2m1x8(q);
                }
                dual_store16(pr + r * ldpr + kb * 16, w);
            }
        }
        if (pc) {
            const float* src = &tile[(t >> 5) * 36 + (t & 31)];
            float m = 0.0f;
#pragma unroll
            for (int i = 0; i < 32; ++i) m = max_nan_abs(m, src[i * kDualPitch]);
            uint8_t scb;
            float inv;
            bool special;
            block_scale<FMT>(__float_as_uint(m), scb, inv, special);
            const int64_t r = j0 + t, kb = i0 >> 5;
            sc[scale_offset(lc, r, kb, rows >> 5, ldsc)] = scb;
            if (FMT == SW_MX_E4M3) {
                uint32_t w[8];
#pragma unroll
                for (int g = 0; g < 8; ++g)
                    w[g] = special ? 0u
                                   : e4m3x4(__fmul_rn(src[(4 * g) * kDualPitch], inv),
                                            __fmul_rn(src[(4 * g + 1) * kDualPitch], inv),
                                            __fmul_rn(src[(4 * g + 2) * kDualPitch], inv),
                                            __fmul_rn(src[(4 * g + 3) * kDualPitch], inv));
                dual_store32(pc + r * ldpc + kb * 32, w);
            } else {
                uint32_t w[4];
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    float q[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) q[e] = __fmul_rn(src[(8 * g + e) * kDualPitch], inv);
                    w[g] = special ? 0u : e2m1x8(q);
                }
                dual_store16(pc + r * ldpc + kb * 16, w);
            }
        }
        __syncthreads();  // the next iteration's copies overwrite this stage
    }
    cp_async_wait<0>();
}

// ---- dequantise ----------------------------------------------------------------
__device__ __forceinline__ float decode_e4m3(uint32_t c) {
    const uint32_t s = (c >> 7) & 1, f = (c >> 3) & 15, m = c & 7;
    float v;
    if (f == 15 && m == 7) return __uint_as_float(0x7FC00000u);
    if (f == 0) v = float(m) * 0.001953125f;  // m * 2^-9
    else v = __uint_as_float(((f + 120u) << 23) | (m << 20));
    return s ? -v : v;
}

__device__ __forceinline__ float decode_e2m1(uint32_t c) {
    const uint32_t s = (c >> 3) & 1, f = (c >> 1) & 3, m = c & 1;
    float v;
    if (f == 0) v = m ? 0.5f : 0.0f;
    else v = __uint_as_float(((f + 126u) << 23) | (m << 22));
    return s ? -v : v;
}

__device__ __forceinline__ float pow2_scale(uint32_t sc) {
    // 2^(sc-127); sc == 0 is the binary32 subnormal 2^-127.
    return sc == 0 ? __uint_as_float(0x00400000u) : __uint_as_float(sc << 23);
}

template <int FMT>
__global__ void __launch_bounds__(256) dequantize_kernel(const uint8_t* __restrict__ payload, int64_t ldp,
                                                         const uint8_t* __restrict__ scales, int layout,
                                                         int64_t lds, int64_t rows, int64_t cols,
                                                         float* __restrict__ out, int64_t ldo) {
    pdl_enter();
    const int64_t kblocks = (cols + 31) / 32;
    const int64_t groups = (cols + 7) / 8;  // 8 elements per thread
    const int64_t total = rows * groups;
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < total; t += stride) {
        const int64_t r = t / groups;
        const int64_t c0 = (t % groups) * 8;
        const uint8_t sc = scales[scale_offset(layout, r, c0 / 32, kblocks, lds)];
        const float scale = pow2_scale(sc);
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int64_t c = c0 + i;
            if (c >= cols) { v[i] = 0.0f; continue; }
            uint32_t code;
            if (FMT == SW_MX_E4M3) code = payload[r * ldp + c];
            else code = (payload[r * ldp + c / 2] >> ((c & 1) * 4)) & 0xF;
            const float e = FMT == SW_MX_E4M3 ? decode_e4m3(code) : decode_e2m1(code);
            v[i] = sc == 0xFF ? __uint_as_float(0x7FC00000u) : __fmul_rn(e, scale);
        }
        float* dst = out + r * ldo + c0;
        if (c0 + 8 <= cols && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
            reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
            reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
        } else {
            for (int i = 0; i < 8 && c0 + i < cols; ++i) dst[i] = v[i];
        }
    }
}

int sm_count_mx() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        cudaGetLastError();
        sms = 148;
    }
    return sms;
}

int grid_for(int64_t items, int threads) {
    const int64_t blocks = (items + threads - 1) / threads;
    return (int)std::max<int64_t>(1, std::min<int64_t>(blocks, int64_t(sm_count_mx()) * 16));
}

// ---- quantise: any hierarchical view, through a carrier swizzle ---------------
// The source is a two-mode view lowered to leaves (first leaf fastest, as in
// sw_reduce_plan): mode 0 gives the row, mode 1 the quantised axis.  A warp
// takes one 32-block: lane i walks element 32 kb + i of row r to its carrier
// flat index (leaf decomposition), through the swizzle, and the block's amax is
// a warp reduction.  Every address is checked against the carrier size before
// it is read; one outside (which the host's range check excludes) reads as NaN
// and records SW_ERR_INVALID in the device error word.
struct ViewLeaves {
    int rank;
    int64_t shape[SW_MAX_LEAVES];
    int64_t stride[SW_MAX_LEAVES];
};

struct ViewPlan {
    int64_t offset;
    int64_t x_size;
    ViewLeaves rows, cols;
    int swz_rank;
    int swz_bits[SW_MAX_SWIZZLE];
    int swz_base[SW_MAX_SWIZZLE];
    int swz_shift[SW_MAX_SWIZZLE];
};

__device__ __forceinline__ int64_t leaf_offset(const ViewLeaves& l, int64_t i) {
    int64_t off = 0;
#pragma unroll 1
    for (int k = 0; k < l.rank; ++k) {
        const int64_t c = i % l.shape[k];
        i /= l.shape[k];
        off += c * l.stride[k];
    }
    return off;
}

// The carrier swizzle of src/strideweave/core/swizzle.py:107-117, stage by stage.
__device__ __forceinline__ int64_t view_swizzle(const ViewPlan& p, int64_t f) {
#pragma unroll
    for (int i = 0; i < SW_MAX_SWIZZLE; ++i) {
        if (i < p.swz_rank) {
            const int64_t mask = (int64_t(1) << p.swz_bits[i]) - 1;
            if (p.swz_shift[i] > 0) f ^= ((f >> (p.swz_base[i] + p.swz_shift[i])) & mask) << p.swz_base[i];
            else f ^= ((f >> p.swz_base[i]) & mask) << (p.swz_base[i] - p.swz_shift[i]);
        }
    }
    return f;
}

// One element of a view at carrier flat index f (before the swizzle).  An
// address outside the carrier (which the host's range check excludes) reads
// as NaN and records SW_ERR_INVALID.
__device__ __forceinline__ float view_load(const float* __restrict__ x, const ViewPlan& p, int64_t f) {
    f = view_swizzle(p, f);
    if (f >= 0 && f < p.x_size) return __ldcs(x + f);
    report_device_error(SW_ERR_INVALID);
    return __int_as_float(0x7FC00000);
}

// Quantises block kb of row r held one element per lane (lane i: column
// c = 32 kb + i, `live` when c < cols): the warp's amax, the scale byte, the
// lane's code; E2M1 lanes pair up into bytes.
template <int FMT>
__device__ __forceinline__ void quantize_lane_block(float v, bool live, int lane, int64_t r, int64_t kb, int64_t c,
                                                    int64_t cols, int64_t kblocks, uint8_t* __restrict__ payload,
                                                    int64_t ldp, uint8_t* __restrict__ scales, int layout,
                                                    int64_t lds) {
    const uint32_t amax = __reduce_max_sync(0xFFFFFFFFu, __float_as_uint(v) & 0x7FFFFFFFu);
    uint8_t sc;
    float inv;
    bool special;
    block_scale<FMT>(amax, sc, inv, special);
    if (lane == 0) scales[scale_offset(layout, r, kb, kblocks, lds)] = sc;
    const float q = special ? 0.0f : __fmul_rn(v, inv);
    if (FMT == SW_MX_E4M3) {
        const uint32_t code = e4m3x4(q, 0.0f, 0.0f, 0.0f) & 0xFF;
        if (live) payload[r * ldp + c] = uint8_t(code);
    } else {
        float eight[8] = {q, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
        const uint32_t nib = e2m1x8(eight) & 0xF;
        const uint32_t hi = __shfl_down_sync(0xFFFFFFFFu, nib, 1);
        if (live && (lane & 1) == 0) {
            uint8_t* dst = payload + r * ldp + c / 2;
            if (c + 1 < cols) *dst = uint8_t(nib | (hi << 4));
            else *dst = uint8_t((*dst & 0xF0) | nib);  // odd row length: the high nibble is not ours
        }
    }
}

template <int FMT>
__global__ void __launch_bounds__(256) quantize_view(const float* __restrict__ x, const ViewPlan p, int64_t rows,
                                                     int64_t cols, uint8_t* __restrict__ payload, int64_t ldp,
                                                     uint8_t* __restrict__ scales, int layout, int64_t lds) {
    pdl_enter();
    const int64_t kblocks = (cols + 31) / 32;
    const int64_t units = rows * kblocks;
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t u = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; u < units; u += nwarps) {
        const int64_t r = u / kblocks;
        const int64_t kb = u - r * kblocks;
        const int64_t c = kb * 32 + lane;
        const bool live = c < cols;
        const float v = live ? view_load(x, p, p.offset + leaf_offset(p.rows, r) + leaf_offset(p.cols, c)) : 0.0f;
        quantize_lane_block<FMT>(v, live, lane, r, kb, c, cols, kblocks, payload, ldp, scales, layout, lds);
    }
}

// The same, for views whose quantised mode starts with a leaf of a whole
// number of 32-blocks (a tile row, a contiguous run): a warp walks 16
// consecutive blocks of one row, lane i at run offset + i * stride of that
// leaf, and steps from block to block with an odometer over the mode's
// leaves instead of decomposing each element's ordinal.
constexpr int kViewSegment = 16;  // blocks a warp walks per unit

template <int FMT>
__global__ void __launch_bounds__(256) quantize_view_runs(const float* __restrict__ x, const ViewPlan p, int64_t rows,
                                                          int64_t cols, uint8_t* __restrict__ payload, int64_t ldp,
                                                          uint8_t* __restrict__ scales, int layout, int64_t lds) {
    pdl_enter();
    const int64_t kblocks = cols / 32;
    const int64_t segs = (kblocks + kViewSegment - 1) / kViewSegment;
    const int64_t units = rows * segs;
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    const int64_t s0 = p.cols.stride[0], e0 = p.cols.shape[0];
    for (int64_t u = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; u < units; u += nwarps) {
        const int64_t r = u / segs;
        const int64_t kb0 = (u - r * segs) * kViewSegment;
        const int64_t kb1 = min(kblocks, kb0 + kViewSegment);
        const int64_t row = p.offset + leaf_offset(p.rows, r);
        // odometer of the quantised mode at element 32 kb0 (lane-uniform)
        int64_t key[SW_MAX_LEAVES];
        int64_t col = 0, o = kb0 * 32;
#pragma unroll
        for (int k = 0; k < SW_MAX_LEAVES; ++k) {
            if (k >= p.cols.rank) break;
            key[k] = o % p.cols.shape[k];
            o /= p.cols.shape[k];
            col += key[k] * p.cols.stride[k];
        }
        // every block's element in flight first, then the folds
        float v[kViewSegment];
#pragma unroll
        for (int b = 0; b < kViewSegment; ++b) {
            if (kb0 + b >= kb1) break;
            v[b] = view_load(x, p, row + col + lane * s0);
            // 32 elements further along the mode: leaf 0 never splits a block
            key[0] += 32;
            col += 32 * s0;
            if (key[0] == e0) {
                key[0] = 0;
                col -= e0 * s0;
#pragma unroll
                for (int k = 1; k < SW_MAX_LEAVES; ++k) {
                    if (k >= p.cols.rank) break;
                    key[k] += 1;
                    col += p.cols.stride[k];
                    if (key[k] < p.cols.shape[k]) break;
                    col -= p.cols.shape[k] * p.cols.stride[k];
                    key[k] = 0;
                }
            }
        }
#pragma unroll
        for (int b = 0; b < kViewSegment; ++b) {
            if (kb0 + b >= kb1) break;
            quantize_lane_block<FMT>(v[b], true, lane, r, kb0 + b, (kb0 + b) * 32 + lane, cols, kblocks, payload,
                                     ldp, scales, layout, lds);
        }
    }
}

// The vectorised walk: the quantised mode starts with a unit-stride leaf of
// whole 32-blocks, every other stride and the offset are multiples of 4, and
// the swizzle (if any) keeps 16-byte chunks whole, so each lane reads four
// consecutive elements with one 16-byte load.  A warp takes 32 consecutive
// blocks of one row: lane j decomposes block j's offset once, and for each of
// eight loads lane L takes block 4 s + L / 8 (eight lanes a block) by a
// shuffle.  A block's amax is a three-step shuffle over its eight lanes; each
// lane stores its four codes (E2M1: two bytes) and the block's first lane its
// scale byte.
constexpr int kViewVecSegment = 32;
#ifndef SW_VIEW_TILES
#define SW_VIEW_TILES 1  // the tile-ordered walk for tiled sources
#endif
#ifndef SW_VIEW_STAGED
#define SW_VIEW_STAGED 1  // the shared-memory staged walk for contiguous tiles
#endif
#ifndef SW_VIEW_TILES_MINB
#define SW_VIEW_TILES_MINB 3  // resident CTAs per SM the tile walk is compiled for
#endif

template <int FMT>
__global__ void __launch_bounds__(256) quantize_view_vec(const float* __restrict__ x, const ViewPlan p, int64_t rows,
                                                         int64_t cols, uint8_t* __restrict__ payload, int64_t ldp,
                                                         uint8_t* __restrict__ scales, int layout, int64_t lds) {
    pdl_enter();
    const int64_t kblocks = cols / 32;
    const int64_t segs = (kblocks + kViewVecSegment - 1) / kViewVecSegment;
    const int64_t units = rows * segs;
    const int lane = threadIdx.x & 31;
    const int sub = lane & 7;  // the lane's four elements: 4 sub .. 4 sub + 3 of its block
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t u = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; u < units; u += nwarps) {
        const int64_t r = u / segs;
        const int64_t kb0 = (u - r * segs) * kViewVecSegment;
        const int64_t row = p.offset + leaf_offset(p.rows, r);
        const int64_t mine = kb0 + lane < kblocks ? leaf_offset(p.cols, (kb0 + lane) * 32) : 0;
        float4 q[kViewVecSegment / 4];
#pragma unroll
        for (int s = 0; s < kViewVecSegment / 4; ++s) {
            const int b = 4 * s + (lane >> 3);
            const int64_t boff = __shfl_sync(0xFFFFFFFFu, mine, b);
            q[s] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (kb0 + b < kblocks) {
                int64_t f = view_swizzle(p, row + boff + 4 * sub);
                if (f >= 0 && f + 3 < p.x_size) {
                    q[s] = __ldcs(reinterpret_cast<const float4*>(x + f));
                } else {
                    report_device_error(SW_ERR_INVALID);
                    const float nan = __int_as_float(0x7FC00000);
                    q[s] = make_float4(nan, nan, nan, nan);
                }
            }
        }
#pragma unroll
        for (int s = 0; s < kViewVecSegment / 4; ++s) {
            const int64_t kb = kb0 + 4 * s + (lane >> 3);
            const bool live = kb < kblocks;  // uniform over the block's eight lanes
            uint32_t amax = max(max(__float_as_uint(q[s].x) & 0x7FFFFFFFu, __float_as_uint(q[s].y) & 0x7FFFFFFFu),
                                max(__float_as_uint(q[s].z) & 0x7FFFFFFFu, __float_as_uint(q[s].w) & 0x7FFFFFFFu));
            amax = max(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
            amax = max(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
            amax = max(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 4));
            uint8_t sc;
            float inv;
            bool special;
            block_scale<FMT>(amax, sc, inv, special);
            if (!live) continue;
            if (sub == 0) scales[scale_offset(layout, r, kb, kblocks, lds)] = sc;
            const float a = special ? 0.0f : __fmul_rn(q[s].x, inv), b = special ? 0.0f : __fmul_rn(q[s].y, inv);
            const float c = special ? 0.0f : __fmul_rn(q[s].z, inv), d = special ? 0.0f : __fmul_rn(q[s].w, inv);
            uint8_t* dst = payload + r * ldp;
            if (FMT == SW_MX_E4M3) {
                *reinterpret_cast<uint32_t*>(dst + kb * 32 + 4 * sub) = e4m3x4(a, b, c, d);
            } else {
                const float e[8] = {a, b, c, d, 0.0f, 0.0f, 0.0f, 0.0f};
                *reinterpret_cast<uint16_t*>(dst + kb * 16 + 2 * sub) = uint16_t(e2m1x8(e) & 0xFFFF);
            }
        }
    }
}

// The vectorised walk for tiled sources, whose next row lies closer in memory
// than the next run of the quantised mode (a 128 x 32 tile stores its rows'
// 32-blocks back to back).  The unit is one block of 32 consecutive rows of
// the first row leaf: each of the warp's eight 16-byte loads covers one block
// of four adjacent rows (eight lanes a row), so a warp reads 32 x 128 bytes
// that the tile holds contiguously.  Units run row group first, then block,
// then the outer rows, which is the tile order of memory: consecutive warps
// read consecutive tiles.  Conditions as for quantize_view_vec, plus a first
// row leaf of whole 32-row groups.
template <int FMT>
__global__ void __launch_bounds__(256, SW_VIEW_TILES_MINB) quantize_view_tiles(const float* __restrict__ x, const ViewPlan p, int64_t rows,
                                                           int64_t cols, uint8_t* __restrict__ payload, int64_t ldp,
                                                           uint8_t* __restrict__ scales, int layout, int64_t lds) {
    pdl_enter();
    const int64_t kblocks = cols / 32;
    const int64_t shape0 = p.rows.shape[0];
    const int64_t groups0 = shape0 / 32;  // 32-row groups along the first row leaf
    const int64_t units = (rows / 32) * kblocks;
    const int64_t stride0 = p.rows.stride[0];
    const int lane = threadIdx.x & 31;
    const int sub = lane & 7;   // the lane's four elements: 4 sub .. 4 sub + 3 of its block
    const int rsub = lane >> 3; // the lane's row within each group of four
    // each warp walks a contiguous run of units; its position is decomposed
    // once and then advanced as an odometer (row group, block, outer rows)
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t per = (units + nwarps - 1) / nwarps;
    int64_t u = warp * per;
    const int64_t u_end = min(units, u + per);
    if (u >= u_end) return;
    int64_t a = u % groups0;
    const int64_t rest = u / groups0;
    int64_t kb = rest % kblocks;
    int64_t hi = rest / kblocks;
    int64_t rowoff = p.offset + leaf_offset(p.rows, hi * shape0);
    int64_t key[SW_MAX_LEAVES];
    int64_t coloff = 0;
    {
        int64_t o = kb * 32;
#pragma unroll
        for (int k = 0; k < SW_MAX_LEAVES; ++k) {
            if (k >= p.cols.rank) break;
            key[k] = o % p.cols.shape[k];
            o /= p.cols.shape[k];
            coloff += key[k] * p.cols.stride[k];
        }
    }
    for (; u < u_end; ++u) {
        const int64_t r0 = hi * shape0 + a * 32;
        // rows r0 + 4 s + rsub: first-leaf coordinate a * 32 + 4 s + rsub, the outer leaves fixed by hi
        const int64_t base = rowoff + (a * 32 + rsub) * stride0 + coloff + 4 * sub;
        float4 q[8];
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const int64_t f = view_swizzle(p, base + int64_t(4 * s) * stride0);
            if (f >= 0 && f + 3 < p.x_size) {
                q[s] = __ldcs(reinterpret_cast<const float4*>(x + f));
            } else {
                report_device_error(SW_ERR_INVALID);
                const float nan = __int_as_float(0x7FC00000);
                q[s] = make_float4(nan, nan, nan, nan);
            }
        }
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const int64_t r = r0 + 4 * s + rsub;
            uint32_t amax = max(max(__float_as_uint(q[s].x) & 0x7FFFFFFFu, __float_as_uint(q[s].y) & 0x7FFFFFFFu),
                                max(__float_as_uint(q[s].z) & 0x7FFFFFFFu, __float_as_uint(q[s].w) & 0x7FFFFFFFu));
            amax = max(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
            amax = max(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
            amax = max(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 4));
            uint8_t sc;
            float inv;
            bool special;
            block_scale<FMT>(amax, sc, inv, special);
            if (sub == 0) scales[scale_offset(layout, r, kb, kblocks, lds)] = sc;
            const float e0 = special ? 0.0f : __fmul_rn(q[s].x, inv), e1 = special ? 0.0f : __fmul_rn(q[s].y, inv);
            const float e2 = special ? 0.0f : __fmul_rn(q[s].z, inv), e3 = special ? 0.0f : __fmul_rn(q[s].w, inv);
            uint8_t* dst = payload + r * ldp;
            if (FMT == SW_MX_E4M3) {
                *reinterpret_cast<uint32_t*>(dst + kb * 32 + 4 * sub) = e4m3x4(e0, e1, e2, e3);
            } else {
                const float e[8] = {e0, e1, e2, e3, 0.0f, 0.0f, 0.0f, 0.0f};
                *reinterpret_cast<uint16_t*>(dst + kb * 16 + 2 * sub) = uint16_t(e2m1x8(e) & 0xFFFF);
            }
        }
        // next unit: row group, then block (an odometer over the quantised
        // mode's leaves, 32 elements a step; leaf 0 holds whole blocks), then
        // the outer rows
        if (++a < groups0) continue;
        a = 0;
        if (++kb < kblocks) {
            key[0] += 32;
            coloff += 32 * p.cols.stride[0];
            if (key[0] == p.cols.shape[0]) {
                key[0] = 0;
                coloff -= p.cols.shape[0] * p.cols.stride[0];
#pragma unroll
                for (int k = 1; k < SW_MAX_LEAVES; ++k) {
                    if (k >= p.cols.rank) break;
                    key[k] += 1;
                    coloff += p.cols.stride[k];
                    if (key[k] < p.cols.shape[k]) break;
                    coloff -= p.cols.shape[k] * p.cols.stride[k];
                    key[k] = 0;
                }
            }
            continue;
        }
        kb = 0;
        coloff = 0;
#pragma unroll
        for (int k = 0; k < SW_MAX_LEAVES; ++k) key[k] = 0;
        ++hi;
        if (u + 1 < u_end) rowoff = p.offset + leaf_offset(p.rows, hi * shape0);
    }
}

// The staged walk for tiled sources whose tiles are contiguous: the first row
// leaf abuts the quantised mode's first leaf (row stride = run length), so a
// tile of E_r rows x E_c columns (E_c whole blocks) fills one contiguous
// E_r * E_c-float range, which one bulk copy brings into shared memory.  The
// carrier swizzle, when there is one, permutes only inside a tile (the host
// checks that every bit it reads or writes lies below the tile's alignment),
// so the tile is copied as it lies and the swizzle is applied to shared-memory
// offsets.  A thread then quantises one whole 32-block from shared memory
// (eight 16-byte reads, the amax, the scale, 32 products and their packed
// codes): a few instructions per element instead of the cross-lane amax and
// the per-lane address arithmetic of the register walks.  A ring of
// kStagedBufs buffers per CTA: the next kStagedBufs - 1 tiles are in flight
// while one is quantised.
constexpr int kStagedThreads = 128;
#ifndef SW_VIEW_STAGED_BUFS
#define SW_VIEW_STAGED_BUFS 2  // tiles in flight or in use per CTA
#endif
constexpr int kStagedBufs = SW_VIEW_STAGED_BUFS;
#ifndef SW_VIEW_STAGED_MINB
#define SW_VIEW_STAGED_MINB 6  // resident CTAs per SM (85 registers; measured best of 1, 4, 6, 7)
#endif
constexpr int64_t kStagedMaxTileFloats = 8192;  // 32 KiB per buffer

__device__ __forceinline__ int swizzle_local(const ViewPlan& p, int f) {
#pragma unroll
    for (int i = 0; i < SW_MAX_SWIZZLE; ++i) {
        if (i < p.swz_rank) {
            const int mask = (1 << p.swz_bits[i]) - 1;
            if (p.swz_shift[i] > 0) f ^= ((f >> (p.swz_base[i] + p.swz_shift[i])) & mask) << p.swz_base[i];
            else f ^= ((f >> p.swz_base[i]) & mask) << (p.swz_base[i] - p.swz_shift[i]);
        }
    }
    return f;
}

template <int FMT>
__global__ void __launch_bounds__(kStagedThreads, SW_VIEW_STAGED_MINB) quantize_view_staged(const float* __restrict__ x, const ViewPlan p,
                                                                       int64_t rows, int64_t cols,
                                                                       uint8_t* __restrict__ payload, int64_t ldp,
                                                                       uint8_t* __restrict__ scales, int layout,
                                                                       int64_t lds) {
    extern __shared__ __align__(128) float staged[];
    const int er = int(p.rows.shape[0]);
    const int ec = int(p.cols.shape[0]);
    const int tile = er * ec;       // floats per tile
    const int bpr = ec / 32;        // blocks per tile row
    const int64_t ncol = cols / ec;
    const int64_t ntiles = (rows / er) * ncol;
    const int64_t kblocks = cols / 32;
    const uint32_t sbase = ptx::smem_addr(staged);
    const uint32_t bar0 = sbase + uint32_t(kStagedBufs * tile) * 4u;  // one mbarrier per buffer, after the buffers
    if (threadIdx.x == 0) {
        for (int b = 0; b < kStagedBufs; ++b) ptx::mbar_init(bar0 + 8u * uint32_t(b), 1);
        ptx::fence_barrier_init();
    }
    __syncthreads();
    pdl_enter();
    // tile t: outer rows t / ncol, outer column group t % ncol, columns fastest
    // (consecutive tiles are consecutive in memory for a row-of-tiles layout)
    auto issue = [&](int64_t t, int buf) {
        const int64_t co = t % ncol, ro = t / ncol;
        const float* src = x + p.offset + leaf_offset(p.rows, ro * er) + leaf_offset(p.cols, co * ec);
        const uint32_t bar = bar0 + 8u * uint32_t(buf);
        ptx::mbar_arrive_expect_tx(bar, uint32_t(tile) * 4u);
        ptx::bulk_load(sbase + uint32_t(buf * tile) * 4u, src, uint32_t(tile) * 4u, bar);
    };
    const int64_t g = gridDim.x;
    int dsw[8];  // swizzled offsets of a block's eight 16-byte chunks from its start
#pragma unroll
    for (int c = 0; c < 8; ++c) dsw[c] = p.swz_rank > 0 ? swizzle_local(p, 4 * c) : 4 * c;
    uint32_t phases = 0u;   // bit b: parity of buffer b's next completion
    uint32_t pending = 0u;  // bit b: a copy into buffer b not yet waited for
    // the first kStagedBufs - 1 tiles of this CTA go out at once
    for (int b = 0; b + 1 < kStagedBufs; ++b) {
        const int64_t t = blockIdx.x + b * g;
        if (t < ntiles) {
            if (threadIdx.x == 0) issue(t, b);
            pending |= 1u << b;
        }
    }
    int k = 0;
    for (int64_t t = blockIdx.x; t < ntiles; t += g, ++k) {
        const int buf = k % kStagedBufs;
        // the buffer the copy kStagedBufs - 1 tiles ahead lands in was freed
        // by the barrier that ended the previous tile; order its readers'
        // accesses before the copy's writes
        const int nb = (k + kStagedBufs - 1) % kStagedBufs;
        const int64_t tn = t + int64_t(kStagedBufs - 1) * g;
        if (tn < ntiles) {
            if (threadIdx.x == 0) {
                ptx::fence_proxy_async_smem();
                issue(tn, nb);
            }
            pending |= 1u << nb;
        }
        const bool ok = ptx::mbar_wait(bar0 + 8u * uint32_t(buf), (phases >> buf) & 1u);
        phases ^= 1u << buf;
        pending &= ~(1u << buf);
        if (!__syncthreads_and(ok)) break;  // a copy that never landed: leave together
        const float* tb = staged + buf * tile;
        const int64_t co = t % ncol, ro = t / ncol;
        for (int item = threadIdx.x; item < er * bpr; item += kStagedThreads) {
            const int i = item / bpr, j = item - (item / bpr) * bpr;
            const int64_t r = ro * er + i, kb = co * bpr + j;
            const int f0 = i * ec + j * 32;
            // the swizzle is linear over the bits (each stage XORs shifted,
            // masked bits in) and f0 + 4 c = f0 ^ 4 c, so the block's eight
            // chunk offsets are swizzle(f0) ^ swizzle(4 c): one evaluation a block
            const int s0 = p.swz_rank > 0 ? swizzle_local(p, f0) : f0;
            float4 v[8];
            uint32_t amax = 0;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const int f = s0 ^ dsw[c];
                v[c] = *reinterpret_cast<const float4*>(tb + f);
                amax = max(amax, max(max(__float_as_uint(v[c].x) & 0x7FFFFFFFu, __float_as_uint(v[c].y) & 0x7FFFFFFFu),
                                     max(__float_as_uint(v[c].z) & 0x7FFFFFFFu, __float_as_uint(v[c].w) & 0x7FFFFFFFu)));
            }
            uint8_t sc;
            float inv;
            bool special;
            block_scale<FMT>(amax, sc, inv, special);
            scales[scale_offset(layout, r, kb, kblocks, lds)] = sc;
            float q[32];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                q[4 * c] = special ? 0.0f : __fmul_rn(v[c].x, inv);
                q[4 * c + 1] = special ? 0.0f : __fmul_rn(v[c].y, inv);
                q[4 * c + 2] = special ? 0.0f : __fmul_rn(v[c].z, inv);
                q[4 * c + 3] = special ? 0.0f : __fmul_rn(v[c].w, inv);
            }
            uint8_t* dst = payload + r * ldp;
            if (FMT == SW_MX_E4M3) {
                uint32_t w[8];
#pragma unroll
                for (int c = 0; c < 8; ++c) w[c] = e4m3x4(q[4 * c], q[4 * c + 1], q[4 * c + 2], q[4 * c + 3]);
                uint4* o = reinterpret_cast<uint4*>(dst + kb * 32);
                o[0] = make_uint4(w[0], w[1], w[2], w[3]);
                o[1] = make_uint4(w[4], w[5], w[6], w[7]);
            } else {
                uint32_t w[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) w[c] = e2m1x8(q + 8 * c);
                *reinterpret_cast<uint4*>(dst + kb * 16) = make_uint4(w[0], w[1], w[2], w[3]);
            }
        }
        __syncthreads();  // buffer `buf` may be refilled from the next tile on
    }
    // a CTA that left early still owns copies in flight: let them land (bounded)
    if (threadIdx.x == 0)
        for (int b = 0; b < kStagedBufs; ++b)
            if (pending & (1u << b)) ptx::mbar_wait(bar0 + 8u * uint32_t(b), (phases >> b) & 1u);
}

// Row-major E8M0 scales -> the SW_SCALES_TC128 atom placement (padding left at
// 127 by the caller), so a plane quantised with a row-major placement (rows or
// blocks not whole atoms) can feed the tensor-core contraction.
__global__ void __launch_bounds__(256) scales_to_tc128(const uint8_t* __restrict__ src, int64_t ld_src, int64_t rows,
                                                       int64_t kblocks, uint8_t* __restrict__ dst) {
    pdl_enter();
    const int64_t total = rows * kblocks;
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < total; t += stride) {
        const int64_t r = t / kblocks, kb = t - r * kblocks;
        dst[scale_offset(SW_SCALES_TC128, r, kb, kblocks, 0)] = src[r * ld_src + kb];
    }
}

}  // namespace
}  // namespace sw

extern "C" int64_t sw_mx_scale_index(int64_t r, int64_t kb, int64_t kblocks) {
    return sw::scale_offset(SW_SCALES_TC128, r, kb, kblocks, 0);
}

extern "C" int64_t sw_mx_scale_bytes_tc128(int64_t rows, int64_t kblocks) {
    if (rows <= 0 || kblocks <= 0) return 0;
    return ((rows + 127) / 128) * ((kblocks + 3) / 4) * 512;
}

extern "C" int sw_mx_quantize(int fmt, const float* x, int64_t rows, int64_t cols, int64_t ld_x_row,
                              int64_t ld_x_col, uint8_t* payload, int64_t ld_payload, uint8_t* scales,
                              int scale_layout, int64_t ld_scales, void* stream) {
    using namespace sw;
    if (fmt != SW_MX_E4M3 && fmt != SW_MX_E2M1) return fail(SW_ERR_INVALID, "sw_mx_quantize: unknown format %d", fmt);
    if (scale_layout != SW_SCALES_ROWMAJOR && scale_layout != SW_SCALES_TC128)
        return fail(SW_ERR_INVALID, "sw_mx_quantize: unknown scale layout %d", scale_layout);
    if (rows < 0 || cols < 0) return fail(SW_ERR_INVALID, "sw_mx_quantize: negative extent");
    if (rows == 0 || cols == 0) return ok();
    if (!x || !payload || !scales) return fail(SW_ERR_INVALID, "sw_mx_quantize: null pointer");
    const int64_t kblocks = (cols + 31) / 32;
    const int64_t min_ldp = fmt == SW_MX_E4M3 ? cols : (cols + 1) / 2;
    if (ld_payload < min_ldp) return fail(SW_ERR_INVALID, "sw_mx_quantize: payload pitch %lld < row bytes %lld",
                                          (long long)ld_payload, (long long)min_ldp);
    if (scale_layout == SW_SCALES_ROWMAJOR && ld_scales < kblocks)
        return fail(SW_ERR_INVALID, "sw_mx_quantize: scale pitch smaller than blocks per row");
    cudaStream_t s = (cudaStream_t)stream;
    if (scale_layout == SW_SCALES_TC128 && (rows % 128 != 0 || kblocks % 4 != 0)) {
        // padding slots of the atom placement read as 1.0 (byte 127)
        SW_CUDA_TRY(cudaMemsetAsync(scales, 127, (size_t)sw_mx_scale_bytes_tc128(rows, kblocks), s),
                    "scale padding fill");
    }
    const bool e4 = fmt == SW_MX_E4M3;
    if (ld_x_col == 1) {
        const int64_t items = rows * ((cols + kQuantSegment - 1) / kQuantSegment) * 32;  // a warp per segment
        const int grid = grid_for(items, 256);
        auto kernel = e4 ? quantize_rows<SW_MX_E4M3> : quantize_rows<SW_MX_E2M1>;
        SW_CUDA_TRY(launch_pdl(kernel, grid, 256, 0, s, x, rows, cols, ld_x_row, payload, ld_payload, scales,
                               scale_layout, ld_scales),
                    "quantize_rows launch");
    } else if (ld_x_row == 1 && rows % 4 == 0 && ld_x_col % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        const int64_t tiles = ((rows + kTileRows - 1) / kTileRows) * kblocks;
        const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(tiles, int64_t(sm_count_mx()) * 8));
        auto kernel = e4 ? quantize_cols_tiled<SW_MX_E4M3> : quantize_cols_tiled<SW_MX_E2M1>;
        SW_CUDA_TRY(launch_pdl(kernel, grid, kTileRows, 0, s, x, rows, cols, ld_x_col, payload, ld_payload, scales,
                               scale_layout, ld_scales),
                    "quantize_cols_tiled launch");
    } else {
        const int grid = grid_for(rows * kblocks, 256);
        auto kernel = e4 ? quantize_strided<SW_MX_E4M3> : quantize_strided<SW_MX_E2M1>;
        SW_CUDA_TRY(launch_pdl(kernel, grid, 256, 0, s, x, rows, cols, ld_x_row, ld_x_col, payload, ld_payload,
                               scales, scale_layout, ld_scales),
                    "quantize_strided launch");
    }
    SW_LAUNCH_CHECK("sw_mx_quantize launch");
    return ok();
}

extern "C" int sw_mx_quantize_view(int fmt, const sw_reduce_plan* view, const float* x, int64_t x_size,
                                   uint8_t* payload, int64_t ld_payload, uint8_t* scales, int scale_layout,
                                   int64_t ld_scales, void* stream) {
    using namespace sw;
    if (fmt != SW_MX_E4M3 && fmt != SW_MX_E2M1)
        return fail(SW_ERR_INVALID, "sw_mx_quantize_view: unknown format %d", fmt);
    if (scale_layout != SW_SCALES_ROWMAJOR && scale_layout != SW_SCALES_TC128)
        return fail(SW_ERR_INVALID, "sw_mx_quantize_view: unknown scale layout %d", scale_layout);
    if (!view) return fail(SW_ERR_INVALID, "sw_mx_quantize_view: null view");
    if (view->kept_rank < 0 || view->kept_rank > SW_MAX_LEAVES || view->reduced_rank < 1 ||
        view->reduced_rank > SW_MAX_LEAVES || view->swizzle_rank < 0 || view->swizzle_rank > SW_MAX_SWIZZLE)
        return fail(SW_ERR_INVALID, "sw_mx_quantize_view: leaf or swizzle rank out of range");
    ViewPlan p;
    std::memset(&p, 0, sizeof(p));
    p.offset = view->offset;
    p.x_size = x_size;
    int64_t rows = 1, cols = 1, lo = view->offset, hi = view->offset;
    auto lower = [&](int rank, const int64_t* shape, const int64_t* stride, ViewLeaves& out, int64_t& n) -> bool {
        out.rank = rank;
        for (int l = 0; l < rank; ++l) {
            if (shape[l] < 0) return false;
            out.shape[l] = shape[l] > 0 ? shape[l] : 1;
            out.stride[l] = stride[l];
            n *= shape[l];
            const int64_t span = (shape[l] > 0 ? shape[l] - 1 : 0) * stride[l];
            if (span < 0) lo += span; else hi += span;
        }
        return true;
    };
    if (!lower(view->kept_rank, view->kept_shape, view->kept_stride, p.rows, rows) ||
        !lower(view->reduced_rank, view->reduced_shape, view->reduced_stride, p.cols, cols))
        return fail(SW_ERR_INVALID, "sw_mx_quantize_view: negative extent");
    p.swz_rank = view->swizzle_rank;
    int top = -1;
    for (int i = 0; i < view->swizzle_rank; ++i) {
        p.swz_bits[i] = view->swizzle_bits[i];
        p.swz_base[i] = view->swizzle_base[i];
        p.swz_shift[i] = view->swizzle_shift[i];
        // the constraints of SwizzleStage (src/strideweave/core/swizzle.py:44-60)
        if (p.swz_bits[i] <= 0 || p.swz_base[i] < 0 || p.swz_shift[i] == 0 ||
            std::abs(p.swz_shift[i]) < p.swz_bits[i] || p.swz_bits[i] + p.swz_base[i] + std::abs(p.swz_shift[i]) > 62)
            return fail(SW_ERR_INVALID, "sw_mx_quantize_view: invalid swizzle stage %d", i);
        const int tgt = p.swz_shift[i] > 0 ? p.swz_base[i] : p.swz_base[i] - p.swz_shift[i];
        top = std::max(top, tgt + p.swz_bits[i] - 1);
    }
    if (rows == 0 || cols == 0) return ok();
    if (!x || !payload || !scales) return fail(SW_ERR_INVALID, "sw_mx_quantize_view: null pointer");
    if (lo < 0 || hi >= x_size)
        return fail(SW_ERR_INVALID, "sw_mx_quantize_view: view addresses [%lld, %lld] outside carrier of %lld elements",
                    (long long)lo, (long long)hi, (long long)x_size);
    if (top >= 0) {
        // a swizzle rewrites bits up to `top` only: addresses stay in their
        // aligned 2^(top+1) window, which must lie inside the carrier
        const int64_t win = int64_t(1) << (top + 1);
        if ((hi / win + 1) * win - 1 >= x_size)
            return fail(SW_ERR_INVALID, "sw_mx_quantize_view: swizzle may address past the carrier end");
    }
    const int64_t kblocks = (cols + 31) / 32;
    const int64_t min_ldp = fmt == SW_MX_E4M3 ? cols : (cols + 1) / 2;
    if (ld_payload < min_ldp)
        return fail(SW_ERR_INVALID, "sw_mx_quantize_view: payload pitch %lld < row bytes %lld", (long long)ld_payload,
                    (long long)min_ldp);
    if (scale_layout == SW_SCALES_ROWMAJOR && ld_scales < kblocks)
        return fail(SW_ERR_INVALID, "sw_mx_quantize_view: scale pitch smaller than blocks per row");
    // a plain strided matrix (one leaf per mode, positive strides, no
    // swizzle) whose rows or columns are contiguous takes the dense kernels:
    // the row walk, or the shared-memory tiles of a column-contiguous source
    if (p.swz_rank == 0 && p.rows.rank == 1 && p.cols.rank == 1 && p.rows.stride[0] > 0 && p.cols.stride[0] > 0 &&
        (p.cols.stride[0] == 1 || (p.rows.stride[0] == 1 && rows % 4 == 0 && p.cols.stride[0] % 4 == 0 &&
                                   ((reinterpret_cast<uintptr_t>(x + p.offset) & 15) == 0))))
        return sw_mx_quantize(fmt, x + p.offset, rows, cols, p.rows.stride[0], p.cols.stride[0], payload, ld_payload,
                              scales, scale_layout, ld_scales, stream);
    cudaStream_t s = (cudaStream_t)stream;
    if (scale_layout == SW_SCALES_TC128 && (rows % 128 != 0 || kblocks % 4 != 0))
        SW_CUDA_TRY(cudaMemsetAsync(scales, 127, (size_t)sw_mx_scale_bytes_tc128(rows, kblocks), s),
                    "scale padding fill");
    const bool runs = p.cols.shape[0] % 32 == 0;  // blocks lie inside runs of the first leaf
    // 16-byte loads: unit-stride runs, 4-aligned offsets, a swizzle that never
    // touches the two lowest index bits, 4-byte payload rows
    bool vec = runs && p.cols.stride[0] == 1 && p.offset % 4 == 0 && ld_payload % 4 == 0 &&
               (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(payload) & 3) == 0;
    for (int k = 0; k < p.rows.rank; ++k) vec = vec && p.rows.stride[k] % 4 == 0;
    for (int k = 1; k < p.cols.rank; ++k) vec = vec && p.cols.stride[k] % 4 == 0;
    for (int i = 0; i < p.swz_rank; ++i) vec = vec && p.swz_base[i] >= 2;
    // tiles that lie contiguously (the first row leaf abuts the first run) and
    // hold whole swizzle windows: staged through shared memory a tile at a time
    bool staged = SW_VIEW_STAGED && vec && p.rows.rank >= 1 && p.rows.stride[0] == p.cols.shape[0] &&
                  p.rows.shape[0] * p.cols.shape[0] <= kStagedMaxTileFloats &&
                  size_t(kStagedBufs) * size_t(p.rows.shape[0] * p.cols.shape[0]) * 4 + 8 * kStagedBufs <= 232448 &&
                  (reinterpret_cast<uintptr_t>(payload) & 15) == 0 && ld_payload % 16 == 0;
    if (staged) {
        int topbit = 1;  // 16-byte alignment of every tile
        for (int i = 0; i < p.swz_rank; ++i)
            topbit = std::max(topbit, p.swz_base[i] + std::abs(p.swz_shift[i]) + p.swz_bits[i] - 1);
        const int64_t align = int64_t(1) << (topbit + 1);
        staged = (p.rows.shape[0] * p.cols.shape[0]) % align == 0 && p.offset % align == 0;
        for (int k = 1; k < p.rows.rank; ++k) staged = staged && p.rows.stride[k] % align == 0;
        for (int k = 1; k < p.cols.rank; ++k) staged = staged && p.cols.stride[k] % align == 0;
    }
    if (staged) {
        const int64_t tile = p.rows.shape[0] * p.cols.shape[0];
        const int64_t ntiles = rows / p.rows.shape[0] * (cols / p.cols.shape[0]);
        const size_t smem = size_t(kStagedBufs * tile) * 4 + 8 * kStagedBufs;
        auto kernel = fmt == SW_MX_E4M3 ? quantize_view_staged<SW_MX_E4M3> : quantize_view_staged<SW_MX_E2M1>;
        SW_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
                    "quantize_view_staged smem");
        int per_sm = 0;  // every CTA resident: a persistent walk over the tiles
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kStagedThreads, smem) != cudaSuccess ||
            per_sm < 1) {
            cudaGetLastError();
            per_sm = 1;
        }
        const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(ntiles, int64_t(sm_count_mx()) * per_sm));
        SW_CUDA_TRY(launch_pdl(kernel, grid, kStagedThreads, smem, s, x, p, rows, cols, payload, ld_payload, scales,
                               scale_layout, ld_scales),
                    "quantize_view_staged launch");
        SW_LAUNCH_CHECK("sw_mx_quantize_view launch");
        return ok();
    }
    // tiled sources (the next row nearer than the next run): 32-row units in tile order
    const bool tiles = SW_VIEW_TILES && vec && p.rows.rank >= 1 && p.rows.shape[0] % 32 == 0 && p.cols.rank >= 2 &&
                       std::llabs(p.rows.stride[0]) < std::llabs(p.cols.stride[1]);
    const int64_t units = tiles  ? (rows / 32) * kblocks
                          : vec  ? rows * ((kblocks + kViewVecSegment - 1) / kViewVecSegment)
                          : runs ? rows * ((kblocks + kViewSegment - 1) / kViewSegment)
                                 : rows * kblocks;
    // the tile walk gives each warp a run of about four units (one
    // decomposition per run); the others a unit per warp and grid step
    const int grid = tiles ? grid_for(units * 8, 256) : grid_for(units * 32, 256);
    auto kernel = tiles  ? (fmt == SW_MX_E4M3 ? quantize_view_tiles<SW_MX_E4M3> : quantize_view_tiles<SW_MX_E2M1>)
                  : vec  ? (fmt == SW_MX_E4M3 ? quantize_view_vec<SW_MX_E4M3> : quantize_view_vec<SW_MX_E2M1>)
                  : runs ? (fmt == SW_MX_E4M3 ? quantize_view_runs<SW_MX_E4M3> : quantize_view_runs<SW_MX_E2M1>)
                         : (fmt == SW_MX_E4M3 ? quantize_view<SW_MX_E4M3> : quantize_view<SW_MX_E2M1>);
    SW_CUDA_TRY(launch_pdl(kernel, grid, 256, 0, s, x, p, rows, cols, payload, ld_payload, scales, scale_layout,
                           ld_scales),
                "quantize_view launch");
    SW_LAUNCH_CHECK("sw_mx_quantize_view launch");
    return ok();
}

extern "C" int sw_mx_scales_to_tc128(const uint8_t* src, int64_t ld_src, int64_t rows, int64_t kblocks, uint8_t* dst,
                                     void* stream) {
    using namespace sw;
    if (rows < 0 || kblocks < 0) return fail(SW_ERR_INVALID, "sw_mx_scales_to_tc128: negative extent");
    if (rows == 0 || kblocks == 0) return ok();
    if (!src || !dst) return fail(SW_ERR_INVALID, "sw_mx_scales_to_tc128: null pointer");
    if (ld_src < kblocks) return fail(SW_ERR_INVALID, "sw_mx_scales_to_tc128: source pitch smaller than blocks per row");
    cudaStream_t s = (cudaStream_t)stream;
    SW_CUDA_TRY(cudaMemsetAsync(dst, 127, (size_t)sw_mx_scale_bytes_tc128(rows, kblocks), s), "scale padding fill");
    const int grid = grid_for(rows * kblocks, 256);
    SW_CUDA_TRY(launch_pdl(scales_to_tc128, grid, 256, 0, s, src, ld_src, rows, kblocks, dst), "scales_to_tc128 launch");
    SW_LAUNCH_CHECK("sw_mx_scales_to_tc128 launch");
    return ok();
}

extern "C" int sw_mx_quantize_dual(int fmt, int transform, const float* x, const float* h, int64_t rows,
                                   int64_t cols, int64_t ld_x, uint8_t* payload_r, int64_t ld_payload_r,
                                   uint8_t* scales_r, int scale_layout_r, int64_t ld_scales_r, uint8_t* payload_c,
                                   int64_t ld_payload_c, uint8_t* scales_c, int scale_layout_c,
                                   int64_t ld_scales_c, void* stream) {
    using namespace sw;
    if (fmt != SW_MX_E4M3 && fmt != SW_MX_E2M1)
        return fail(SW_ERR_INVALID, "sw_mx_quantize_dual: unknown format %d", fmt);
    if (transform != SW_XF_NONE && transform != SW_XF_GELU && transform != SW_XF_GELU_GRAD)
        return fail(SW_ERR_INVALID, "sw_mx_quantize_dual: unknown transform %d", transform);
    if (rows < 0 || cols < 0) return fail(SW_ERR_INVALID, "sw_mx_quantize_dual: negative extent");
    if (rows == 0 || cols == 0) return ok();
    if (!x || (transform == SW_XF_GELU_GRAD && !h)) return fail(SW_ERR_INVALID, "sw_mx_quantize_dual: null input");
    if (!payload_r != !scales_r || !payload_c != !scales_c)
        return fail(SW_ERR_INVALID, "sw_mx_quantize_dual: a plane needs both its payload and its scales");
    if (!payload_r && !payload_c) return fail(SW_ERR_INVALID, "sw_mx_quantize_dual: no output plane");
    for (int layout : {scale_layout_r, scale_layout_c})
        if (layout != SW_SCALES_ROWMAJOR && layout != SW_SCALES_TC128)
            return fail(SW_ERR_INVALID, "sw_mx_quantize_dual: unknown scale layout %d", layout);
    if (ld_x < cols) return fail(SW_ERR_INVALID, "sw_mx_quantize_dual: row pitch smaller than a row");
    if (rows % kDualRows != 0 || cols % kDualCols != 0 || ld_x % 4 != 0 ||
        (reinterpret_cast<uintptr_t>(x) & 15) != 0 ||
        (transform == SW_XF_GELU_GRAD && (reinterpret_cast<uintptr_t>(h) & 15) != 0))
        return fail(SW_ERR_UNSUPPORTED,
                    "sw_mx_quantize_dual: needs rows %% 32 == 0, cols %% 128 == 0, a pitch of whole 16-byte "
                    "vectors and 16-byte aligned inputs (rows %lld, cols %lld, pitch %lld)",
                    (long long)rows, (long long)cols, (long long)ld_x);
    const bool e4 = fmt == SW_MX_E4M3;
    cudaStream_t s = (cudaStream_t)stream;
    // plane geometry: (operand rows, K) = (rows, cols) for the row planes, (cols, rows) for the column planes
    struct Plane { uint8_t* payload; int64_t ldp; uint8_t* scales; int layout; int64_t lds; int64_t n; int64_t k; };
    const Plane planes[2] = {{payload_r, ld_payload_r, scales_r, scale_layout_r, ld_scales_r, rows, cols},
                             {payload_c, ld_payload_c, scales_c, scale_layout_c, ld_scales_c, cols, rows}};
    for (const Plane& p : planes) {
        if (!p.payload) continue;
        const int64_t kblocks = p.k / 32;
        if (p.ldp < (e4 ? p.k : p.k / 2))
            return fail(SW_ERR_INVALID, "sw_mx_quantize_dual: payload pitch %lld < row bytes", (long long)p.ldp);
        if (p.layout == SW_SCALES_ROWMAJOR && p.lds < kblocks)
            return fail(SW_ERR_INVALID, "sw_mx_quantize_dual: scale pitch smaller than blocks per row");
        if (p.layout == SW_SCALES_TC128 && (p.n % 128 != 0 || kblocks % 4 != 0))
            SW_CUDA_TRY(cudaMemsetAsync(p.scales, 127, (size_t)sw_mx_scale_bytes_tc128(p.n, kblocks), s),
                        "scale padding fill");
    }
    const int64_t tiles = (rows / kDualRows) * (cols / kDualCols);
    const int per_sm = transform == SW_XF_GELU_GRAD ? 3 : 6;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(tiles, int64_t(sm_count_mx()) * per_sm));
    using Kernel = void (*)(const float*, const float*, int64_t, int64_t, int64_t, uint8_t*, int64_t, uint8_t*, int,
                            int64_t, uint8_t*, int64_t, uint8_t*, int, int64_t);
    Kernel kernel;
    if (transform == SW_XF_NONE) kernel = e4 ? quantize_dual<SW_MX_E4M3, SW_XF_NONE> : quantize_dual<SW_MX_E2M1, SW_XF_NONE>;
    else if (transform == SW_XF_GELU) kernel = e4 ? quantize_dual<SW_MX_E4M3, SW_XF_GELU> : quantize_dual<SW_MX_E2M1, SW_XF_GELU>;
    else kernel = e4 ? quantize_dual<SW_MX_E4M3, SW_XF_GELU_GRAD> : quantize_dual<SW_MX_E2M1, SW_XF_GELU_GRAD>;
    const size_t smem = size_t(transform == SW_XF_GELU_GRAD ? 4 : 2) * kDualTileFloats * sizeof(float);
    SW_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), "dual smem");
    SW_CUDA_TRY(launch_pdl(kernel, grid, kDualCols, smem, s, x, h, rows, cols, ld_x, payload_r, ld_payload_r, scales_r,
                           scale_layout_r, ld_scales_r, payload_c, ld_payload_c, scales_c, scale_layout_c,
                           ld_scales_c),
                "quantize_dual launch");
    SW_LAUNCH_CHECK("sw_mx_quantize_dual launch");
    return ok();
}

extern "C" int sw_mx_dequantize(int fmt, const uint8_t* payload, int64_t ld_payload, const uint8_t* scales,
                                int scale_layout, int64_t ld_scales, int64_t rows, int64_t cols, float* out,
                                int64_t ld_out, void* stream) {
    using namespace sw;
    if (fmt != SW_MX_E4M3 && fmt != SW_MX_E2M1) return fail(SW_ERR_INVALID, "sw_mx_dequantize: unknown format %d", fmt);
    if (scale_layout != SW_SCALES_ROWMAJOR && scale_layout != SW_SCALES_TC128)
        return fail(SW_ERR_INVALID, "sw_mx_dequantize: unknown scale layout %d", scale_layout);
    if (rows < 0 || cols < 0) return fail(SW_ERR_INVALID, "sw_mx_dequantize: negative extent");
    if (rows == 0 || cols == 0) return ok();
    if (!payload || !scales || !out) return fail(SW_ERR_INVALID, "sw_mx_dequantize: null pointer");
    if (ld_out < cols) return fail(SW_ERR_INVALID, "sw_mx_dequantize: output pitch smaller than a row");
    cudaStream_t s = (cudaStream_t)stream;
    const int grid = grid_for(rows * ((cols + 7) / 8), 256);
    auto kernel = fmt == SW_MX_E4M3 ? dequantize_kernel<SW_MX_E4M3> : dequantize_kernel<SW_MX_E2M1>;
    SW_CUDA_TRY(launch_pdl(kernel, grid, 256, 0, s, payload, ld_payload, scales, scale_layout, ld_scales, rows, cols,
                           out, ld_out),
                "dequantize launch");
    SW_LAUNCH_CHECK("sw_mx_dequantize launch");
    return ok();
}
