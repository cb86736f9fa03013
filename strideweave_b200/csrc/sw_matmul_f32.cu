// sw_matmul_f32.cu - the reference's own Float32 contraction plan
// (BINARY32 products, FLOATING accumulation in Float32;
// src/strideweave/carriers/operation_policy.py:784-815) for arbitrary element
// strides: C[m, n] = sum_k A[m, k] * B[n, k].
//
// Each product is rounded to binary32 before it is added (no fused
// multiply-add), as CpuMatmulOperation does
// (src/strideweave/carriers/cpu/native/_cpu_accumulation.hpp:38-41); only the
// summation order differs, which the policy leaves backend-defined
// (operation_policy.py:109-114).  The widened plan (accumulator_dtype
// Float64, _cpu_accumulation.hpp:38-41) adds the same binary32 products in
// binary64 and rounds the sum once.  This path keeps Float32 semantics and is
// not the tensor-core path: MX operands use sw_mx_gemm.
#include "sw_common.cuh"

namespace sw {
namespace {

constexpr int kTile = 64;
constexpr int kKTile = 16;

__device__ __forceinline__ float acc_add(float s, float p) { return __fadd_rn(s, p); }
__device__ __forceinline__ double acc_add(double s, float p) { return __dadd_rn(s, double(p)); }
__device__ __forceinline__ float acc_out(float s) { return s; }
__device__ __forceinline__ float acc_out(double s) { return __double2float_rn(s); }

// blockIdx.z (+ z0) selects one contraction of a batch: operands advance by
// their batch strides (0 for a single contraction).  Acc is the accumulator
// type (float, or double for the widened plan).
template <class Acc>
__global__ void __launch_bounds__(256) matmul_f32_kernel(const float* __restrict__ a, int64_t sab, int64_t sam,
                                                         int64_t sak, const float* __restrict__ b, int64_t sbb,
                                                         int64_t sbn, int64_t sbk, float* __restrict__ c,
                                                         int64_t scb, int64_t scm, int64_t scn, int64_t M,
                                                         int64_t N, int64_t K, int64_t z0) {
    const int64_t z = z0 + blockIdx.z;
    a += z * sab;
    b += z * sbb;
    c += z * scb;
    __shared__ float as[kKTile][kTile + 1];
    __shared__ float bs[kKTile][kTile + 1];
    const int tx = threadIdx.x % 16;  // n direction
    const int ty = threadIdx.x / 16;  // m direction
    const int64_t m0 = int64_t(blockIdx.y) * kTile;
    const int64_t n0 = int64_t(blockIdx.x) * kTile;
    Acc acc[4][4] = {};
    for (int64_t k0 = 0; k0 < K; k0 += kKTile) {
        for (int i = threadIdx.x; i < kKTile * kTile; i += 256) {
            // consecutive threads walk k when it is the unit-stride axis
            const int kk = (sak == 1) ? (i % kKTile) : (i / kTile);
            const int mm = (sak == 1) ? (i / kKTile) : (i % kTile);
            const int64_t gm = m0 + mm, gk = k0 + kk;
            as[kk][mm] = (gm < M && gk < K) ? a[gm * sam + gk * sak] : 0.0f;
            const int kb = (sbk == 1) ? (i % kKTile) : (i / kTile);
            const int nn = (sbk == 1) ? (i / kKTile) : (i % kTile);
            const int64_t gn = n0 + nn, gk2 = k0 + kb;
            bs[kb][nn] = (gn < N && gk2 < K) ? b[gn * sbn + gk2 * sbk] : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < kKTile; ++kk) {
            float av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) av[i] = as[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) bv[j] = bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = acc_add(acc[i][j], __fmul_rn(av[i], bv[j]));
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t gm = m0 + ty * 4 + i, gn = n0 + tx * 4 + j;
            if (gm < M && gn < N) c[gm * scm + gn * scn] = acc_out(acc[i][j]);
        }
}

}  // namespace
}  // namespace sw

extern "C" int sw_matmul_f32_batched_ex(const float* a, int64_t sab, int64_t sam, int64_t sak, const float* b,
                                        int64_t sbb, int64_t sbn, int64_t sbk, float* c, int64_t scb, int64_t scm,
                                        int64_t scn, int64_t batch, int64_t M, int64_t N, int64_t K,
                                        int accumulator, void* stream) {
    using namespace sw;
    if (accumulator != SW_ACC_F32 && accumulator != SW_ACC_F64)
        return fail(SW_ERR_INVALID, "sw_matmul_f32: unknown accumulator %d", accumulator);
    if (batch < 0 || M < 0 || N < 0 || K < 0) return fail(SW_ERR_INVALID, "sw_matmul_f32: negative extent");
    if (batch == 0 || M == 0 || N == 0) return ok();
    if (!a || !b || !c) return fail(SW_ERR_INVALID, "sw_matmul_f32: null pointer");
    if ((M + kTile - 1) / kTile > 65535) return fail(SW_ERR_UNSUPPORTED, "sw_matmul_f32: M too large");
    for (int64_t z0 = 0; z0 < batch; z0 += 65535) {
        const int64_t nz = batch - z0 < 65535 ? batch - z0 : 65535;
        dim3 grid((unsigned)((N + kTile - 1) / kTile), (unsigned)((M + kTile - 1) / kTile), (unsigned)nz);
        if (accumulator == SW_ACC_F64)
            matmul_f32_kernel<double><<<grid, 256, 0, (cudaStream_t)stream>>>(a, sab, sam, sak, b, sbb, sbn, sbk, c,
                                                                              scb, scm, scn, M, N, K, z0);
        else
            matmul_f32_kernel<float><<<grid, 256, 0, (cudaStream_t)stream>>>(a, sab, sam, sak, b, sbb, sbn, sbk, c,
                                                                             scb, scm, scn, M, N, K, z0);
        SW_LAUNCH_CHECK("sw_matmul_f32 launch");
    }
    return ok();
}

extern "C" int sw_matmul_f32_batched(const float* a, int64_t sab, int64_t sam, int64_t sak, const float* b,
                                     int64_t sbb, int64_t sbn, int64_t sbk, float* c, int64_t scb, int64_t scm,
                                     int64_t scn, int64_t batch, int64_t M, int64_t N, int64_t K, void* stream) {
    return sw_matmul_f32_batched_ex(a, sab, sam, sak, b, sbb, sbn, sbk, c, scb, scm, scn, batch, M, N, K, SW_ACC_F32,
                                    stream);
}

extern "C" int sw_matmul_f32(const float* a, int64_t sam, int64_t sak, const float* b, int64_t sbn, int64_t sbk,
                             float* c, int64_t scm, int64_t scn, int64_t M, int64_t N, int64_t K, void* stream) {
    return sw_matmul_f32_batched_ex(a, 0, sam, sak, b, 0, sbn, sbk, c, 0, scm, scn, 1, M, N, K, SW_ACC_F32, stream);
}
