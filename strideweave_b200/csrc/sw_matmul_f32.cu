// sw_matmul_f32.cu - the reference's own Float32 contraction plan
// (BINARY32 products, FLOATING accumulation in Float32;
// src/strideweave/carriers/operation_policy.py:784-815) for arbitrary element
// strides: C[m, n] = sum_k A[m, k] * B[n, k].
//
// Each product is rounded to binary32 before it is added (no fused
// multiply-add), as CpuMatmulOperation does
// (src/strideweave/carriers/cpu/native/_cpu_accumulation.hpp:38-41); only the
// summation order differs, which the policy leaves backend-defined
// (operation_policy.py:109-114).  This path keeps Float32 semantics and is not
// the tensor-core path: MX operands use sw_mx_gemm.
#include "sw_common.cuh"

namespace sw {
namespace {

constexpr int kTile = 64;
constexpr int kKTile = 16;

__global__ void __launch_bounds__(256) matmul_f32_kernel(const float* __restrict__ a, int64_t sam, int64_t sak,
                                                         const float* __restrict__ b, int64_t sbn, int64_t sbk,
                                                         float* __restrict__ c, int64_t scm, int64_t scn, int64_t M,
                                                         int64_t N, int64_t K) {
    __shared__ float as[kKTile][kTile + 1];
    __shared__ float bs[kKTile][kTile + 1];
    const int tx = threadIdx.x % 16;  // n direction
    const int ty = threadIdx.x / 16;  // m direction
    const int64_t m0 = int64_t(blockIdx.y) * kTile;
    const int64_t n0 = int64_t(blockIdx.x) * kTile;
    float acc[4][4] = {};
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
                for (int j = 0; j < 4; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(av[i], bv[j]));
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t gm = m0 + ty * 4 + i, gn = n0 + tx * 4 + j;
            if (gm < M && gn < N) c[gm * scm + gn * scn] = acc[i][j];
        }
}

}  // namespace
}  // namespace sw

extern "C" int sw_matmul_f32(const float* a, int64_t sam, int64_t sak, const float* b, int64_t sbn, int64_t sbk,
                             float* c, int64_t scm, int64_t scn, int64_t M, int64_t N, int64_t K, void* stream) {
    using namespace sw;
    if (M < 0 || N < 0 || K < 0) return fail(SW_ERR_INVALID, "sw_matmul_f32: negative extent");
    if (M == 0 || N == 0) return ok();
    if (!a || !b || !c) return fail(SW_ERR_INVALID, "sw_matmul_f32: null pointer");
    if ((M + kTile - 1) / kTile > 65535) return fail(SW_ERR_UNSUPPORTED, "sw_matmul_f32: M too large");
    dim3 grid((unsigned)((N + kTile - 1) / kTile), (unsigned)((M + kTile - 1) / kTile));
    matmul_f32_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(a, sam, sak, b, sbn, sbk, c, scm, scn, M, N, K);
    SW_LAUNCH_CHECK("sw_matmul_f32 launch");
    return ok();
}
