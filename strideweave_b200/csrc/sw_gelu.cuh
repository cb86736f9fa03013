// sw_gelu.cuh - the erf GELU and its derivative, shared by the elementwise
// kernels and the quantisers that apply them on the fly, so that both paths
// produce the same bits (GELU formula: src/strideweave/carriers/cpu/native/
// _cpu_operation.hpp:33-40).
#pragma once

namespace sw {

__device__ __forceinline__ float gelu(float x) {
    return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

__device__ __forceinline__ float gelu_grad(float x) {
    const float cdf = 0.5f * (1.0f + erff(x * 0.70710678118654752f));
    const float pdf = 0.39894228040143268f * expf(-0.5f * x * x);
    return cdf + x * pdf;
}

}  // namespace sw
