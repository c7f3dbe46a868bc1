// SwiGLU's element-wise math, shared by the stand-alone kernels (swiglu.cu) and the GEMM epilogues
// that fuse it into the projections around it (gemm_sm100.cu), so that both give the same bits.
//   forward  h = silu(g) * u, silu(g) = g / (1 + exp(-g))       src/libs/ops/Activations.cpp:13-16,
//                                                               src/libs/train/Model.cpp:201-202
//   backward dg = (dh * u) * s * (1 + g (1 - s)), s = sigmoid(g) src/libs/autograd/NonLinear.cpp:47-63
//            du = dh * silu(g)                                  src/libs/autograd/Variable.cpp:218-239
#pragma once

namespace veda::cuda
{

// sigmoid(g) = 1 / (1 + e^-g) with the hardware exponential and reciprocal-divide: a few ulp,
// far inside the fp32 tolerance, and exact at the ends (e^-g = inf gives 0, e^-g = 0 gives 1)
__device__ __forceinline__ float sigmoid_of(float g) { return __fdividef(1.0f, 1.0f + __expf(-g)); }

__device__ __forceinline__ float swiglu_value(float g, float u) { return g * sigmoid_of(g) * u; }

__device__ __forceinline__ void swiglu_grads(float g, float u, float d, float& dg, float& du)
{
    const float sg = sigmoid_of(g);
    const float through = d * u;
    dg = through * sg * (1.0f + g * (1.0f - sg));
    du = d * (g * sg);
}

} // namespace veda::cuda
