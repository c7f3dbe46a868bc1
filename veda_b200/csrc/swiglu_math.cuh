// SwiGLU's element-wise math, shared by the stand-alone kernels (swiglu.cu) and the GEMM epilogues
// that fuse it into the projections around it (gemm_sm100.cu), so that both give the same bits.
//   forward  h = silu(g) * u, silu(g) = g / (1 + exp(-g))       src/libs/ops/Activations.cpp:13-16,
//                                                               src/libs/train/Model.cpp:201-202
//   backward dg = (dh * u) * s * (1 + g (1 - s)), s = sigmoid(g) src/libs/autograd/NonLinear.cpp:47-63
//            du = dh * silu(g)                                  src/libs/autograd/Variable.cpp:218-239
#pragma once

#include "common.cuh"

namespace veda::cuda
{

// sigmoid(g) = 1 / (1 + e^-g) with the hardware exponential and reciprocal-divide: a few ulp,
// far inside the fp32 tolerance, and exact at the ends (e^-g = inf gives 0, e^-g = 0 gives 1)
__device__ __forceinline__ float sigmoid_of(float g) { return __fdividef(1.0f, 1.0f + __expf(-g)); }

__device__ __forceinline__ float swiglu_value(float g, float u) { return g * sigmoid_of(g) * u; }

// The gradient with every operation rounded on its own (no contraction left to the compiler), so
// that the packed form below gives the same bits.
__device__ __forceinline__ void swiglu_grads(float g, float u, float d, float& dg, float& du)
{
    const float sg = sigmoid_of(g);
    const float through = __fmul_rn(d, u);
    dg = __fmul_rn(__fmul_rn(through, sg), __fmaf_rn(g, __fsub_rn(1.0f, sg), 1.0f));
    du = __fmul_rn(d, __fmul_rn(g, sg));
}

// Two elements at once on fp32 pairs (g2, u2, d2 packed as by pk): the operations of swiglu_grads
// on f32x2 instructions, each rounded as its scalar form (1 - s as fma(s, -1, 1), exact before its
// one rounding like the subtraction).
__device__ __forceinline__ void swiglu_grads2(uint64_t g2, uint64_t u2, uint64_t d2, uint64_t& dg2,
                                              uint64_t& du2)
{
    float g0, g1;
    upk(g2, g0, g1);
    const uint64_t s2 = pk(sigmoid_of(g0), sigmoid_of(g1));
    const uint64_t one = pk(1.0f, 1.0f);
    const uint64_t a = mul2(mul2(d2, u2), s2);
    const uint64_t b = fma2(g2, fma2(s2, pk(-1.0f, -1.0f), one), one);
    dg2 = mul2(a, b);
    du2 = mul2(d2, mul2(g2, s2));
}

} // namespace veda::cuda
