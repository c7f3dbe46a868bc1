// SwiGLU forward and backward — HBM-bound element-wise kernels.
//   forward  h = silu(g) * u, silu(g) = g / (1 + exp(-g))       src/libs/ops/Activations.cpp:13-16,
//                                                               src/libs/train/Model.cpp:201-202
//   backward dg = (dh * u) * s * (1 + g (1 - s)), s = sigmoid(g) src/libs/autograd/NonLinear.cpp:47-63
//            du = dh * silu(g)                                  src/libs/autograd/Variable.cpp:218-239
// gate and up may be column slices of one [rows, 2F] buffer (the fused gate|up projection).
#include "common.cuh"

namespace veda::cuda
{
namespace
{

__device__ __forceinline__ float silu_of(float g) { return g / (1.0f + expf(-g)); }

template <typename T, bool VEC>
__global__ void swiglu_fwd_kernel(const T* __restrict__ gate, int64_t ldg, const T* __restrict__ up,
                                  int64_t ldu, T* __restrict__ h, int64_t ldh, int64_t rows,
                                  int64_t n)
{
    constexpr int V = VEC ? Vec16<T>::N : 1;
    const int64_t per_row = n / V;
    const int64_t total = rows * per_row;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        const int64_t r = idx / per_row;
        const int64_t c = (idx - r * per_row) * V;
        if constexpr (VEC)
        {
            float g[V], u[V];
            load16(gate + r * ldg + c, g);
            load16(up + r * ldu + c, u);
#pragma unroll
            for (int j = 0; j < V; ++j)
            {
                g[j] = silu_of(g[j]) * u[j];
            }
            store16(h + r * ldh + c, g);
        }
        else
        {
            const float g = to_f32(gate[r * ldg + c]);
            h[r * ldh + c] = from_f32<T>(silu_of(g) * to_f32(up[r * ldu + c]));
        }
    }
}

template <typename T, bool VEC>
__global__ void swiglu_bwd_kernel(const T* __restrict__ gate, int64_t ldg, const T* __restrict__ up,
                                  int64_t ldu, const T* __restrict__ dh, int64_t lddh,
                                  T* __restrict__ dgate, int64_t lddg, T* __restrict__ dup,
                                  int64_t lddu, int64_t rows, int64_t n)
{
    constexpr int V = VEC ? Vec16<T>::N : 1;
    const int64_t per_row = n / V;
    const int64_t total = rows * per_row;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        const int64_t r = idx / per_row;
        const int64_t c = (idx - r * per_row) * V;
        float g[V], u[V], d[V];
        if constexpr (VEC)
        {
            load16(gate + r * ldg + c, g);
            load16(up + r * ldu + c, u);
            load16(dh + r * lddh + c, d);
        }
        else
        {
            g[0] = to_f32(gate[r * ldg + c]);
            u[0] = to_f32(up[r * ldu + c]);
            d[0] = to_f32(dh[r * lddh + c]);
        }
        float dg[V], du[V];
#pragma unroll
        for (int j = 0; j < V; ++j)
        {
            const float e = expf(-g[j]);
            const float s = 1.0f / (1.0f + e);
            const float through = d[j] * u[j];
            dg[j] = through * s * (1.0f + g[j] * (1.0f - s));
            du[j] = d[j] * (g[j] / (1.0f + e));
        }
        if constexpr (VEC)
        {
            store16(dgate + r * lddg + c, dg);
            store16(dup + r * lddu + c, du);
        }
        else
        {
            dgate[r * lddg + c] = from_f32<T>(dg[0]);
            dup[r * lddu + c] = from_f32<T>(du[0]);
        }
    }
}

bool vec_ok(const void* p, int64_t ld, int64_t n, size_t es)
{
    const int64_t v = 16 / static_cast<int64_t>(es);
    return aligned16(p) && ld % v == 0 && n % v == 0;
}

} // namespace
} // namespace veda::cuda

using namespace veda::cuda;

extern "C" int veda_swiglu_fwd(const void* gate, int64_t ldg, const void* up, int64_t ldu, void* h,
                               int64_t ldh, int64_t rows, int64_t n, int dtype,
                               veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype), "unknown dtype");
    VEDA_REQUIRE(rows >= 0 && n >= 0 && ldg >= n && ldu >= n && ldh >= n, "bad shape");
    if (rows == 0 || n == 0)
    {
        return VEDA_OK;
    }
    VEDA_REQUIRE(gate && up && h, "null pointer");
    const size_t es = dtype_size(dtype);
    const bool vec = vec_ok(gate, ldg, n, es) && vec_ok(up, ldu, n, es) && vec_ok(h, ldh, n, es);
    const int64_t work = rows * (vec ? n / (16 / static_cast<int64_t>(es)) : n);
    const unsigned grid = grid_for(work, 256);
#define VEDA_SW_FWD(T, VEC)                                                                       \
    swiglu_fwd_kernel<T, VEC><<<grid, 256, 0, stream>>>(static_cast<const T*>(gate), ldg,        \
                                                        static_cast<const T*>(up), ldu,          \
                                                        static_cast<T*>(h), ldh, rows, n)
    if (dtype == VEDA_BF16)
    {
        if (vec) VEDA_SW_FWD(bf16, true); else VEDA_SW_FWD(bf16, false);
    }
    else
    {
        if (vec) VEDA_SW_FWD(float, true); else VEDA_SW_FWD(float, false);
    }
#undef VEDA_SW_FWD
    count_launch();
    return check_launch("veda_swiglu_fwd");
}

extern "C" int veda_swiglu_bwd(const void* gate, int64_t ldg, const void* up, int64_t ldu,
                               const void* dh, int64_t lddh, void* dgate, int64_t lddg, void* dup,
                               int64_t lddu, int64_t rows, int64_t n, int dtype,
                               veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype), "unknown dtype");
    VEDA_REQUIRE(rows >= 0 && n >= 0 && ldg >= n && ldu >= n && lddh >= n && lddg >= n &&
                     lddu >= n,
                 "bad shape");
    if (rows == 0 || n == 0)
    {
        return VEDA_OK;
    }
    VEDA_REQUIRE(gate && up && dh && dgate && dup, "null pointer");
    const size_t es = dtype_size(dtype);
    const bool vec = vec_ok(gate, ldg, n, es) && vec_ok(up, ldu, n, es) &&
                     vec_ok(dh, lddh, n, es) && vec_ok(dgate, lddg, n, es) &&
                     vec_ok(dup, lddu, n, es);
    const int64_t work = rows * (vec ? n / (16 / static_cast<int64_t>(es)) : n);
    const unsigned grid = grid_for(work, 256);
#define VEDA_SW_BWD(T, VEC)                                                                       \
    swiglu_bwd_kernel<T, VEC><<<grid, 256, 0, stream>>>(                                          \
        static_cast<const T*>(gate), ldg, static_cast<const T*>(up), ldu,                        \
        static_cast<const T*>(dh), lddh, static_cast<T*>(dgate), lddg, static_cast<T*>(dup),     \
        lddu, rows, n)
    if (dtype == VEDA_BF16)
    {
        if (vec) VEDA_SW_BWD(bf16, true); else VEDA_SW_BWD(bf16, false);
    }
    else
    {
        if (vec) VEDA_SW_BWD(float, true); else VEDA_SW_BWD(float, false);
    }
#undef VEDA_SW_BWD
    count_launch();
    return check_launch("veda_swiglu_bwd");
}
