// SwiGLU forward and backward — HBM-bound element-wise kernels (the math is in swiglu_math.cuh).
// gate and up may be column slices of one [rows, 2F] buffer (the fused gate|up projection). The
// training step runs neither: the gate|up projection's GEMM writes h as well, and the down
// projection's input-gradient GEMM writes dg and du (gemm_sm100.cu, the same math).
#include "common.cuh"
#include "swiglu_math.cuh"

namespace veda::cuda
{
namespace
{

template <typename T, int V>
__device__ __forceinline__ void load_vec(const T* p, float (&out)[V])
{
    if constexpr (V == 1)
        out[0] = to_f32(*p);
    else
        load16(p, out);
}

template <typename T, int V>
__device__ __forceinline__ void store_vec(T* p, const float (&in)[V])
{
    if constexpr (V == 1)
        *p = from_f32<T>(in[0]);
    else
        store16(p, in);
}

// rows a thread loads before computing (bytes in flight); four in the forward measured slower
// (fewer blocks fit an SM)
constexpr int kFwdRows = 2;
constexpr int kBwdRows = 2;

// Row-blocked: a block takes kFwdRows (kBwdRows) rows at a time, its threads the 16-byte vectors of
// those rows, so no index needs a division and every thread keeps two rows' loads in flight.
template <typename T, bool VEC>
__global__ void swiglu_fwd_kernel(const T* __restrict__ gate, int64_t ldg, const T* __restrict__ up,
                                  int64_t ldu, T* __restrict__ h, int64_t ldh, int64_t rows,
                                  int64_t n)
{
    dep_wait();
    dep_release();
    constexpr int V = VEC ? Vec16<T>::N : 1;
    constexpr int U = kFwdRows;
    const int64_t nv = n / V;
    for (int64_t r0 = static_cast<int64_t>(blockIdx.x) * U; r0 < rows;
         r0 += static_cast<int64_t>(gridDim.x) * U)
    {
        for (int64_t cv = threadIdx.x; cv < nv; cv += blockDim.x)
        {
            const int64_t c = cv * V;
            float g[U][V], u[U][V];
#pragma unroll
            for (int k = 0; k < U; ++k)
            {
                if (r0 + k < rows)
                {
                    load_vec<T, V>(gate + (r0 + k) * ldg + c, g[k]);
                    load_vec<T, V>(up + (r0 + k) * ldu + c, u[k]);
                }
            }
#pragma unroll
            for (int k = 0; k < U; ++k)
            {
                if (r0 + k < rows)
                {
#pragma unroll
                    for (int j = 0; j < V; ++j) g[k][j] = swiglu_value(g[k][j], u[k][j]);
                    store_vec<T, V>(h + (r0 + k) * ldh + c, g[k]);
                }
            }
        }
    }
}

template <typename T, bool VEC>
__global__ void swiglu_bwd_kernel(const T* __restrict__ gate, int64_t ldg, const T* __restrict__ up,
                                  int64_t ldu, const T* __restrict__ dh, int64_t lddh,
                                  T* __restrict__ dgate, int64_t lddg, T* __restrict__ dup,
                                  int64_t lddu, int64_t rows, int64_t n)
{
    dep_wait();
    dep_release();
    constexpr int V = VEC ? Vec16<T>::N : 1;
    constexpr int U = kBwdRows;
    const int64_t nv = n / V;
    for (int64_t r0 = static_cast<int64_t>(blockIdx.x) * U; r0 < rows;
         r0 += static_cast<int64_t>(gridDim.x) * U)
    {
        for (int64_t cv = threadIdx.x; cv < nv; cv += blockDim.x)
        {
            const int64_t c = cv * V;
            float g[U][V], u[U][V], d[U][V];
#pragma unroll
            for (int k = 0; k < U; ++k)
            {
                if (r0 + k < rows)
                {
                    load_vec<T, V>(gate + (r0 + k) * ldg + c, g[k]);
                    load_vec<T, V>(up + (r0 + k) * ldu + c, u[k]);
                    load_vec<T, V>(dh + (r0 + k) * lddh + c, d[k]);
                }
            }
#pragma unroll
            for (int k = 0; k < U; ++k)
            {
                if (r0 + k < rows)
                {
                    float dg[V], du[V];
#pragma unroll
                    for (int j = 0; j < V; ++j) swiglu_grads(g[k][j], u[k][j], d[k][j], dg[j], du[j]);
                    store_vec<T, V>(dgate + (r0 + k) * lddg + c, dg);
                    store_vec<T, V>(dup + (r0 + k) * lddu + c, du);
                }
            }
        }
    }
}

// Block size: the row's vectors rounded up to warps (one vector per thread per row), 64-512.
unsigned row_threads(int64_t nv)
{
    int64_t t = (nv + 31) / 32 * 32;
    t = t < 64 ? 64 : (t > 512 ? 512 : t);
    return static_cast<unsigned>(t);
}

unsigned row_blocks(int64_t rows, unsigned threads, int rows_per_block)
{
    const int64_t want = (rows + rows_per_block - 1) / rows_per_block;
    const int64_t cap = static_cast<int64_t>(sm_count()) * (2048 / threads);
    return static_cast<unsigned>(want < cap ? want : cap);
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
    const unsigned threads = row_threads(vec ? n / (16 / static_cast<int64_t>(es)) : n);
    const unsigned grid = row_blocks(rows, threads, kFwdRows);
#define VEDA_SW_FWD(T, VEC)                                                                       \
    launch("veda_swiglu_fwd", swiglu_fwd_kernel<T, VEC>, dim3(grid), dim3(threads), 0, stream,     \
           static_cast<const T*>(gate), ldg, static_cast<const T*>(up), ldu, static_cast<T*>(h),  \
           ldh, rows, n)
    if (dtype == VEDA_BF16)
    {
        return vec ? VEDA_SW_FWD(bf16, true) : VEDA_SW_FWD(bf16, false);
    }
    return vec ? VEDA_SW_FWD(float, true) : VEDA_SW_FWD(float, false);
#undef VEDA_SW_FWD
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
    const unsigned threads = row_threads(vec ? n / (16 / static_cast<int64_t>(es)) : n);
    const unsigned grid = row_blocks(rows, threads, kBwdRows);
#define VEDA_SW_BWD(T, VEC)                                                                       \
    launch("veda_swiglu_bwd", swiglu_bwd_kernel<T, VEC>, dim3(grid), dim3(threads), 0, stream,     \
           static_cast<const T*>(gate), ldg, static_cast<const T*>(up), ldu,                     \
           static_cast<const T*>(dh), lddh, static_cast<T*>(dgate), lddg, static_cast<T*>(dup),  \
           lddu, rows, n)
    if (dtype == VEDA_BF16)
    {
        return vec ? VEDA_SW_BWD(bf16, true) : VEDA_SW_BWD(bf16, false);
    }
    return vec ? VEDA_SW_BWD(float, true) : VEDA_SW_BWD(float, false);
#undef VEDA_SW_BWD
}
