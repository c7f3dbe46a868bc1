// RMSNorm, QK-norm + RoPE and RoPE kernels — HBM-bound, one warp per row.
//
// Arithmetic follows the reference exactly where it can (fp32 throughout):
//   forward   r = sqrt(sum(x^2)/n + eps); y = (x / r) * gamma
//             src/libs/ops/Normalize.cpp:50-63, then mul by gamma (src/libs/train/Model.cpp:242-243)
//   backward  G = dy * gamma; dx = G / r - x * (sum(G x) / (n r^3)); dgamma = sum_rows dy * (x/r)
//             src/libs/autograd/NonLinear.cpp:171-196, the gain's mul/unbroadcast
//             (src/libs/autograd/Variable.cpp:218-239, 48-87)
//   RoPE      out_i = x_i c - x_{i+p} s; out_{i+p} = x_{i+p} c + x_i s; backward with -s
//             src/libs/autograd/Views.cpp:124-125, 163-164
// The gain gradient is reduced deterministically: each warp owns a shared-memory row, warps are
// summed in a fixed order into one partial per block, and a second kernel sums the block
// partials in a fixed order and adds the result into dgamma.
#include "common.cuh"
#include "norm_stream.cuh"

#include <algorithm>
#include <mutex>

namespace veda::cuda
{
namespace
{

constexpr int kWarps = 8;   // warps per block for the row kernels

// QK-norm backward: two resident blocks per SM, each writing one 128-float partial row of the
// gain gradient.
inline int qk_bwd_grid(int64_t rows)
{
    int64_t blocks = (rows + 4 * kWarps - 1) / (4 * kWarps);
    const int64_t cap = 2LL * sm_count();
    return static_cast<int>(blocks < cap ? (blocks < 1 ? 1 : blocks) : cap);
}

inline int norm_bwd_grid(int64_t rows)
{
    int64_t blocks = (rows + kWarps - 1) / kWarps;
    const int64_t cap = 2LL * sm_count();
    return static_cast<int>(blocks < cap ? (blocks < 1 ? 1 : blocks) : cap);
}

// ---- forward ---------------------------------------------------------------------------------
template <typename T, bool VEC>
__global__ void __launch_bounds__(kWarps * 32)
rmsnorm_fwd_kernel(const T* __restrict__ x, int64_t ldx, const T* __restrict__ gamma,
                   T* __restrict__ y, int64_t ldy, int64_t rows, int n, float eps)
{
    constexpr int V = Vec16<T>::N;
    const int lane = threadIdx.x & 31;
    const int64_t warp = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kWarps;
    for (int64_t row = warp; row < rows; row += stride)
    {
        const T* xr = x + row * ldx;
        T* yr = y + row * ldy;
        float ss = 0.0f;
        if constexpr (VEC)
        {
            for (int i = lane * V; i < n; i += 32 * V)
            {
                float v[V];
                load16(xr + i, v);
#pragma unroll
                for (int j = 0; j < V; ++j)
                {
                    ss += v[j] * v[j];
                }
            }
        }
        else
        {
            for (int i = lane; i < n; i += 32)
            {
                const float v = to_f32(xr[i]);
                ss += v * v;
            }
        }
        ss = warp_sum(ss);
        const float r = sqrtf(ss / static_cast<float>(n) + eps);
        if constexpr (VEC)
        {
            for (int i = lane * V; i < n; i += 32 * V)
            {
                float v[V], g[V];
                load16(xr + i, v);
                if (gamma != nullptr)
                {
                    load16(gamma + i, g);
                }
#pragma unroll
                for (int j = 0; j < V; ++j)
                {
                    const float t = v[j] / r;
                    v[j] = gamma != nullptr ? t * g[j] : t;
                }
                store16(yr + i, v);
            }
        }
        else
        {
            for (int i = lane; i < n; i += 32)
            {
                const float t = to_f32(xr[i]) / r;
                yr[i] = from_f32<T>(gamma != nullptr ? t * to_f32(gamma[i]) : t);
            }
        }
    }
}

// ---- backward --------------------------------------------------------------------------------
// Shared memory: [kWarps][n] fp32 gain-gradient rows, one per warp (only when partials != null).
template <typename T, bool VEC>
__global__ void __launch_bounds__(kWarps * 32)
rmsnorm_bwd_kernel(const T* __restrict__ x, int64_t ldx, const T* __restrict__ gamma,
                   const T* __restrict__ dy, int64_t lddy, const T* __restrict__ dresid,
                   int64_t ldr, T* __restrict__ dx, int64_t lddx, float* __restrict__ partials,
                   int64_t rows, int n, float eps)
{
    constexpr int V = Vec16<T>::N;
    extern __shared__ float smem[];
    const int lane = threadIdx.x & 31;
    const int wid = threadIdx.x >> 5;
    float* mine = smem + static_cast<size_t>(wid) * n;
    if (partials != nullptr)
    {
        for (int i = lane; i < n; i += 32)
        {
            mine[i] = 0.0f;
        }
    }
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kWarps;
    for (int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + wid; row < rows; row += stride)
    {
        const T* xr = x + row * ldx;
        const T* gr = dy + row * lddy;
        float ss = 0.0f, w = 0.0f;
        if constexpr (VEC)
        {
            for (int i = lane * V; i < n; i += 32 * V)
            {
                float xv[V], gv[V], gm[V];
                load16(xr + i, xv);
                load16(gr + i, gv);
                if (gamma != nullptr)
                {
                    load16(gamma + i, gm);
                }
#pragma unroll
                for (int j = 0; j < V; ++j)
                {
                    const float G = gamma != nullptr ? gv[j] * gm[j] : gv[j];
                    ss += xv[j] * xv[j];
                    w += G * xv[j];
                }
            }
        }
        else
        {
            for (int i = lane; i < n; i += 32)
            {
                const float xv = to_f32(xr[i]);
                const float G = gamma != nullptr ? to_f32(gr[i]) * to_f32(gamma[i]) : to_f32(gr[i]);
                ss += xv * xv;
                w += G * xv;
            }
        }
        ss = warp_sum(ss);
        w = warp_sum(w);
        const float nf = static_cast<float>(n);
        const float r = sqrtf(ss / nf + eps);
        const float coupling = w / (nf * r * r * r);
        T* out = dx + row * lddx;
        const T* rr = dresid != nullptr ? dresid + row * ldr : nullptr;
        if constexpr (VEC)
        {
            for (int i = lane * V; i < n; i += 32 * V)
            {
                float xv[V], gv[V], gm[V], res[V];
                load16(xr + i, xv);
                load16(gr + i, gv);
                if (gamma != nullptr)
                {
                    load16(gamma + i, gm);
                }
                if (rr != nullptr)
                {
                    load16(rr + i, res);
                }
#pragma unroll
                for (int j = 0; j < V; ++j)
                {
                    const float G = gamma != nullptr ? gv[j] * gm[j] : gv[j];
                    float d = G / r - xv[j] * coupling;
                    if (rr != nullptr)
                    {
                        d = res[j] + d;
                    }
                    if (partials != nullptr)
                    {
                        mine[i + j] += gv[j] * (xv[j] / r);
                    }
                    xv[j] = d;
                }
                store16(out + i, xv);
            }
        }
        else
        {
            for (int i = lane; i < n; i += 32)
            {
                const float xv = to_f32(xr[i]);
                const float gv = to_f32(gr[i]);
                const float G = gamma != nullptr ? gv * to_f32(gamma[i]) : gv;
                float d = G / r - xv * coupling;
                if (rr != nullptr)
                {
                    d = to_f32(rr[i]) + d;
                }
                if (partials != nullptr)
                {
                    mine[i] += gv * (xv / r);
                }
                out[i] = from_f32<T>(d);
            }
        }
    }
    if (partials != nullptr)
    {
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += blockDim.x)
        {
            float s = 0.0f;
            for (int k = 0; k < kWarps; ++k)
            {
                s += smem[static_cast<size_t>(k) * n + i];
            }
            partials[static_cast<size_t>(blockIdx.x) * n + i] = s;
        }
    }
}

// dgamma[i] += sum over blocks of partials[b][i], in a fixed order; blockIdx.y picks one of two
// (partials, blocks, dgamma) sets (the q and k gains of a QK-norm backward).
__global__ void __launch_bounds__(256)
reduce_partials_kernel(const float* __restrict__ partials0, int blocks0, float* __restrict__ dgamma0,
                       const float* __restrict__ partials1, int blocks1, float* __restrict__ dgamma1,
                       int n)
{
    dep_wait();
    dep_release();
    const float* __restrict__ partials = blockIdx.y == 0 ? partials0 : partials1;
    const int blocks = blockIdx.y == 0 ? blocks0 : blocks1;
    float* __restrict__ dgamma = blockIdx.y == 0 ? dgamma0 : dgamma1;
    // 8 columns x 32 row groups per block: group g sums partial rows g, g + 32, ... of its column
    // in that order, then the 32 group sums are added in group order (deterministic).
    __shared__ float part[32][9];
    const int c = threadIdx.x & 7, grp = threadIdx.x >> 3;
    const int col = blockIdx.x * 8 + c;
    float acc = 0.0f;
    if (col < n)
    {
#pragma unroll 4
        for (int b = grp; b < blocks; b += 32)
        {
            acc += partials[static_cast<size_t>(b) * n + col];
        }
    }
    part[grp][c] = acc;
    __syncthreads();
    if (grp == 0 && col < n)
    {
        float s = 0.0f;
#pragma unroll
        for (int g = 0; g < 32; ++g)
        {
            s += part[g][c];
        }
        dgamma[col] += s;
    }
}

// sum = x + r over rows of n (the residual add of the fused add + norm, when the streaming
// kernel does not apply)
template <typename T>
__global__ void add_rows_kernel(const T* __restrict__ x, int64_t ldx, const T* __restrict__ r,
                                int64_t ldr, T* __restrict__ sum, int64_t lds, int64_t rows,
                                int64_t n)
{
    const int64_t total = rows * n;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        const int64_t row = i / n, c = i % n;
        sum[row * lds + c] = from_f32<T>(to_f32(x[row * ldx + c]) + to_f32(r[row * ldr + c]));
    }
}

inline int launch_reduce_partials(const float* partials, int blocks, int n, float* dgamma,
                                  cudaStream_t s, const float* partials1 = nullptr, int blocks1 = 0,
                                  float* dgamma1 = nullptr)
{
    const dim3 grid((n + 7) / 8, partials1 != nullptr ? 2 : 1);
    return launch("gain gradient (sum of block partials)", reduce_partials_kernel, grid, dim3(256), 0,
                  s, partials, blocks, dgamma, partials1, blocks1, dgamma1, n);
}

// ---- register-resident row kernels (n == CH * 32 * V, 16-byte aligned rows) ------------------
// Every 16-byte chunk of a row is loaded before any is used, so a warp keeps the whole row in
// flight instead of one dependent load at a time; the row is then reused from registers.
template <typename T>
__device__ __forceinline__ void unpack16(const uint4& raw, float (&out)[16 / sizeof(T)])
{
    if constexpr (sizeof(T) == 4)
    {
        out[0] = __uint_as_float(raw.x);
        out[1] = __uint_as_float(raw.y);
        out[2] = __uint_as_float(raw.z);
        out[3] = __uint_as_float(raw.w);
    }
    else
    {
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
        {
            out[2 * i] = __uint_as_float(w[i] << 16);
            out[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        }
    }
}

// ---- row-group kernels: TPR threads per row, each owning V consecutive columns ----------------
// A 512-thread block works on 512 / TPR rows at a time; the next row of each group is loaded
// before the current one is reduced, so loads stay in flight across the block-wide reduction.
// Each thread's columns are fixed, so gamma stays in registers and (backward) the gain gradient
// accumulates per thread without a shared-memory pass per row.
constexpr int kRowThreads = 512;

template <typename T, int TPR>
__global__ void __launch_bounds__(kRowThreads)
rmsnorm_fwd_rows_kernel(const T* __restrict__ x, int64_t ldx, const T* __restrict__ gamma,
                        T* __restrict__ y, int64_t ldy, int64_t rows, float eps)
{
    constexpr int V = Vec16<T>::N;
    constexpr int G = kRowThreads / TPR;     // rows per block step
    constexpr int W = TPR / 32;              // warps per row
    constexpr int n = TPR * V;
    __shared__ float red[2][G][W];
    const int g = threadIdx.x / TPR, t = threadIdx.x % TPR;
    const int wr = t >> 5, lane = threadIdx.x & 31;
    const int64_t step = static_cast<int64_t>(gridDim.x) * G;
    const int64_t first = static_cast<int64_t>(blockIdx.x) * G;
    const int64_t iters = first < rows ? (rows - first + step - 1) / step : 0;
    float gm[V];
    if (gamma != nullptr)
    {
        load16(gamma + t * V, gm);
    }
    int64_t row = first + g;
    uint4 cur = make_uint4(0, 0, 0, 0);
    if (row < rows)
    {
        cur = *reinterpret_cast<const uint4*>(x + row * ldx + t * V);
    }
    for (int64_t k = 0; k < iters; ++k)
    {
        const int64_t nrow = row + step;
        uint4 nxt = make_uint4(0, 0, 0, 0);
        if (nrow < rows)
        {
            nxt = *reinterpret_cast<const uint4*>(x + nrow * ldx + t * V);
        }
        float v[V];
        unpack16<T>(cur, v);
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < V; ++j) ss += v[j] * v[j];
        ss = warp_sum(ss);
        const int b = static_cast<int>(k & 1);
        if (lane == 0) red[b][g][wr] = ss;
        __syncthreads();
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < W; ++w) tot += red[b][g][w];
        const float inv = 1.0f / sqrtf(tot / static_cast<float>(n) + eps);
        if (row < rows)
        {
#pragma unroll
            for (int j = 0; j < V; ++j)
            {
                const float tn = v[j] * inv;
                v[j] = gamma != nullptr ? tn * gm[j] : tn;
            }
            store16(y + row * ldy + t * V, v);
        }
        cur = nxt;
        row = nrow;
    }
}

// Shared memory: [G][n] fp32 for the final cross-group sum of the gain gradient.
// Two blocks per SM (64 registers a thread) keep 32 warps and 64 rows of loads in flight per SM.
template <typename T, int TPR>
__global__ void __launch_bounds__(kRowThreads, 2)
rmsnorm_bwd_rows_kernel(const T* __restrict__ x, int64_t ldx, const T* __restrict__ gamma,
                        const T* __restrict__ dy, int64_t lddy, const T* __restrict__ dresid,
                        int64_t ldr, T* __restrict__ dx, int64_t lddx, float* __restrict__ partials,
                        int64_t rows, float eps)
{
    constexpr int V = Vec16<T>::N;
    constexpr int G = kRowThreads / TPR;
    constexpr int W = TPR / 32;
    constexpr int n = TPR * V;
    __shared__ float2 red[2][G][W];
    extern __shared__ float part[];
    const int g = threadIdx.x / TPR, t = threadIdx.x % TPR;
    const int wr = t >> 5, lane = threadIdx.x & 31;
    const int64_t step = static_cast<int64_t>(gridDim.x) * G;
    const int64_t first = static_cast<int64_t>(blockIdx.x) * G;
    const int64_t iters = first < rows ? (rows - first + step - 1) / step : 0;
    const int64_t col = static_cast<int64_t>(t) * V;
    float acc[V];
#pragma unroll
    for (int j = 0; j < V; ++j) acc[j] = 0.0f;
    const uint4 zero = make_uint4(0, 0, 0, 0);
    int64_t row = first + g;
    uint4 cx = zero, cg = zero, cr = zero;
    if (row < rows)
    {
        cx = *reinterpret_cast<const uint4*>(x + row * ldx + col);
        cg = *reinterpret_cast<const uint4*>(dy + row * lddy + col);
        if (dresid != nullptr) cr = *reinterpret_cast<const uint4*>(dresid + row * ldr + col);
    }
    for (int64_t k = 0; k < iters; ++k)
    {
        const int64_t nrow = row + step;
        uint4 nx = zero, ng = zero, nr = zero;
        if (nrow < rows)
        {
            nx = *reinterpret_cast<const uint4*>(x + nrow * ldx + col);
            ng = *reinterpret_cast<const uint4*>(dy + nrow * lddy + col);
            if (dresid != nullptr) nr = *reinterpret_cast<const uint4*>(dresid + nrow * ldr + col);
        }
        float ss = 0.0f, w = 0.0f;
        {
            float xv[V], gv[V], gm[V];
            unpack16<T>(cx, xv);
            unpack16<T>(cg, gv);
            if (gamma != nullptr)
            {
                load16(gamma + col, gm);   // an L1 hit after the first row
            }
            else
            {
#pragma unroll
                for (int j = 0; j < V; ++j) gm[j] = 1.0f;
            }
#pragma unroll
            for (int j = 0; j < V; ++j)
            {
                ss += xv[j] * xv[j];
                w += (gv[j] * gm[j]) * xv[j];
            }
        }
        ss = warp_sum(ss);
        w = warp_sum(w);
        const int b = static_cast<int>(k & 1);
        if (lane == 0) red[b][g][wr] = make_float2(ss, w);
        __syncthreads();
        float tss = 0.0f, tw = 0.0f;
#pragma unroll
        for (int q = 0; q < W; ++q)
        {
            tss += red[b][g][q].x;
            tw += red[b][g][q].y;
        }
        if (row < rows)
        {
            // the row is unpacked again from its packed registers (fewer live values across the
            // barrier)
            float xv[V], gv[V], gm[V];
            unpack16<T>(cx, xv);
            unpack16<T>(cg, gv);
            if (gamma != nullptr)
            {
                load16(gamma + col, gm);
            }
            else
            {
#pragma unroll
                for (int j = 0; j < V; ++j) gm[j] = 1.0f;
            }
            const float inv = 1.0f / sqrtf(tss / static_cast<float>(n) + eps);
            const float coupling = tw * inv * inv * inv / static_cast<float>(n);
            float res[V];
            if (dresid != nullptr) unpack16<T>(cr, res);
#pragma unroll
            for (int j = 0; j < V; ++j)
            {
                float d = (gv[j] * gm[j]) * inv - xv[j] * coupling;
                if (dresid != nullptr) d = res[j] + d;
                acc[j] += gv[j] * (xv[j] * inv);
                xv[j] = d;
            }
            store16(dx + row * lddx + col, xv);
        }
        cx = nx;
        cg = ng;
        cr = nr;
        row = nrow;
    }
    if (partials != nullptr)
    {
#pragma unroll
        for (int j = 0; j < V; ++j) part[g * n + col + j] = acc[j];
        __syncthreads();
        for (int c = threadIdx.x; c < n; c += kRowThreads)
        {
            float s = 0.0f;
#pragma unroll
            for (int q = 0; q < G; ++q) s += part[q * n + c];
            partials[static_cast<size_t>(blockIdx.x) * n + c] = s;
        }
    }
}

template <typename T, int CH>
__global__ void __launch_bounds__(kWarps * 32)
rmsnorm_fwd_reg_kernel(const T* __restrict__ x, int64_t ldx, const T* __restrict__ gamma,
                       T* __restrict__ y, int64_t ldy, int64_t rows, float eps)
{
    constexpr int V = Vec16<T>::N;
    constexpr int n = CH * 32 * V;
    const int lane = threadIdx.x & 31;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kWarps;
    for (int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5); row < rows;
         row += stride)
    {
        uint4 xr[CH];
#pragma unroll
        for (int c = 0; c < CH; ++c)
        {
            xr[c] = *reinterpret_cast<const uint4*>(x + row * ldx + (c * 32 + lane) * V);
        }
        float ss = 0.0f;
#pragma unroll
        for (int c = 0; c < CH; ++c)
        {
            float v[V];
            unpack16<T>(xr[c], v);
#pragma unroll
            for (int j = 0; j < V; ++j)
            {
                ss += v[j] * v[j];
            }
        }
        ss = warp_sum(ss);
        const float r = sqrtf(ss / static_cast<float>(n) + eps);
#pragma unroll
        for (int c = 0; c < CH; ++c)
        {
            float v[V], g[V];
            unpack16<T>(xr[c], v);
            if (gamma != nullptr)
            {
                load16(gamma + (c * 32 + lane) * V, g);
            }
#pragma unroll
            for (int j = 0; j < V; ++j)
            {
                const float t = v[j] / r;
                v[j] = gamma != nullptr ? t * g[j] : t;
            }
            store16(y + row * ldy + (c * 32 + lane) * V, v);
        }
    }
}

// Shared memory (when partials != null): [kWarps][n] fp32, one gain-gradient row per warp.
template <typename T, int CH>
__global__ void __launch_bounds__(kWarps * 32)
rmsnorm_bwd_reg_kernel(const T* __restrict__ x, int64_t ldx, const T* __restrict__ gamma,
                       const T* __restrict__ dy, int64_t lddy, const T* __restrict__ dresid,
                       int64_t ldr, T* __restrict__ dx, int64_t lddx,
                       float* __restrict__ partials, int64_t rows, float eps)
{
    constexpr int V = Vec16<T>::N;
    constexpr int n = CH * 32 * V;
    extern __shared__ float smem[];
    const int lane = threadIdx.x & 31;
    const int wid = threadIdx.x >> 5;
    float acc[CH][V];
#pragma unroll
    for (int c = 0; c < CH; ++c)
#pragma unroll
        for (int j = 0; j < V; ++j) acc[c][j] = 0.0f;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kWarps;
    for (int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + wid; row < rows; row += stride)
    {
        uint4 xr[CH], gr[CH], rr[CH];
#pragma unroll
        for (int c = 0; c < CH; ++c)
        {
            const int64_t col = (c * 32 + lane) * V;
            xr[c] = *reinterpret_cast<const uint4*>(x + row * ldx + col);
            gr[c] = *reinterpret_cast<const uint4*>(dy + row * lddy + col);
            if (dresid != nullptr)
            {
                rr[c] = *reinterpret_cast<const uint4*>(dresid + row * ldr + col);
            }
        }
        float ss = 0.0f, w = 0.0f;
#pragma unroll
        for (int c = 0; c < CH; ++c)
        {
            float xv[V], gv[V], gm[V];
            unpack16<T>(xr[c], xv);
            unpack16<T>(gr[c], gv);
            if (gamma != nullptr)
            {
                load16(gamma + (c * 32 + lane) * V, gm);
            }
#pragma unroll
            for (int j = 0; j < V; ++j)
            {
                const float G = gamma != nullptr ? gv[j] * gm[j] : gv[j];
                ss += xv[j] * xv[j];
                w += G * xv[j];
            }
        }
        ss = warp_sum(ss);
        w = warp_sum(w);
        const float nf = static_cast<float>(n);
        const float r = sqrtf(ss / nf + eps);
        const float coupling = w / (nf * r * r * r);
#pragma unroll
        for (int c = 0; c < CH; ++c)
        {
            float xv[V], gv[V], gm[V], res[V];
            unpack16<T>(xr[c], xv);
            unpack16<T>(gr[c], gv);
            if (gamma != nullptr)
            {
                load16(gamma + (c * 32 + lane) * V, gm);
            }
            if (dresid != nullptr)
            {
                unpack16<T>(rr[c], res);
            }
#pragma unroll
            for (int j = 0; j < V; ++j)
            {
                const float G = gamma != nullptr ? gv[j] * gm[j] : gv[j];
                float d = G / r - xv[j] * coupling;
                if (dresid != nullptr)
                {
                    d = res[j] + d;
                }
                acc[c][j] += gv[j] * (xv[j] / r);
                xv[j] = d;
            }
            store16(dx + row * lddx + (c * 32 + lane) * V, xv);
        }
    }
    if (partials != nullptr)
    {
        float* mine = smem + static_cast<size_t>(wid) * n;
#pragma unroll
        for (int c = 0; c < CH; ++c)
#pragma unroll
            for (int j = 0; j < V; ++j) mine[(c * 32 + lane) * V + j] = acc[c][j];
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += blockDim.x)
        {
            float s = 0.0f;
            for (int k = 0; k < kWarps; ++k)
            {
                s += smem[static_cast<size_t>(k) * n + i];
            }
            partials[static_cast<size_t>(blockIdx.x) * n + i] = s;
        }
    }
}

// ---- QK-norm + RoPE, head_dim 128, bf16: eight lanes per (token, head) row ---------------------
// Lane q of an 8-lane group holds elements [8q, 8q+8) and their rotation partners
// [64+8q, 64+8q+8) as two 16-byte vectors; a warp works on 4 rows at once and loads its next 4
// rows (kept packed as bf16) before working on the current ones.
__device__ __forceinline__ float group8_sum(float v)
{
    v += __shfl_xor_sync(0xFFFFFFFFu, v, 1);
    v += __shfl_xor_sync(0xFFFFFFFFu, v, 2);
    v += __shfl_xor_sync(0xFFFFFFFFu, v, 4);
    return v;
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4& raw, float (&out)[8])
{
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        out[2 * i] = __uint_as_float(w[i] << 16);
        out[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

__device__ __forceinline__ void rope_row(const float* cosv, const float* sinv, int t, int q,
                                         float (&cs)[8], float (&sn)[8])
{
    const float4* cp = reinterpret_cast<const float4*>(cosv + static_cast<int64_t>(t) * 128 + 8 * q);
    const float4* sp = reinterpret_cast<const float4*>(sinv + static_cast<int64_t>(t) * 128 + 8 * q);
    const float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
    cs[0] = c0.x; cs[1] = c0.y; cs[2] = c0.z; cs[3] = c0.w;
    cs[4] = c1.x; cs[5] = c1.y; cs[6] = c1.z; cs[7] = c1.w;
    sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w;
    sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
}

// One of the (up to) two sets of rows of a QK-norm forward launch: the q heads and the k heads of
// one attention layer share a launch, each with its own blocks, gain and output (blocks = 0: no
// second set).
struct QkFwdSet
{
    const bf16* x;
    const bf16* gamma;
    bf16* y;
    int64_t ldx, ldy;
    int heads, blocks;
};

__global__ void __launch_bounds__(kWarps * 32)
qknorm_rope_fwd_d128_kernel(const QkFwdSet s0, const QkFwdSet s1, const float* __restrict__ cosv,
                            const float* __restrict__ sinv, int64_t tokens, int seq_len, float eps)
{
    dep_wait();
    dep_release();
    // this block's set, and the block's index within it
    const bool second = static_cast<int>(blockIdx.x) >= s0.blocks;
    const bf16* __restrict__ x = second ? s1.x : s0.x;
    const bf16* __restrict__ gamma = second ? s1.gamma : s0.gamma;
    bf16* __restrict__ y = second ? s1.y : s0.y;
    const int64_t ldx = second ? s1.ldx : s0.ldx, ldy = second ? s1.ldy : s0.ldy;
    const int heads = second ? s1.heads : s0.heads;
    const int nblk = second ? s1.blocks : s0.blocks;
    const int blk = second ? static_cast<int>(blockIdx.x) - s0.blocks : static_cast<int>(blockIdx.x);
    const int lane = threadIdx.x & 31, q = lane & 7;
    const int64_t rows = tokens * heads;
    const int64_t stride = static_cast<int64_t>(nblk) * kWarps * 4;
    int64_t row = (static_cast<int64_t>(blk) * kWarps + (threadIdx.x >> 5)) * 4 + (lane >> 3);
    const uint4 zero = make_uint4(0, 0, 0, 0);
    auto load_row = [&](int64_t r, uint4& a, uint4& b) {
        if (r < rows)
        {
            // rows < 2^31 (checked by the launcher): 32-bit division
            const int64_t token = static_cast<uint32_t>(r) / static_cast<uint32_t>(heads);
            const bf16* xr = x + token * ldx + (r - token * heads) * 128;
            a = *reinterpret_cast<const uint4*>(xr + 8 * q);
            b = *reinterpret_cast<const uint4*>(xr + 64 + 8 * q);
        }
        else
        {
            a = zero;
            b = zero;
        }
    };
    uint4 ca, cb;
    load_row(row, ca, cb);
    // every lane of a warp runs the same number of steps (the group sums shuffle across rows)
    const int64_t wfirst = row - (lane >> 3);
    const int64_t iters = wfirst < rows ? (rows - wfirst + stride - 1) / stride : 0;
    for (int64_t k = 0; k < iters; ++k)
    {
        uint4 na, nb;
        load_row(row + stride, na, nb);
        float a[8], b[8];
        bf16x8_to_f32(ca, a);
        bf16x8_to_f32(cb, b);
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) ss += a[j] * a[j] + b[j] * b[j];
        ss = group8_sum(ss);
        if (row < rows)
        {
            const float inv = 1.0f / sqrtf(ss / 128.0f + eps);
            const int64_t token = static_cast<uint32_t>(row) / static_cast<uint32_t>(heads);
            const int t = static_cast<int>(static_cast<uint32_t>(token) % static_cast<uint32_t>(seq_len));
            float ga[8], gb[8], cs[8], sn[8];
            load16(gamma + 8 * q, ga);
            load16(gamma + 64 + 8 * q, gb);
            rope_row(cosv, sinv, t, q, cs, sn);
            float oa[8], ob[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
            {
                const float na2 = (a[j] * inv) * ga[j], nb2 = (b[j] * inv) * gb[j];
                oa[j] = na2 * cs[j] - nb2 * sn[j];
                ob[j] = nb2 * cs[j] + na2 * sn[j];
            }
            bf16* yr = y + token * ldy + (row - token * heads) * 128;
            store16(yr + 8 * q, oa);
            store16(yr + 64 + 8 * q, ob);
        }
        ca = na;
        cb = nb;
        row += stride;
    }
}

// One of the (up to) two sets of rows a QK-norm backward launch works through: the q heads and
// the k heads of one attention layer share a launch, each with its own blocks, gain and partial
// rows of the gain gradient (blocks = 0: no second set).
struct QkSet
{
    const bf16* x;
    const bf16* gamma;
    const bf16* dy;
    bf16* dx;
    float* partials;
    int64_t ldx, lddy, lddx;
    int heads, blocks;
    // instead of dy: fp32 rows (stride lddy floats) read as bf16(dyf * dy_scale) — the attention
    // backward's dQ accumulator and the rounding it would have applied itself
    const float* dyf;
    float dy_scale;
};

// Shared memory: [kWarps * 4][128] fp32 gain-gradient rows (one per row slot).
__global__ void __launch_bounds__(kWarps * 32, 2)
qknorm_rope_bwd_d128_kernel(const QkSet s0, const QkSet s1, const float* __restrict__ cosv,
                            const float* __restrict__ sinv, int64_t tokens, int seq_len, float eps)
{
    dep_wait();
    dep_release();
    __shared__ float part[kWarps * 4][128];
    // this block's set, and the block's index within it
    const bool second = static_cast<int>(blockIdx.x) >= s0.blocks;
    const bf16* __restrict__ x = second ? s1.x : s0.x;
    const bf16* __restrict__ gamma = second ? s1.gamma : s0.gamma;
    const bf16* __restrict__ dy = second ? s1.dy : s0.dy;
    const float* __restrict__ dyf = second ? s1.dyf : s0.dyf;
    const float dy_scale = second ? s1.dy_scale : s0.dy_scale;
    bf16* __restrict__ dx = second ? s1.dx : s0.dx;
    float* __restrict__ partials = second ? s1.partials : s0.partials;
    const int64_t ldx = second ? s1.ldx : s0.ldx, lddy = second ? s1.lddy : s0.lddy,
                  lddx = second ? s1.lddx : s0.lddx;
    const int heads = second ? s1.heads : s0.heads;
    const int nblk = second ? s1.blocks : s0.blocks;
    const int blk = second ? static_cast<int>(blockIdx.x) - s0.blocks : static_cast<int>(blockIdx.x);
    const int lane = threadIdx.x & 31, q = lane & 7, slot = (threadIdx.x >> 5) * 4 + (lane >> 3);
    const int64_t rows = tokens * heads;   // below 2^31 (checked by the launcher)
    const int stride = nblk * kWarps * 4;
    int64_t row = (static_cast<int64_t>(blk) * kWarps + (threadIdx.x >> 5)) * 4 + (lane >> 3);
    // (token, head, position) of a row, stepped by `stride` rows without a division per step
    const int sdiv = stride / heads, smod = stride % heads, tstep = sdiv % seq_len;
    auto advance = [&](int& tok, int& hh, int& tt) {
        hh += smod;
        tok += sdiv;
        tt += tstep;
        if (hh >= heads)
        {
            hh -= heads;
            ++tok;
            ++tt;
        }
        if (tt >= seq_len) tt -= seq_len;
    };
    int token = static_cast<int>(row / heads);
    int h = static_cast<int>(row - static_cast<int64_t>(token) * heads);
    int t = token % seq_len;
    // the gain of this lane's elements, as fp32 pairs
    uint64_t ga[4], gb[4];
    unpack4x2(*reinterpret_cast<const uint4*>(gamma + 8 * q), ga);
    unpack4x2(*reinterpret_cast<const uint4*>(gamma + 64 + 8 * q), gb);
    uint64_t acca[4] = {0, 0, 0, 0}, accb[4] = {0, 0, 0, 0};
    const uint4 zero = make_uint4(0, 0, 0, 0);
    auto load_row = [&](int64_t r, int tok, int hh, uint4& a, uint4& b, uint4& da, uint4& db) {
        if (r < rows)
        {
            const bf16* xr = x + static_cast<int64_t>(tok) * ldx + hh * 128;
            a = *reinterpret_cast<const uint4*>(xr + 8 * q);
            b = *reinterpret_cast<const uint4*>(xr + 64 + 8 * q);
            if (dyf != nullptr)
            {
                const float* gf = dyf + static_cast<int64_t>(tok) * lddy + hh * 128;
                auto round8 = [&](const float* src) {
                    const float4 u = *reinterpret_cast<const float4*>(src);
                    const float4 w = *reinterpret_cast<const float4*>(src + 4);
                    const __nv_bfloat162 p0 = __floats2bfloat162_rn(u.x * dy_scale, u.y * dy_scale);
                    const __nv_bfloat162 p1 = __floats2bfloat162_rn(u.z * dy_scale, u.w * dy_scale);
                    const __nv_bfloat162 p2 = __floats2bfloat162_rn(w.x * dy_scale, w.y * dy_scale);
                    const __nv_bfloat162 p3 = __floats2bfloat162_rn(w.z * dy_scale, w.w * dy_scale);
                    return make_uint4(*reinterpret_cast<const uint32_t*>(&p0),
                                      *reinterpret_cast<const uint32_t*>(&p1),
                                      *reinterpret_cast<const uint32_t*>(&p2),
                                      *reinterpret_cast<const uint32_t*>(&p3));
                };
                da = round8(gf + 8 * q);
                db = round8(gf + 64 + 8 * q);
            }
            else
            {
                const bf16* gr = dy + static_cast<int64_t>(tok) * lddy + hh * 128;
                da = *reinterpret_cast<const uint4*>(gr + 8 * q);
                db = *reinterpret_cast<const uint4*>(gr + 64 + 8 * q);
            }
        }
        else
        {
            a = b = da = db = zero;
        }
    };
    uint4 ca, cb, cda, cdb;
    load_row(row, token, h, ca, cb, cda, cdb);
    int ntok = token, nh = h, nt = t;
    advance(ntok, nh, nt);
    // every lane of a warp runs the same number of steps (the group sums shuffle across rows)
    const int64_t wfirst = row - (lane >> 3);
    const int64_t iters = wfirst < rows ? (rows - wfirst + stride - 1) / stride : 0;
    constexpr uint64_t kSign = 0x8000000080000000ull;
    for (int64_t k = 0; k < iters; ++k)
    {
        uint4 na, nb, nda, ndb;
        load_row(row + stride, ntok, nh, na, nb, nda, ndb);
        const ulonglong2* cp = reinterpret_cast<const ulonglong2*>(cosv + static_cast<int64_t>(t) * 128 + 8 * q);
        const ulonglong2* sp = reinterpret_cast<const ulonglong2*>(sinv + static_cast<int64_t>(t) * 128 + 8 * q);
        const ulonglong2 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
        const uint64_t cs[4] = {c0.x, c0.y, c1.x, c1.y};
        const uint64_t sn[4] = {s0.x, s0.y, s1.x, s1.y};
        uint64_t a[4], b[4], ra[4], rb[4];
        {
            uint64_t da[4], db[4];
            unpack4x2(cda, da);
            unpack4x2(cdb, db);
#pragma unroll
            for (int j = 0; j < 4; ++j)
            {
                // rotation by -theta: the gradient at the normed-and-scaled value
                ra[j] = fma2(db[j], sn[j], mul2(da[j], cs[j]));
                rb[j] = fma2(da[j], sn[j] ^ kSign, mul2(db[j], cs[j]));
            }
        }
        unpack4x2(ca, a);
        unpack4x2(cb, b);
        uint64_t ss2 = 0, w2 = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j)
        {
            ss2 = fma2(a[j], a[j], ss2);
            ss2 = fma2(b[j], b[j], ss2);
            w2 = fma2(mul2(ra[j], ga[j]), a[j], w2);
            w2 = fma2(mul2(rb[j], gb[j]), b[j], w2);
        }
        float s0f, s1f, w0f, w1f;
        upk(ss2, s0f, s1f);
        upk(w2, w0f, w1f);
        const float ss = group8_sum(s0f + s1f);
        const float w = group8_sum(w0f + w1f);
        if (row < rows)
        {
            const float inv = 1.0f / sqrtf(ss / 128.0f + eps);
            const float coupling = w * inv * inv * inv / 128.0f;
            const uint64_t inv2 = pk(inv, inv), ncp2 = pk(-coupling, -coupling);
            float oa[8], ob[8];
#pragma unroll
            for (int j = 0; j < 4; ++j)
            {
                acca[j] = fma2(ra[j], mul2(a[j], inv2), acca[j]);
                accb[j] = fma2(rb[j], mul2(b[j], inv2), accb[j]);
                upk(fma2(mul2(ra[j], ga[j]), inv2, mul2(a[j], ncp2)), oa[2 * j], oa[2 * j + 1]);
                upk(fma2(mul2(rb[j], gb[j]), inv2, mul2(b[j], ncp2)), ob[2 * j], ob[2 * j + 1]);
            }
            bf16* out = dx + static_cast<int64_t>(token) * lddx + h * 128;
            store16(out + 8 * q, oa);
            store16(out + 64 + 8 * q, ob);
        }
        ca = na;
        cb = nb;
        cda = nda;
        cdb = ndb;
        row += stride;
        token = ntok;
        h = nh;
        t = nt;
        advance(ntok, nh, nt);
    }
    if (partials != nullptr)
    {
#pragma unroll
        for (int j = 0; j < 4; ++j)
        {
            upk(acca[j], part[slot][8 * q + 2 * j], part[slot][8 * q + 2 * j + 1]);
            upk(accb[j], part[slot][64 + 8 * q + 2 * j], part[slot][64 + 8 * q + 2 * j + 1]);
        }
        __syncthreads();
        for (int i = threadIdx.x; i < 128; i += blockDim.x)
        {
            float s = 0.0f;
            for (int k2 = 0; k2 < kWarps * 4; ++k2)
            {
                s += part[k2][i];
            }
            partials[static_cast<size_t>(blk) * 128 + i] = s;
        }
    }
}

// ---- QK-norm + RoPE ---------------------------------------------------------------------------
// One warp per (token, head). Lane handles rotation pairs (p, p+1) at p = 2*lane + 64*k, i.e.
// elements p, p+1 and their partners p+half, p+1+half. Requires head_dim % 4 == 0.
template <typename T>
__device__ __forceinline__ void load2(const T* p, float& a, float& b)
{
    if constexpr (sizeof(T) == 4)
    {
        const float2 v = *reinterpret_cast<const float2*>(p);
        a = v.x;
        b = v.y;
    }
    else
    {
        const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(p);
        a = __low2float(v);
        b = __high2float(v);
    }
}

template <typename T>
__device__ __forceinline__ void store2(T* p, float a, float b)
{
    if constexpr (sizeof(T) == 4)
    {
        *reinterpret_cast<float2*>(p) = make_float2(a, b);
    }
    else
    {
        *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
    }
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32)
qknorm_rope_fwd_kernel(const T* __restrict__ x, int64_t ldx, const T* __restrict__ gamma,
                       const float* __restrict__ cosv, const float* __restrict__ sinv,
                       T* __restrict__ y, int64_t ldy, int64_t tokens, int heads, int seq_len,
                       int dh, float eps)
{
    const int lane = threadIdx.x & 31;
    const int half = dh / 2;
    const int64_t rows = tokens * heads;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kWarps;
    for (int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5); row < rows;
         row += stride)
    {
        const int64_t token = row / heads;
        const int head = static_cast<int>(row - token * heads);
        const int t = static_cast<int>(token % seq_len);
        const T* xr = x + token * ldx + static_cast<int64_t>(head) * dh;
        T* yr = y + token * ldy + static_cast<int64_t>(head) * dh;
        float ss = 0.0f;
        for (int p = 2 * lane; p < half; p += 64)
        {
            float a0, a1, b0, b1;
            load2(xr + p, a0, a1);
            load2(xr + p + half, b0, b1);
            ss += a0 * a0 + a1 * a1 + b0 * b0 + b1 * b1;
        }
        ss = warp_sum(ss);
        const float r = sqrtf(ss / static_cast<float>(dh) + eps);
        const float* cr = cosv + static_cast<int64_t>(t) * dh;
        const float* sr = sinv + static_cast<int64_t>(t) * dh;
        for (int p = 2 * lane; p < half; p += 64)
        {
            float a0, a1, b0, b1, ga0, ga1, gb0, gb1;
            load2(xr + p, a0, a1);
            load2(xr + p + half, b0, b1);
            load2(gamma + p, ga0, ga1);
            load2(gamma + p + half, gb0, gb1);
            a0 = (a0 / r) * ga0;
            a1 = (a1 / r) * ga1;
            b0 = (b0 / r) * gb0;
            b1 = (b1 / r) * gb1;
            const float c0 = cr[p], c1 = cr[p + 1], s0 = sr[p], s1 = sr[p + 1];
            store2(yr + p, a0 * c0 - b0 * s0, a1 * c1 - b1 * s1);
            store2(yr + p + half, b0 * c0 + a0 * s0, b1 * c1 + a1 * s1);
        }
    }
}

// Shared memory: [kWarps][dh] fp32 gain-gradient rows.
template <typename T>
__global__ void __launch_bounds__(kWarps * 32)
qknorm_rope_bwd_kernel(const T* __restrict__ x, int64_t ldx, const T* __restrict__ gamma,
                       const float* __restrict__ cosv, const float* __restrict__ sinv,
                       const T* __restrict__ dy, int64_t lddy, T* __restrict__ dx, int64_t lddx,
                       float* __restrict__ partials, int64_t tokens, int heads, int seq_len, int dh,
                       float eps)
{
    extern __shared__ float smem[];
    const int lane = threadIdx.x & 31;
    const int wid = threadIdx.x >> 5;
    const int half = dh / 2;
    float* mine = smem + static_cast<size_t>(wid) * dh;
    if (partials != nullptr)
    {
        for (int i = lane; i < dh; i += 32)
        {
            mine[i] = 0.0f;
        }
    }
    const int64_t rows = tokens * heads;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kWarps;
    for (int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + wid; row < rows; row += stride)
    {
        const int64_t token = row / heads;
        const int head = static_cast<int>(row - token * heads);
        const int t = static_cast<int>(token % seq_len);
        const T* xr = x + token * ldx + static_cast<int64_t>(head) * dh;
        const T* gr = dy + token * lddy + static_cast<int64_t>(head) * dh;
        T* out = dx + token * lddx + static_cast<int64_t>(head) * dh;
        const float* cr = cosv + static_cast<int64_t>(t) * dh;
        const float* sr = sinv + static_cast<int64_t>(t) * dh;
        float ss = 0.0f, w = 0.0f;
        for (int p = 2 * lane; p < half; p += 64)
        {
            float a0, a1, b0, b1, da0, da1, db0, db1, ga0, ga1, gb0, gb1;
            load2(xr + p, a0, a1);
            load2(xr + p + half, b0, b1);
            load2(gr + p, da0, da1);
            load2(gr + p + half, db0, db1);
            load2(gamma + p, ga0, ga1);
            load2(gamma + p + half, gb0, gb1);
            const float c0 = cr[p], c1 = cr[p + 1], s0 = sr[p], s1 = sr[p + 1];
            // rotation by -theta: the gradient at the normed-and-scaled value
            const float na0 = da0 * c0 + db0 * s0, nb0 = db0 * c0 - da0 * s0;
            const float na1 = da1 * c1 + db1 * s1, nb1 = db1 * c1 - da1 * s1;
            ss += a0 * a0 + a1 * a1 + b0 * b0 + b1 * b1;
            w += (na0 * ga0) * a0 + (na1 * ga1) * a1 + (nb0 * gb0) * b0 + (nb1 * gb1) * b1;
        }
        ss = warp_sum(ss);
        w = warp_sum(w);
        const float nf = static_cast<float>(dh);
        const float r = sqrtf(ss / nf + eps);
        const float coupling = w / (nf * r * r * r);
        for (int p = 2 * lane; p < half; p += 64)
        {
            float a0, a1, b0, b1, da0, da1, db0, db1, ga0, ga1, gb0, gb1;
            load2(xr + p, a0, a1);
            load2(xr + p + half, b0, b1);
            load2(gr + p, da0, da1);
            load2(gr + p + half, db0, db1);
            load2(gamma + p, ga0, ga1);
            load2(gamma + p + half, gb0, gb1);
            const float c0 = cr[p], c1 = cr[p + 1], s0 = sr[p], s1 = sr[p + 1];
            const float na0 = da0 * c0 + db0 * s0, nb0 = db0 * c0 - da0 * s0;
            const float na1 = da1 * c1 + db1 * s1, nb1 = db1 * c1 - da1 * s1;
            if (partials != nullptr)
            {
                mine[p] += na0 * (a0 / r);
                mine[p + 1] += na1 * (a1 / r);
                mine[p + half] += nb0 * (b0 / r);
                mine[p + 1 + half] += nb1 * (b1 / r);
            }
            store2(out + p, (na0 * ga0) / r - a0 * coupling, (na1 * ga1) / r - a1 * coupling);
            store2(out + p + half, (nb0 * gb0) / r - b0 * coupling,
                   (nb1 * gb1) / r - b1 * coupling);
        }
    }
    if (partials != nullptr)
    {
        __syncthreads();
        for (int i = threadIdx.x; i < dh; i += blockDim.x)
        {
            float s = 0.0f;
            for (int k = 0; k < kWarps; ++k)
            {
                s += smem[static_cast<size_t>(k) * dh + i];
            }
            partials[static_cast<size_t>(blockIdx.x) * dh + i] = s;
        }
    }
}

// Plain RoPE over contiguous [lanes, T, Dh]; one thread per rotation pair.
template <typename T>
__global__ void rope_kernel(const T* __restrict__ x, T* __restrict__ y,
                            const float* __restrict__ cosv, const float* __restrict__ sinv,
                            int64_t pairs_total, int seq_len, int dh, float sign)
{
    const int half = dh / 2;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
         idx < pairs_total; idx += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        const int64_t row = idx / half;
        const int i = static_cast<int>(idx - row * half);
        const int t = static_cast<int>(row % seq_len);
        const float c = cosv[static_cast<int64_t>(t) * dh + i];
        const float s = sign * sinv[static_cast<int64_t>(t) * dh + i];
        const float a = to_f32(x[row * dh + i]);
        const float b = to_f32(x[row * dh + i + half]);
        y[row * dh + i] = from_f32<T>(a * c - b * s);
        y[row * dh + i + half] = from_f32<T>(b * c + a * s);
    }
}

bool vec_ok(const void* p, int64_t ld, int n, size_t esize)
{
    const int64_t v = 16 / static_cast<int64_t>(esize);
    return p == nullptr || (aligned16(p) && (ld % v) == 0 && (n % v) == 0);
}

template <typename T>
int launch_rms_fwd(const void* x, int64_t ldx, const void* gamma, void* y, int64_t ldy,
                   int64_t rows, int64_t n, float eps, cudaStream_t s)
{
    if constexpr (sizeof(T) == 2)
    {
        const int rc = rms_fwd_stream(static_cast<const bf16*>(x), ldx, nullptr, 0,
                                      static_cast<const bf16*>(gamma), static_cast<bf16*>(y), ldy,
                                      nullptr, 0, rows, n, eps, s);
        if (rc != -1)
        {
            return rc;
        }
    }
    const bool vec = vec_ok(x, ldx, static_cast<int>(n), sizeof(T)) &&
                     vec_ok(y, ldy, static_cast<int>(n), sizeof(T)) &&
                     vec_ok(gamma, n, static_cast<int>(n), sizeof(T));
    const unsigned grid = static_cast<unsigned>(
        std::min<int64_t>((rows + kWarps - 1) / kWarps, static_cast<int64_t>(sm_count()) * 16));
    constexpr int64_t V = 16 / sizeof(T);
    const int64_t chunks = n % (32 * V) == 0 ? n / (32 * V) : 0;
    const int64_t tpr = n % V == 0 ? n / V : 0;
    if (vec && (tpr == 64 || tpr == 128 || tpr == 256 || tpr == 512))
    {
        // 512 / tpr rows per block step; enough blocks for four per SM
        const int64_t per = kRowThreads / tpr;
        const unsigned g2 = static_cast<unsigned>(
            std::max<int64_t>(1, std::min<int64_t>((rows + per - 1) / per, static_cast<int64_t>(sm_count()) * 4)));
        const T* xp = static_cast<const T*>(x);
        const T* gp = static_cast<const T*>(gamma);
        T* yp = static_cast<T*>(y);
        if (tpr == 64)
            rmsnorm_fwd_rows_kernel<T, 64><<<g2, kRowThreads, 0, s>>>(xp, ldx, gp, yp, ldy, rows, eps);
        else if (tpr == 128)
            rmsnorm_fwd_rows_kernel<T, 128><<<g2, kRowThreads, 0, s>>>(xp, ldx, gp, yp, ldy, rows, eps);
        else if (tpr == 256)
            rmsnorm_fwd_rows_kernel<T, 256><<<g2, kRowThreads, 0, s>>>(xp, ldx, gp, yp, ldy, rows, eps);
        else
            rmsnorm_fwd_rows_kernel<T, 512><<<g2, kRowThreads, 0, s>>>(xp, ldx, gp, yp, ldy, rows, eps);
    }
    else if (vec && (chunks == 1 || chunks == 2 || chunks == 4 || chunks == 8))
    {
        const T* xp = static_cast<const T*>(x);
        const T* gp = static_cast<const T*>(gamma);
        T* yp = static_cast<T*>(y);
        if (chunks == 1)
            rmsnorm_fwd_reg_kernel<T, 1><<<grid, kWarps * 32, 0, s>>>(xp, ldx, gp, yp, ldy, rows, eps);
        else if (chunks == 2)
            rmsnorm_fwd_reg_kernel<T, 2><<<grid, kWarps * 32, 0, s>>>(xp, ldx, gp, yp, ldy, rows, eps);
        else if (chunks == 4)
            rmsnorm_fwd_reg_kernel<T, 4><<<grid, kWarps * 32, 0, s>>>(xp, ldx, gp, yp, ldy, rows, eps);
        else
            rmsnorm_fwd_reg_kernel<T, 8><<<grid, kWarps * 32, 0, s>>>(xp, ldx, gp, yp, ldy, rows, eps);
    }
    else if (vec)
    {
        rmsnorm_fwd_kernel<T, true><<<grid, kWarps * 32, 0, s>>>(
            static_cast<const T*>(x), ldx, static_cast<const T*>(gamma), static_cast<T*>(y), ldy,
            rows, static_cast<int>(n), eps);
    }
    else
    {
        rmsnorm_fwd_kernel<T, false><<<grid, kWarps * 32, 0, s>>>(
            static_cast<const T*>(x), ldx, static_cast<const T*>(gamma), static_cast<T*>(y), ldy,
            rows, static_cast<int>(n), eps);
    }
    count_launch();
    return check_launch("veda_rmsnorm_fwd");
}

template <typename T>
int launch_rms_bwd(const void* x, int64_t ldx, const void* gamma, const void* dy, int64_t lddy,
                   const void* dresid, int64_t ldr, void* dx, int64_t lddx, float* dgamma,
                   void* ws, int64_t rows, int64_t n, float eps, cudaStream_t s)
{
    const int ni = static_cast<int>(n);
    const bool vec = vec_ok(x, ldx, ni, sizeof(T)) && vec_ok(dy, lddy, ni, sizeof(T)) &&
                     vec_ok(dx, lddx, ni, sizeof(T)) && vec_ok(dresid, ldr, ni, sizeof(T)) &&
                     vec_ok(gamma, n, ni, sizeof(T));
    const int grid = norm_bwd_grid(rows);
    float* partials = dgamma != nullptr ? static_cast<float*>(ws) : nullptr;
    if constexpr (sizeof(T) == 2)
    {
        int blocks = 0;
        const int rc = rms_bwd_stream(static_cast<const bf16*>(x), ldx, static_cast<const bf16*>(gamma),
                                      static_cast<const bf16*>(dy), lddy, static_cast<const bf16*>(dresid),
                                      ldr, static_cast<bf16*>(dx), lddx, partials, grid, rows, n, eps, s,
                                      &blocks);
        if (rc != -1)
        {
            if (rc == VEDA_OK && partials != nullptr)
            {
                return launch_reduce_partials(partials, blocks, ni, dgamma, s);
            }
            return rc;
        }
    }
    const size_t smem = partials != nullptr ? static_cast<size_t>(kWarps) * n * sizeof(float) : 0;
    constexpr int64_t V = 16 / sizeof(T);
    const int64_t chunks = n % (32 * V) == 0 ? n / (32 * V) : 0;
    const T* xp = static_cast<const T*>(x);
    const T* gp = static_cast<const T*>(gamma);
    const T* dyp = static_cast<const T*>(dy);
    const T* rp = static_cast<const T*>(dresid);
    T* dxp = static_cast<T*>(dx);
    auto allow_smem = [&](auto kernel) {
        if (smem > 48 * 1024)
        {
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem));
        }
    };
    const int64_t tpr = n % V == 0 ? n / V : 0;
    if (vec && (tpr == 64 || tpr == 128 || tpr == 256 || tpr == 512))
    {
        // same grid (and partials layout) as the other backward kernels: one partial row per block
        const size_t psmem = partials != nullptr ? static_cast<size_t>(kRowThreads) * V * sizeof(float) : 0;
        auto launch_rows = [&](auto kernel) {
            kernel<<<grid, kRowThreads, psmem, s>>>(xp, ldx, gp, dyp, lddy, rp, ldr, dxp, lddx,
                                                   partials, rows, eps);
        };
        if (tpr == 64) launch_rows(rmsnorm_bwd_rows_kernel<T, 64>);
        else if (tpr == 128) launch_rows(rmsnorm_bwd_rows_kernel<T, 128>);
        else if (tpr == 256) launch_rows(rmsnorm_bwd_rows_kernel<T, 256>);
        else launch_rows(rmsnorm_bwd_rows_kernel<T, 512>);
    }
    else if (vec && (chunks == 1 || chunks == 2 || chunks == 4 || chunks == 8))
    {
        auto launch_reg = [&](auto kernel) {
            allow_smem(kernel);
            kernel<<<grid, kWarps * 32, smem, s>>>(xp, ldx, gp, dyp, lddy, rp, ldr, dxp, lddx,
                                                  partials, rows, eps);
        };
        if (chunks == 1) launch_reg(rmsnorm_bwd_reg_kernel<T, 1>);
        else if (chunks == 2) launch_reg(rmsnorm_bwd_reg_kernel<T, 2>);
        else if (chunks == 4) launch_reg(rmsnorm_bwd_reg_kernel<T, 4>);
        else launch_reg(rmsnorm_bwd_reg_kernel<T, 8>);
    }
    else
    {
        auto kernel = vec ? rmsnorm_bwd_kernel<T, true> : rmsnorm_bwd_kernel<T, false>;
        allow_smem(kernel);
        kernel<<<grid, kWarps * 32, smem, s>>>(xp, ldx, gp, dyp, lddy, rp, ldr, dxp, lddx,
                                              partials, rows, ni, eps);
    }
    count_launch();
    const int rc = check_launch("veda_rmsnorm_bwd");
    if (rc == VEDA_OK && partials != nullptr)
    {
        return launch_reduce_partials(partials, grid, ni, dgamma, s);
    }
    return rc;
}

} // namespace
} // namespace veda::cuda

using namespace veda::cuda;

extern "C" size_t veda_rmsnorm_bwd_workspace(int64_t rows, int64_t n)
{
    return static_cast<size_t>(norm_bwd_grid(rows)) * static_cast<size_t>(n) * sizeof(float);
}

extern "C" int veda_rmsnorm_fwd(const void* x, int64_t ldx, const void* gamma, void* y,
                                int64_t ldy, int64_t rows, int64_t n, float eps, int dtype,
                                veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype), "unknown dtype");
    VEDA_REQUIRE(rows >= 0 && n > 0 && ldx >= n && ldy >= n, "bad shape or leading dimension");
    VEDA_REQUIRE(n <= (1 << 24), "row too long");
    if (rows == 0)
    {
        return VEDA_OK;
    }
    VEDA_REQUIRE(x != nullptr && y != nullptr, "null pointer");
    return dtype == VEDA_BF16
               ? launch_rms_fwd<bf16>(x, ldx, gamma, y, ldy, rows, n, eps, stream)
               : launch_rms_fwd<float>(x, ldx, gamma, y, ldy, rows, n, eps, stream);
}

extern "C" int veda_add_rmsnorm_fwd(const void* x, int64_t ldx, const void* r, int64_t ldr,
                                    const void* gamma, void* sum, int64_t lds, void* y,
                                    int64_t ldy, int64_t rows, int64_t n, float eps, int dtype,
                                    veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype), "unknown dtype");
    VEDA_REQUIRE(rows >= 0 && n > 0 && ldx >= n && ldr >= n && lds >= n && ldy >= n,
                 "bad shape or leading dimension");
    VEDA_REQUIRE(n <= (1 << 24), "row too long");
    if (rows == 0)
    {
        return VEDA_OK;
    }
    VEDA_REQUIRE(x != nullptr && r != nullptr && sum != nullptr && y != nullptr, "null pointer");
    if (dtype == VEDA_BF16)
    {
        const int rc = rms_fwd_stream(static_cast<const bf16*>(x), ldx, static_cast<const bf16*>(r), ldr,
                                      static_cast<const bf16*>(gamma), static_cast<bf16*>(y), ldy,
                                      static_cast<bf16*>(sum), lds, rows, n, eps, stream);
        if (rc != -1)
        {
            return rc;
        }
    }
    const unsigned grid = grid_for(rows * n, 256);
    if (dtype == VEDA_BF16)
        add_rows_kernel<bf16><<<grid, 256, 0, stream>>>(static_cast<const bf16*>(x), ldx,
                                                        static_cast<const bf16*>(r), ldr,
                                                        static_cast<bf16*>(sum), lds, rows, n);
    else
        add_rows_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float*>(x), ldx,
                                                         static_cast<const float*>(r), ldr,
                                                         static_cast<float*>(sum), lds, rows, n);
    count_launch();
    const int rc = check_launch("veda_add_rmsnorm_fwd");
    if (rc != VEDA_OK)
    {
        return rc;
    }
    return veda_rmsnorm_fwd(sum, lds, gamma, y, ldy, rows, n, eps, dtype, stream);
}

extern "C" int veda_rmsnorm_bwd(const void* x, int64_t ldx, const void* gamma, const void* dy,
                                int64_t lddy, const void* dresid, int64_t ldr, void* dx,
                                int64_t lddx, float* dgamma, void* workspace,
                                size_t workspace_bytes, int64_t rows, int64_t n, float eps,
                                int dtype, veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype), "unknown dtype");
    VEDA_REQUIRE(rows >= 0 && n > 0 && ldx >= n && lddy >= n && lddx >= n, "bad shape");
    VEDA_REQUIRE(dresid == nullptr || ldr >= n, "bad residual leading dimension");
    VEDA_REQUIRE(static_cast<size_t>(kWarps) * n * sizeof(float) <= 200 * 1024 || dgamma == nullptr,
                 "row too long for the gain reduction");
    if (rows == 0)
    {
        return VEDA_OK;
    }
    VEDA_REQUIRE(x != nullptr && dy != nullptr && dx != nullptr, "null pointer");
    if (dgamma != nullptr)
    {
        VEDA_REQUIRE(gamma != nullptr, "dgamma needs gamma");
        VEDA_REQUIRE(workspace != nullptr &&
                         workspace_bytes >= veda_rmsnorm_bwd_workspace(rows, n),
                     "workspace too small (see veda_rmsnorm_bwd_workspace)");
    }
    return dtype == VEDA_BF16
               ? launch_rms_bwd<bf16>(x, ldx, gamma, dy, lddy, dresid, ldr, dx, lddx, dgamma,
                                      workspace, rows, n, eps, stream)
               : launch_rms_bwd<float>(x, ldx, gamma, dy, lddy, dresid, ldr, dx, lddx, dgamma,
                                       workspace, rows, n, eps, stream);
}

extern "C" size_t veda_qknorm_rope_bwd_workspace(int64_t tokens, int64_t heads, int64_t head_dim)
{
    return static_cast<size_t>(qk_bwd_grid(tokens * heads)) * static_cast<size_t>(head_dim) *
           sizeof(float);
}

namespace
{
// The eight-lanes-per-row kernels need bf16, head_dim 128 and 16-byte aligned rows and tables.
bool d128_ok(const void* x, int64_t ldx, const void* gamma, const float* c, const float* s,
             const void* y, int64_t ldy, int64_t head_dim, int dtype)
{
    return dtype == VEDA_BF16 && head_dim == 128 && aligned16(x) && aligned16(y) &&
           aligned16(gamma) && aligned16(c) && aligned16(s) && ldx % 8 == 0 && ldy % 8 == 0;
}

int qk_checks(const void* x, int64_t ldx, const void* gamma, const float* c, const float* s,
              int64_t tokens, int64_t heads, int64_t seq_len, int64_t dh, int dtype)
{
    VEDA_REQUIRE(valid_dtype(dtype), "unknown dtype");
    VEDA_REQUIRE(tokens >= 0 && heads > 0 && seq_len > 0 && dh > 0, "bad shape");
    VEDA_REQUIRE(dh % 4 == 0 && dh <= 4096, "head_dim must be a multiple of 4 (<= 4096)");
    VEDA_REQUIRE(ldx >= heads * dh, "leading dimension smaller than heads * head_dim");
    VEDA_REQUIRE(ldx % 2 == 0, "leading dimension must be even");
    VEDA_REQUIRE(x != nullptr && gamma != nullptr && c != nullptr && s != nullptr,
                 "null pointer");
    VEDA_REQUIRE((reinterpret_cast<uintptr_t>(x) % (2 * dtype_size(dtype))) == 0,
                 "misaligned input");
    return VEDA_OK;
}
} // namespace

extern "C" int veda_qknorm_rope_fwd(const void* x, int64_t ldx, const void* gamma,
                                    const float* cosv, const float* sinv, void* y, int64_t ldy,
                                    int64_t tokens, int64_t heads, int64_t seq_len,
                                    int64_t head_dim, float eps, int dtype, veda_stream_t stream)
{
    int rc = qk_checks(x, ldx, gamma, cosv, sinv, tokens, heads, seq_len, head_dim, dtype);
    if (rc != VEDA_OK)
    {
        return rc;
    }
    VEDA_REQUIRE(y != nullptr && ldy >= heads * head_dim && ldy % 2 == 0, "bad output");
    if (tokens == 0)
    {
        return VEDA_OK;
    }
    const int64_t rows = tokens * heads;
    const unsigned grid = static_cast<unsigned>(
        std::min<int64_t>((rows + kWarps - 1) / kWarps, static_cast<int64_t>(sm_count()) * 16));
    if (d128_ok(x, ldx, gamma, cosv, sinv, y, ldy, head_dim, dtype) && rows < (1ll << 31))
    {
        const unsigned g4 = static_cast<unsigned>(std::min<int64_t>(
            (rows + 4 * kWarps - 1) / (4 * kWarps), static_cast<int64_t>(sm_count()) * 4));
        const QkFwdSet one{static_cast<const bf16*>(x), static_cast<const bf16*>(gamma),
                           static_cast<bf16*>(y), ldx, ldy, static_cast<int>(heads),
                           static_cast<int>(g4)};
        const QkFwdSet none{nullptr, nullptr, nullptr, 0, 0, 1, 0};
        qknorm_rope_fwd_d128_kernel<<<g4, kWarps * 32, 0, stream>>>(one, none, cosv, sinv, tokens,
                                                                   static_cast<int>(seq_len), eps);
    }
    else if (dtype == VEDA_BF16)
    {
        qknorm_rope_fwd_kernel<bf16><<<grid, kWarps * 32, 0, stream>>>(
            static_cast<const bf16*>(x), ldx, static_cast<const bf16*>(gamma), cosv, sinv,
            static_cast<bf16*>(y), ldy, tokens, static_cast<int>(heads),
            static_cast<int>(seq_len), static_cast<int>(head_dim), eps);
    }
    else
    {
        qknorm_rope_fwd_kernel<float><<<grid, kWarps * 32, 0, stream>>>(
            static_cast<const float*>(x), ldx, static_cast<const float*>(gamma), cosv, sinv,
            static_cast<float*>(y), ldy, tokens, static_cast<int>(heads),
            static_cast<int>(seq_len), static_cast<int>(head_dim), eps);
    }
    count_launch();
    return check_launch("veda_qknorm_rope_fwd");
}

extern "C" int veda_qknorm_rope_fwd_qk(const void* xq, const void* xk, int64_t ldx,
                                       const void* q_gamma, const void* k_gamma, const float* cosv,
                                       const float* sinv, void* yq, int64_t ldyq, void* yk,
                                       int64_t ldyk, int64_t tokens, int64_t heads,
                                       int64_t kv_heads, int64_t seq_len, int64_t head_dim,
                                       float eps, int dtype, veda_stream_t stream)
{
    int rc = qk_checks(xq, ldx, q_gamma, cosv, sinv, tokens, heads, seq_len, head_dim, dtype);
    if (rc == VEDA_OK)
    {
        rc = qk_checks(xk, ldx, k_gamma, cosv, sinv, tokens, kv_heads, seq_len, head_dim, dtype);
    }
    if (rc != VEDA_OK)
    {
        return rc;
    }
    VEDA_REQUIRE(yq != nullptr && yk != nullptr && ldyq >= heads * head_dim &&
                     ldyk >= kv_heads * head_dim && ldyq % 2 == 0 && ldyk % 2 == 0,
                 "bad output");
    if (tokens == 0)
    {
        return VEDA_OK;
    }
    const bool one_launch = d128_ok(xq, ldx, q_gamma, cosv, sinv, yq, ldyq, head_dim, dtype) &&
                            d128_ok(xk, ldx, k_gamma, cosv, sinv, yk, ldyk, head_dim, dtype) &&
                            tokens * std::max(heads, kv_heads) < (1ll << 31);
    if (!one_launch)
    {
        rc = veda_qknorm_rope_fwd(xq, ldx, q_gamma, cosv, sinv, yq, ldyq, tokens, heads, seq_len,
                                  head_dim, eps, dtype, stream);
        if (rc != VEDA_OK)
        {
            return rc;
        }
        return veda_qknorm_rope_fwd(xk, ldx, k_gamma, cosv, sinv, yk, ldyk, tokens, kv_heads,
                                    seq_len, head_dim, eps, dtype, stream);
    }
    // blocks in proportion to the rows (both sets finish together), at most four per SM in all
    const int64_t per = 4 * kWarps, total = static_cast<int64_t>(sm_count()) * 4;
    int64_t bq = total * heads / (heads + kv_heads);
    bq = std::max<int64_t>(1, std::min<int64_t>(bq, (tokens * heads + per - 1) / per));
    const int64_t bk =
        std::max<int64_t>(1, std::min<int64_t>(total - bq, (tokens * kv_heads + per - 1) / per));
    const QkFwdSet sq{static_cast<const bf16*>(xq), static_cast<const bf16*>(q_gamma),
                      static_cast<bf16*>(yq), ldx, ldyq, static_cast<int>(heads), static_cast<int>(bq)};
    const QkFwdSet sk{static_cast<const bf16*>(xk), static_cast<const bf16*>(k_gamma),
                      static_cast<bf16*>(yk), ldx, ldyk, static_cast<int>(kv_heads), static_cast<int>(bk)};
    return launch("veda_qknorm_rope_fwd_qk", qknorm_rope_fwd_d128_kernel, dim3(static_cast<unsigned>(bq + bk)),
                  dim3(kWarps * 32), 0, stream, sq, sk, cosv, sinv, tokens, static_cast<int>(seq_len),
                  eps);
}

extern "C" int veda_qknorm_rope_bwd(const void* x, int64_t ldx, const void* gamma,
                                    const float* cosv, const float* sinv, const void* dy,
                                    int64_t lddy, void* dx, int64_t lddx, float* dgamma,
                                    void* workspace, size_t workspace_bytes, int64_t tokens,
                                    int64_t heads, int64_t seq_len, int64_t head_dim, float eps,
                                    int dtype, veda_stream_t stream)
{
    int rc = qk_checks(x, ldx, gamma, cosv, sinv, tokens, heads, seq_len, head_dim, dtype);
    if (rc != VEDA_OK)
    {
        return rc;
    }
    VEDA_REQUIRE(dy != nullptr && dx != nullptr && lddy >= heads * head_dim &&
                     lddx >= heads * head_dim && lddy % 2 == 0 && lddx % 2 == 0,
                 "bad gradient operands");
    if (tokens == 0)
    {
        return VEDA_OK;
    }
    if (dgamma != nullptr)
    {
        VEDA_REQUIRE(workspace != nullptr &&
                         workspace_bytes >= veda_qknorm_rope_bwd_workspace(tokens, heads, head_dim),
                     "workspace too small (see veda_qknorm_rope_bwd_workspace)");
    }
    const int64_t rows = tokens * heads;
    const int grid = qk_bwd_grid(rows);
    float* partials = dgamma != nullptr ? static_cast<float*>(workspace) : nullptr;
    const size_t smem = partials != nullptr ? kWarps * head_dim * sizeof(float) : 0;
    if (d128_ok(x, ldx, gamma, cosv, sinv, dy, lddy, head_dim, dtype) &&
        d128_ok(x, ldx, gamma, cosv, sinv, dx, lddx, head_dim, dtype) && rows < (1ll << 31))
    {
        const QkSet one{static_cast<const bf16*>(x), static_cast<const bf16*>(gamma),
                        static_cast<const bf16*>(dy), static_cast<bf16*>(dx), partials, ldx, lddy, lddx,
                        static_cast<int>(heads), grid, nullptr, 1.0f};
        const QkSet none{nullptr, nullptr, nullptr, nullptr, nullptr, 0, 0, 0, 1, 0, nullptr, 1.0f};
        qknorm_rope_bwd_d128_kernel<<<grid, kWarps * 32, 0, stream>>>(
            one, none, cosv, sinv, tokens, static_cast<int>(seq_len), eps);
    }
    else if (dtype == VEDA_BF16)
    {
        qknorm_rope_bwd_kernel<bf16><<<grid, kWarps * 32, smem, stream>>>(
            static_cast<const bf16*>(x), ldx, static_cast<const bf16*>(gamma), cosv, sinv,
            static_cast<const bf16*>(dy), lddy, static_cast<bf16*>(dx), lddx, partials, tokens,
            static_cast<int>(heads), static_cast<int>(seq_len), static_cast<int>(head_dim), eps);
    }
    else
    {
        qknorm_rope_bwd_kernel<float><<<grid, kWarps * 32, smem, stream>>>(
            static_cast<const float*>(x), ldx, static_cast<const float*>(gamma), cosv, sinv,
            static_cast<const float*>(dy), lddy, static_cast<float*>(dx), lddx, partials, tokens,
            static_cast<int>(heads), static_cast<int>(seq_len), static_cast<int>(head_dim), eps);
    }
    count_launch();
    rc = check_launch("veda_qknorm_rope_bwd");
    if (rc == VEDA_OK && partials != nullptr)
    {
        return launch_reduce_partials(partials, grid, static_cast<int>(head_dim), dgamma, stream);
    }
    return rc;
}

namespace
{
// Blocks of a q + k launch: in proportion to their rows (both finish together), each set at least
// one block and at most one per 4 x kWarps rows.
void qk_pair_blocks(int64_t tokens, int64_t heads, int64_t kv_heads, int* gq, int* gk)
{
    const int64_t per = 4 * kWarps;
    const int64_t total = 2LL * sm_count();
    int64_t bq = total * heads / (heads + kv_heads);
    bq = std::max<int64_t>(1, std::min<int64_t>(bq, (tokens * heads + per - 1) / per));
    const int64_t bk =
        std::max<int64_t>(1, std::min<int64_t>(total - bq, (tokens * kv_heads + per - 1) / per));
    *gq = static_cast<int>(bq);
    *gk = static_cast<int>(bk);
}

size_t round256(size_t b) { return (b + 255) / 256 * 256; }
} // namespace

extern "C" size_t veda_qknorm_rope_bwd_qk_workspace(int64_t tokens, int64_t heads, int64_t kv_heads,
                                                    int64_t head_dim)
{
    // room for both forms: one launch over both sets, or the two sets one after the other
    int gq = 1, gk = 1;
    qk_pair_blocks(tokens, heads, kv_heads, &gq, &gk);
    const size_t pair = static_cast<size_t>(gq + gk) * static_cast<size_t>(head_dim) * sizeof(float);
    const size_t split = round256(veda_qknorm_rope_bwd_workspace(tokens, heads, head_dim)) +
                         veda_qknorm_rope_bwd_workspace(tokens, kv_heads, head_dim);
    return std::max(pair, split);
}

extern "C" int veda_qknorm_rope_bwd_qk(const void* xq, const void* xk, int64_t ldx,
                                       const void* q_gamma, const void* k_gamma, const float* cosv,
                                       const float* sinv, const void* dyq, int64_t lddyq,
                                       int dyq_f32, float dyq_scale, const void* dyk, int64_t lddyk,
                                       void* dxq, void* dxk, int64_t lddx, float* dq_gamma,
                                       float* dk_gamma, void* workspace, size_t workspace_bytes,
                                       int64_t tokens, int64_t heads, int64_t kv_heads,
                                       int64_t seq_len, int64_t head_dim, float eps, int dtype,
                                       veda_stream_t stream)
{
    int rc = qk_checks(xq, ldx, q_gamma, cosv, sinv, tokens, heads, seq_len, head_dim, dtype);
    if (rc == VEDA_OK)
    {
        rc = qk_checks(xk, ldx, k_gamma, cosv, sinv, tokens, kv_heads, seq_len, head_dim, dtype);
    }
    if (rc != VEDA_OK)
    {
        return rc;
    }
    VEDA_REQUIRE(dyq != nullptr && dyk != nullptr && dxq != nullptr && dxk != nullptr &&
                     lddyq >= heads * head_dim && lddyk >= kv_heads * head_dim &&
                     lddx >= heads * head_dim && lddx >= kv_heads * head_dim && lddyq % 2 == 0 &&
                     lddyk % 2 == 0 && lddx % 2 == 0,
                 "bad gradient operands");
    if (tokens == 0)
    {
        return VEDA_OK;
    }
    if (dq_gamma != nullptr || dk_gamma != nullptr)
    {
        VEDA_REQUIRE(workspace != nullptr &&
                         workspace_bytes >= veda_qknorm_rope_bwd_qk_workspace(tokens, heads, kv_heads,
                                                                             head_dim),
                     "workspace too small (see veda_qknorm_rope_bwd_qk_workspace)");
    }
    // fp32 dyq rows: 16-byte aligned rows of floats
    const bool dyq_ok = dyq_f32 ? (aligned16(dyq) && lddyq % 4 == 0)
                                : d128_ok(xq, ldx, q_gamma, cosv, sinv, dyq, lddyq, head_dim, dtype);
    const bool one_launch =
        dyq_ok &&
        d128_ok(xq, ldx, q_gamma, cosv, sinv, dxq, lddx, head_dim, dtype) &&
        d128_ok(xk, ldx, k_gamma, cosv, sinv, dyk, lddyk, head_dim, dtype) &&
        d128_ok(xk, ldx, k_gamma, cosv, sinv, dxk, lddx, head_dim, dtype) &&
        tokens * std::max(heads, kv_heads) < (1ll << 31);
    if (!one_launch)
    {
        VEDA_REQUIRE(!dyq_f32, "fp32 q gradients need bf16, head_dim 128 and 16-byte aligned rows");
        // the general kernels: the two sets one after the other, each with its part of the
        // workspace
        const size_t wq = round256(veda_qknorm_rope_bwd_workspace(tokens, heads, head_dim));
        char* w = static_cast<char*>(workspace);
        rc = veda_qknorm_rope_bwd(xq, ldx, q_gamma, cosv, sinv, dyq, lddyq, dxq, lddx, dq_gamma,
                                  w, w != nullptr ? wq : 0, tokens, heads, seq_len, head_dim, eps,
                                  dtype, stream);
        if (rc != VEDA_OK)
        {
            return rc;
        }
        return veda_qknorm_rope_bwd(xk, ldx, k_gamma, cosv, sinv, dyk, lddyk, dxk, lddx, dk_gamma,
                                    w != nullptr ? w + wq : nullptr,
                                    w != nullptr ? workspace_bytes - wq : 0, tokens, kv_heads,
                                    seq_len, head_dim, eps, dtype, stream);
    }
    int gq = 1, gk = 1;
    qk_pair_blocks(tokens, heads, kv_heads, &gq, &gk);
    float* pq = dq_gamma != nullptr ? static_cast<float*>(workspace) : nullptr;
    float* pk = dk_gamma != nullptr ? static_cast<float*>(workspace) + static_cast<size_t>(gq) * 128
                                    : nullptr;
    const QkSet sq{static_cast<const bf16*>(xq), static_cast<const bf16*>(q_gamma),
                   dyq_f32 ? nullptr : static_cast<const bf16*>(dyq), static_cast<bf16*>(dxq), pq,
                   ldx, lddyq, lddx, static_cast<int>(heads), gq,
                   dyq_f32 ? static_cast<const float*>(dyq) : nullptr, dyq_scale};
    const QkSet sk{static_cast<const bf16*>(xk), static_cast<const bf16*>(k_gamma),
                   static_cast<const bf16*>(dyk), static_cast<bf16*>(dxk), pk, ldx, lddyk, lddx,
                   static_cast<int>(kv_heads), gk, nullptr, 1.0f};
    rc = launch("veda_qknorm_rope_bwd_qk", qknorm_rope_bwd_d128_kernel, dim3(gq + gk),
                dim3(kWarps * 32), 0, stream, sq, sk, cosv, sinv, tokens, static_cast<int>(seq_len),
                eps);
    if (rc != VEDA_OK)
    {
        return rc;
    }
    if (pq != nullptr && pk != nullptr)
    {
        return launch_reduce_partials(pq, gq, 128, dq_gamma, stream, pk, gk, dk_gamma);
    }
    if (pq != nullptr)
    {
        return launch_reduce_partials(pq, gq, 128, dq_gamma, stream);
    }
    if (pk != nullptr)
    {
        return launch_reduce_partials(pk, gk, 128, dk_gamma, stream);
    }
    return VEDA_OK;
}

extern "C" int veda_rope(const void* x, void* y, const float* cosv, const float* sinv,
                         int64_t lanes, int64_t seq_len, int64_t head_dim, int inverse, int dtype,
                         veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype), "unknown dtype");
    VEDA_REQUIRE(lanes >= 0 && seq_len > 0 && head_dim > 0 && head_dim % 2 == 0,
                 "head_dim must be even");
    const int64_t pairs = lanes * seq_len * (head_dim / 2);
    if (pairs == 0)
    {
        return VEDA_OK;
    }
    VEDA_REQUIRE(x != nullptr && y != nullptr && cosv != nullptr && sinv != nullptr,
                 "null pointer");
    const unsigned grid = grid_for(pairs, 256);
    const float sign = inverse ? -1.0f : 1.0f;
    if (dtype == VEDA_BF16)
    {
        rope_kernel<bf16><<<grid, 256, 0, stream>>>(static_cast<const bf16*>(x),
                                                    static_cast<bf16*>(y), cosv, sinv, pairs,
                                                    static_cast<int>(seq_len),
                                                    static_cast<int>(head_dim), sign);
    }
    else
    {
        rope_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float*>(x),
                                                     static_cast<float*>(y), cosv, sinv, pairs,
                                                     static_cast<int>(seq_len),
                                                     static_cast<int>(head_dim), sign);
    }
    count_launch();
    return check_launch("veda_rope");
}

// ---- RMSNorm backward without allocation --------------------------------------------------
// Some callers cannot hand veda_rmsnorm_bwd a workspace: cudaMalloc synchronises the whole device
// (a stall in the middle of a pipelined training step) and fails or fragments memory under an
// engine that reserves its device memory up front, and a caller binding this library through a
// plain C ABI (Go via cgo, Java via JNI) may have no allocator of its own on the device.
// veda_rmsnorm_bwd_noalloc takes its scratch — the per-block partial sums of the gain gradient —
// from a fixed array compiled into this library instead.
namespace
{
// 1 Mi floats = 4 MiB, reserved on every GPU that loads the library, until the process exits.
constexpr size_t kNoAllocScratchFloats = size_t{1} << 20;
static __device__ __align__(256) float g_rmsnorm_bwd_scratch[kNoAllocScratchFloats];

// Device address of the array for the current device, looked up on the first call made on
// that device. Host code cannot use the array's name as a device pointer (on the host it names a
// host-side shadow), so the address is obtained with cudaGetSymbolAddress while the device is
// current and cached per device.
float* rmsnorm_scratch_for_current_device(int* status)
{
    static std::mutex mu;
    static float* cached[64] = {nullptr};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64)
    {
        *status = fail(VEDA_ERR_CUDA, "veda_rmsnorm_bwd_noalloc: no current CUDA device");
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (cached[device] == nullptr)
    {
        void* p = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&p, g_rmsnorm_bwd_scratch);
        if (err != cudaSuccess || p == nullptr)
        {
            *status = fail(VEDA_ERR_CUDA, std::string("veda_rmsnorm_bwd_noalloc: "
                                                      "cudaGetSymbolAddress failed: ") +
                                              cudaGetErrorString(err));
            return nullptr;
        }
        cached[device] = static_cast<float*>(p);
    }
    return cached[device];
}
} // namespace

extern "C" int veda_rmsnorm_bwd_noalloc(const void* x, int64_t ldx, const void* gamma,
                                        const void* dy, int64_t lddy, const void* dresid,
                                        int64_t ldr, void* dx, int64_t lddx, float* dgamma,
                                        int64_t rows, int64_t n, float eps, int dtype,
                                        veda_stream_t stream)
{
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
    if (dgamma != nullptr && rows > 0 && n > 0)
    {
        const size_t need = veda_rmsnorm_bwd_workspace(rows, n);
        const size_t have = kNoAllocScratchFloats * sizeof(float);
        if (need > have)
        {
            return fail(VEDA_ERR_INVALID_ARGUMENT,
                        "veda_rmsnorm_bwd_noalloc: rows of " + std::to_string(n) +
                            " need " + std::to_string(need) +
                            " bytes of gain-gradient scratch, above the fixed " +
                            std::to_string(have) + " (use veda_rmsnorm_bwd with a workspace)");
        }
        int status = VEDA_OK;
        scratch = rmsnorm_scratch_for_current_device(&status);
        if (scratch == nullptr)
        {
            return status;
        }
        scratch_bytes = have;
    }
    // Each block writes its own partial sums in full before the reduction reads them, so the
    // scratch needs no clearing between calls.
    return veda_rmsnorm_bwd(x, ldx, gamma, dy, lddy, dresid, ldr, dx, lddx, dgamma, scratch,
                            scratch_bytes, rows, n, eps, dtype, stream);
}
