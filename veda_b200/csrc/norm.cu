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

#include <algorithm>
#include <mutex>

namespace veda::cuda
{
namespace
{

constexpr int kWarps = 8;   // warps per block for the row kernels

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

// dgamma[i] += sum over blocks b (in order) of partials[b][i]
__global__ void reduce_partials_kernel(const float* __restrict__ partials, int blocks, int n,
                                       float* __restrict__ dgamma)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n)
    {
        return;
    }
    float s = 0.0f;
    for (int b = 0; b < blocks; ++b)
    {
        s += partials[static_cast<size_t>(b) * n + i];
    }
    dgamma[i] += s;
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
    const bool vec = vec_ok(x, ldx, static_cast<int>(n), sizeof(T)) &&
                     vec_ok(y, ldy, static_cast<int>(n), sizeof(T)) &&
                     vec_ok(gamma, n, static_cast<int>(n), sizeof(T));
    const unsigned grid = static_cast<unsigned>(
        std::min<int64_t>((rows + kWarps - 1) / kWarps, static_cast<int64_t>(sm_count()) * 16));
    if (vec)
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
    const size_t smem = partials != nullptr ? static_cast<size_t>(kWarps) * n * sizeof(float) : 0;
    auto kernel = vec ? rmsnorm_bwd_kernel<T, true> : rmsnorm_bwd_kernel<T, false>;
    if (smem > 48 * 1024)
    {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    }
    kernel<<<grid, kWarps * 32, smem, s>>>(
        static_cast<const T*>(x), ldx, static_cast<const T*>(gamma), static_cast<const T*>(dy),
        lddy, static_cast<const T*>(dresid), ldr, static_cast<T*>(dx), lddx, partials, rows, ni,
        eps);
    count_launch();
    if (partials != nullptr)
    {
        reduce_partials_kernel<<<(ni + 255) / 256, 256, 0, s>>>(partials, grid, ni, dgamma);
        count_launch();
    }
    return check_launch("veda_rmsnorm_bwd");
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
    return static_cast<size_t>(norm_bwd_grid(tokens * heads)) * static_cast<size_t>(head_dim) *
           sizeof(float);
}

namespace
{
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
    if (dtype == VEDA_BF16)
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
    const int grid = norm_bwd_grid(rows);
    float* partials = dgamma != nullptr ? static_cast<float*>(workspace) : nullptr;
    const size_t smem = partials != nullptr ? kWarps * head_dim * sizeof(float) : 0;
    if (dtype == VEDA_BF16)
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
    if (partials != nullptr)
    {
        const int n = static_cast<int>(head_dim);
        reduce_partials_kernel<<<(n + 255) / 256, 256, 0, stream>>>(partials, grid, n, dgamma);
        count_launch();
    }
    return check_launch("veda_qknorm_rope_bwd");
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
