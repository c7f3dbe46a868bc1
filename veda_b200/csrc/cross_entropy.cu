// Fused softmax cross-entropy: loss rows and dlogits in one streaming pass over the logits.
//
// The reference (src/libs/autograd/Loss.cpp:18-103 with ops::log_softmax,
// src/libs/ops/Softmax.cpp:82-151) materialises fp32 log-probabilities and probabilities for the
// whole [lanes, V] block. Here one CTA owns a row: pass 1 reads it once keeping a running
// (max, sum of exp) per thread (online normaliser), reduced across the CTA; pass 2 re-reads it
// (from L2: 2 CTAs on each of 148 SMs keep 296 rows of 300 KB in flight, held there by L2
// eviction priorities) and writes
//   dlogits = grad_scale * exp(x - max - log(sum))   minus grad_scale at the target,
// the (p - onehot) * g/lanes of Loss.cpp:80-99 with p = exp(log_softmax) as the reference forms
// it. row_loss = -(x_t - max - log(sum)) in fp32; the mean over rows is taken in double by
// veda_mean_f64, as Loss.cpp:52-60 does.
#include "common.cuh"

#include <cfloat>

namespace veda::cuda
{
namespace
{

constexpr int kThreads = 512;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// 2^x with the hardware approximation (relative error ~2^-22; -inf -> 0)
__device__ __forceinline__ float ex2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// (m, s): running max of x log2(e) and sum of 2^(x log2(e) - m)
__device__ __forceinline__ void online_merge(float& m, float& s, float om, float os)
{
    if (om == -INFINITY)
    {
        return;
    }
    if (m == -INFINITY)
    {
        m = om;
        s = os;
        return;
    }
    if (om > m)
    {
        s = s * ex2(m - om) + os;
        m = om;
    }
    else
    {
        s = s + os * ex2(om - m);
    }
}

// Adds a group of N logits to (m, s), m in log2 units: one max over the group (max(x) log2 e =
// max(x log2 e), the scaling being monotone), a rescale only when the group raises the running
// max, then N exponentials 2^(x log2 e - m), each argument formed by one fused multiply-add.
template <int N>
__device__ __forceinline__ void online_add(float& m, float& s, const float (&x)[N])
{
    float gx = x[0];
#pragma unroll
    for (int j = 1; j < N; ++j) gx = fmaxf(gx, x[j]);
    const float gm = gx * kLog2e;
    if (gm > m)
    {
        s = (m == -INFINITY) ? 0.0f : s * ex2(m - gm);
        m = gm;
    }
    if (m == -INFINITY)
    {
        return;   // every value so far is -inf
    }
    float a = 0.0f, b = 0.0f;
#pragma unroll
    for (int j = 0; j < N; j += 2)
    {
        a += ex2(fmaf(x[j], kLog2e, -m));
        if (j + 1 < N) b += ex2(fmaf(x[j + 1], kLog2e, -m));
    }
    s += a + b;
}

// L2 eviction policies: the row's first read marks its lines to be kept for the second pass,
// which reads them for the last time and writes the gradient as first to be evicted, so the
// 2 x 148 rows in flight (90 MB of logits, as much again of gradient) stay in the 126 MB L2.
__device__ __forceinline__ uint64_t l2_policy_keep()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t l2_policy_drop()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

template <typename T>
__device__ __forceinline__ void load16_hint(const T* p, float (&out)[16 / sizeof(T)], uint64_t pol)
{
    uint4 r;
    asm volatile("ld.global.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p), "l"(pol));
    load16(reinterpret_cast<const T*>(&r), out);
}

template <typename T>
__device__ __forceinline__ void store16_hint(T* p, const float (&in)[16 / sizeof(T)], uint64_t pol)
{
    uint4 r;
    store16(reinterpret_cast<T*>(&r), in);
    asm volatile("st.global.L2::cache_hint.v4.u32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(p), "r"(r.x),
                 "r"(r.y), "r"(r.z), "r"(r.w), "l"(pol)
                 : "memory");
}

// One CTA per row (grid-stride). Pass 1 streams the row from HBM; pass 2 re-reads it from L2
// (at most 2 CTAs per SM; the eviction policies above keep the 296 rows in flight resident) and
// writes the gradient. Exponentials run in the log2 domain on the MUFU unit.
template <typename T, bool VEC>
__global__ void __launch_bounds__(kThreads, 2)
ce_kernel(const T* __restrict__ logits, int64_t ldl, const int64_t* __restrict__ targets,
          float* __restrict__ row_loss, T* dlogits, int64_t ldd, int64_t rows, int64_t vocab,
          float grad_scale, int* status)
{
    constexpr int V = VEC ? Vec16<T>::N : 1;
    constexpr int U = VEC ? 4 : 1;   // vectors in flight per thread (64 KB a block)
    __shared__ float red_m[kThreads / 32];
    __shared__ float red_s[kThreads / 32];
    __shared__ float final_m, final_log2;
    dep_wait();
    dep_release();
    const uint64_t keep = l2_policy_keep(), drop = l2_policy_drop();
    // a power-of-two grad_scale (1 / lanes for a power-of-two lane count) folds into the exponent
    // exactly: grad_scale 2^a = 2^(a + log2 grad_scale)
    const bool pow2 = grad_scale > 0.0f && (__float_as_uint(grad_scale) & 0x7FFFFFu) == 0 &&
                      (__float_as_uint(grad_scale) >> 23) != 0;
    const float log2_scale =
        pow2 ? static_cast<float>(static_cast<int>(__float_as_uint(grad_scale) >> 23) - 127) : 0.0f;
    const float mul_scale = pow2 ? 1.0f : grad_scale;
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x)
    {
        const T* x = logits + row * ldl;
        const int64_t t = targets[row];
        const bool valid = t >= 0 && t < vocab;
        // the target logit is read before the block barrier: with dlogits aliasing logits, pass 2
        // of other threads may overwrite it afterwards
        const float xt = (threadIdx.x == 0 && valid) ? to_f32(x[t]) : 0.0f;
        float m = -INFINITY, s = 0.0f;
        int64_t i = static_cast<int64_t>(threadIdx.x) * V;
        for (; i + static_cast<int64_t>(kThreads) * V * (U - 1) < vocab; i += static_cast<int64_t>(kThreads) * V * U)
        {
            float v[U][V];
#pragma unroll
            for (int u = 0; u < U; ++u)
            {
                if constexpr (VEC)
                    load16_hint(x + i + static_cast<int64_t>(u) * kThreads * V, v[u], keep);
                else
                    v[u][0] = to_f32(x[i]);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) online_add<V>(m, s, v[u]);
        }
        for (; i < vocab; i += static_cast<int64_t>(kThreads) * V)
        {
            float v[V];
            if constexpr (VEC)
                load16_hint(x + i, v, keep);
            else
                v[0] = to_f32(x[i]);
            online_add<V>(m, s, v);
        }
        // warp then block merge of (m, s)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
        {
            const float om = __shfl_xor_sync(0xFFFFFFFFu, m, o);
            const float os = __shfl_xor_sync(0xFFFFFFFFu, s, o);
            online_merge(m, s, om, os);
        }
        const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
        if (lane == 0)
        {
            red_m[wid] = m;
            red_s[wid] = s;
        }
        __syncthreads();
        if (threadIdx.x == 0)
        {
            float bm = red_m[0], bs = red_s[0];
            for (int w = 1; w < kThreads / 32; ++w)
            {
                online_merge(bm, bs, red_m[w], red_s[w]);
            }
            final_m = bm;
            final_log2 = log2f(bs);
        }
        __syncthreads();
        const float shift = final_m + final_log2;   // log2 of the normaliser, in log2 units
        if (threadIdx.x == 0)
        {
            if (!valid)
            {
                if (status != nullptr)
                {
                    *status = VEDA_ERR_OUT_OF_RANGE;
                }
                if (row_loss != nullptr)
                {
                    row_loss[row] = NAN;
                }
            }
            else if (row_loss != nullptr)
            {
                // -log softmax at the target = ln 2 * (shift - x_t log2 e)
                row_loss[row] = (shift - xt * kLog2e) * kLn2;
            }
        }
        if (dlogits != nullptr && valid)
        {
            T* d = dlogits + row * ldd;
            constexpr int U2 = VEC ? 4 : 1;   // vectors in flight per thread in the L2 pass
            const float shift_g = shift - log2_scale;
            auto grad = [&](int64_t k, float (&v)[V]) {
#pragma unroll
                for (int j = 0; j < V; ++j) v[j] = mul_scale * ex2(fmaf(v[j], kLog2e, -shift_g));
                if (t >= k && t < k + V)
                {
#pragma unroll
                    for (int j = 0; j < V; ++j)
                        if (k + j == t) v[j] -= grad_scale;
                }
            };
            int64_t k = static_cast<int64_t>(threadIdx.x) * V;
            for (; k + static_cast<int64_t>(kThreads) * V * (U2 - 1) < vocab;
                 k += static_cast<int64_t>(kThreads) * V * U2)
            {
                float v[U2][V];
#pragma unroll
                for (int u = 0; u < U2; ++u)
                {
                    if constexpr (VEC)
                        load16_hint(x + k + static_cast<int64_t>(u) * kThreads * V, v[u], drop);
                    else
                        v[u][0] = to_f32(x[k]);
                }
#pragma unroll
                for (int u = 0; u < U2; ++u)
                {
                    const int64_t ku = k + static_cast<int64_t>(u) * kThreads * V;
                    grad(ku, v[u]);
                    if constexpr (VEC)
                        store16_hint(d + ku, v[u], drop);
                    else
                        d[ku] = from_f32<T>(v[u][0]);
                }
            }
            for (; k < vocab; k += static_cast<int64_t>(kThreads) * V)
            {
                float v[V];
                if constexpr (VEC)
                    load16_hint(x + k, v, drop);
                else
                    v[0] = to_f32(x[k]);
                grad(k, v);
                if constexpr (VEC)
                    store16_hint(d + k, v, drop);
                else
                    d[k] = from_f32<T>(v[0]);
            }
        }
        __syncthreads();
    }
}

// Deterministic double-precision mean: one CTA, fixed order of partial sums.
__global__ void mean_f64_kernel(const float* __restrict__ v, int64_t n, float* out,
                                double* out_f64)
{
    __shared__ double part[1024 / 32];
    dep_wait();
    dep_release();
    double s = 0.0;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x)
    {
        s += static_cast<double>(v[i]);
    }
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0)
    {
        part[threadIdx.x >> 5] = s;
    }
    __syncthreads();
    if (threadIdx.x == 0)
    {
        double total = 0.0;
        for (int w = 0; w < static_cast<int>(blockDim.x / 32); ++w)
        {
            total += part[w];
        }
        const double mean = total / static_cast<double>(n);
        if (out != nullptr)
        {
            *out = static_cast<float>(mean);
        }
        if (out_f64 != nullptr)
        {
            *out_f64 = mean;
        }
    }
}

} // namespace
} // namespace veda::cuda

using namespace veda::cuda;

extern "C" int veda_cross_entropy(const void* logits, int64_t ldl, const int64_t* targets,
                                  float* row_loss, void* dlogits, int64_t ldd, int64_t rows,
                                  int64_t vocab, float grad_scale, int* status, int dtype,
                                  veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype), "unknown dtype");
    VEDA_REQUIRE(rows >= 0 && vocab > 0 && ldl >= vocab, "bad shape");
    VEDA_REQUIRE(dlogits == nullptr || ldd >= vocab, "bad dlogits leading dimension");
    if (rows == 0)
    {
        return VEDA_OK;
    }
    VEDA_REQUIRE(logits != nullptr && targets != nullptr, "null pointer");
    const size_t es = dtype_size(dtype);
    const int64_t v = 16 / static_cast<int64_t>(es);
    const bool vec = aligned16(logits) && ldl % v == 0 && vocab % v == 0 &&
                     (dlogits == nullptr || (aligned16(dlogits) && ldd % v == 0));
    const unsigned grid = static_cast<unsigned>(
        rows < static_cast<int64_t>(sm_count()) * 2 ? rows : static_cast<int64_t>(sm_count()) * 2);
#define VEDA_CE(T, VEC)                                                                           \
    launch("veda_cross_entropy", ce_kernel<T, VEC>, dim3(grid), dim3(kThreads), 0, stream,         \
           static_cast<const T*>(logits), ldl, targets, row_loss, static_cast<T*>(dlogits), ldd,  \
           rows, vocab, grad_scale, status)
    if (dtype == VEDA_BF16)
    {
        return vec ? VEDA_CE(bf16, true) : VEDA_CE(bf16, false);
    }
    return vec ? VEDA_CE(float, true) : VEDA_CE(float, false);
#undef VEDA_CE
}

extern "C" int veda_mean_f64(const float* v, int64_t n, float* out, double* out_f64,
                             veda_stream_t stream)
{
    VEDA_REQUIRE(n > 0, "nothing to average over");
    VEDA_REQUIRE(v != nullptr, "null pointer");
    return launch("veda_mean_f64", mean_f64_kernel, dim3(1), dim3(1024), 0, stream, v, n, out, out_f64);
}
