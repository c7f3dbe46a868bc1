// Global-norm gradient clip and AdamW on fp32 master weights — one streaming pass each.
//
// sumsq   sum of g^2 in double (src/libs/optim/Clip.cpp:21-33), two-stage with a fixed grid so
//         the summation order, and therefore the result, is the same on every call.
// clip    total = sqrt(sumsq); scale = float(max/total) only if total is finite and > max
//         (Clip.cpp:35-60); a non-finite total scales nothing.
// AdamW   src/libs/optim/AdamW.cpp:38-93 operation for operation: m and v in fp32, m_hat and
//         v_hat and the adaptive ratio in double, decoupled decay applied first. Products and
//         sums use explicit round-to-nearest intrinsics so the compiler cannot contract them into
//         fused multiply-adds, which keeps the result equal to the CPU's bit for bit on equal
//         gradients. The clip scale is computed in the kernel from the device-side sumsq, so the
//         clipped step needs no host round trip.
#include "common.cuh"

namespace veda::cuda
{
namespace
{

constexpr int kThreads = 512;

inline int sumsq_grid(int64_t n)
{
    const int64_t cap = 2LL * sm_count();
    const int64_t want = (n + kThreads * 8 - 1) / (kThreads * 8);
    return static_cast<int>(want < 1 ? 1 : (want < cap ? want : cap));
}

__global__ void __launch_bounds__(kThreads)
sumsq_partial_kernel(const float* __restrict__ g, int64_t n, double* __restrict__ partials)
{
    __shared__ double part[kThreads / 32];
    dep_wait();
    dep_release();
    double s = 0.0;
    const int64_t n4 = (reinterpret_cast<uintptr_t>(g) & 15u) == 0 ? n / 4 : 0;
    const float4* g4 = reinterpret_cast<const float4*>(g);
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += stride)
    {
        const float4 v = g4[i];
        s += static_cast<double>(v.x) * v.x;
        s += static_cast<double>(v.y) * v.y;
        s += static_cast<double>(v.z) * v.z;
        s += static_cast<double>(v.w) * v.w;
    }
    for (int64_t i = n4 * 4 + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += stride)
    {
        const double v = g[i];
        s += v * v;
    }
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0)
    {
        part[threadIdx.x >> 5] = s;
    }
    __syncthreads();
    if (threadIdx.x == 0)
    {
        double t = 0.0;
        for (int w = 0; w < kThreads / 32; ++w)
        {
            t += part[w];
        }
        partials[blockIdx.x] = t;
    }
}

__global__ void sumsq_final_kernel(const double* __restrict__ partials, int count, double* out,
                                   int accumulate)
{
    dep_wait();
    dep_release();
    if (threadIdx.x == 0 && blockIdx.x == 0)
    {
        double t = accumulate ? *out : 0.0;
        double s = 0.0;
        for (int b = 0; b < count; ++b)
        {
            s += partials[b];
        }
        *out = t + s;
    }
}

// total = sqrt(sumsq) * grad_scale: the norm of the gradient after the grad_scale factor (the
// 1/world average of data-parallel training) has been applied.
__device__ __forceinline__ float clip_scale(const double* sumsq, float max_norm,
                                            float grad_scale = 1.0f)
{
    if (sumsq == nullptr)
    {
        return 1.0f;
    }
    double total = sqrt(*sumsq);
    if (grad_scale != 1.0f)
    {
        total *= fabs(static_cast<double>(grad_scale));
    }
    if (!isfinite(total) || total <= static_cast<double>(max_norm))
    {
        return 1.0f;
    }
    return static_cast<float>(static_cast<double>(max_norm) / total);
}

__global__ void clip_kernel(float* __restrict__ g, int64_t n, const double* __restrict__ sumsq,
                            float max_norm)
{
    const float scale = clip_scale(sumsq, max_norm);
    if (scale == 1.0f)
    {
        return;   // nothing is written at all (Clip.cpp:40-43)
    }
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        g[i] = __fmul_rn(g[i], scale);
    }
}

struct AdamArgs
{
    float lr, beta1, beta2, eps, wd;
    double bias1, bias2;
    float max_norm, grad_scale;
    int write_grad;   // bit 0: store g' back; bit 1: skip the step on a non-finite norm
};

__device__ __forceinline__ float adam_one(float& w, float& m, float& v, float g, const AdamArgs& a)
{
    m = __fadd_rn(__fmul_rn(a.beta1, m), __fmul_rn(__fsub_rn(1.0f, a.beta1), g));
    v = __fadd_rn(__fmul_rn(a.beta2, v), __fmul_rn(__fmul_rn(__fsub_rn(1.0f, a.beta2), g), g));
    const double m_hat = static_cast<double>(m) / a.bias1;
    const double v_hat = static_cast<double>(v) / a.bias2;
    const double adaptive = m_hat / (sqrt(v_hat) + static_cast<double>(a.eps));
    w = __fsub_rn(w, __fmul_rn(__fmul_rn(a.lr, a.wd), w));
    w = __fsub_rn(w, __fmul_rn(a.lr, static_cast<float>(adaptive)));
    return w;
}

__global__ void __launch_bounds__(kThreads)
adamw_kernel(float* __restrict__ master, float* __restrict__ m, float* __restrict__ v,
             float* __restrict__ g, bf16* __restrict__ lowp, int64_t n,
             const double* __restrict__ sumsq, AdamArgs a, const double* __restrict__ bias, bool vec)
{
    dep_wait();
    dep_release();
    if (bias != nullptr)
    {
        // bias corrections computed by the host for this step and left in device memory (a step
        // replayed from a CUDA graph reads the current ones)
        a.bias1 = bias[0];
        a.bias2 = bias[1];
    }
    if ((a.write_grad & 2) && sumsq != nullptr &&
        !isfinite(static_cast<float>(sqrt(*sumsq) * fabs(static_cast<double>(a.grad_scale)))))
    {
        return;   // a non-finite norm: the whole step is skipped, nothing is written
    }
    const float clip = clip_scale(sumsq, a.max_norm, a.grad_scale);
    // an unscaled gradient is already what the write-back would store
    const bool store_g = (a.write_grad & 1) && (clip != 1.0f || a.grad_scale != 1.0f);
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t n4 = vec ? n / 4 : 0;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += stride)
    {
        float4 w4 = reinterpret_cast<float4*>(master)[i];
        float4 m4 = reinterpret_cast<float4*>(m)[i];
        float4 v4 = reinterpret_cast<float4*>(v)[i];
        float4 g4 = reinterpret_cast<float4*>(g)[i];
        float* wp = &w4.x;
        float* mp = &m4.x;
        float* vp = &v4.x;
        float* gp = &g4.x;
#pragma unroll
        for (int j = 0; j < 4; ++j)
        {
            float gj = gp[j];
            if (a.grad_scale != 1.0f)
            {
                gj = __fmul_rn(gj, a.grad_scale);
            }
            if (clip != 1.0f)
            {
                gj = __fmul_rn(gj, clip);
            }
            gp[j] = gj;
            adam_one(wp[j], mp[j], vp[j], gj, a);
        }
        reinterpret_cast<float4*>(master)[i] = w4;
        reinterpret_cast<float4*>(m)[i] = m4;
        reinterpret_cast<float4*>(v)[i] = v4;
        if (store_g)
        {
            reinterpret_cast<float4*>(g)[i] = g4;
        }
        if (lowp != nullptr)
        {
            const __nv_bfloat162 lo = __floats2bfloat162_rn(w4.x, w4.y);
            const __nv_bfloat162 hi = __floats2bfloat162_rn(w4.z, w4.w);
            uint2 packed;
            packed.x = *reinterpret_cast<const uint32_t*>(&lo);
            packed.y = *reinterpret_cast<const uint32_t*>(&hi);
            reinterpret_cast<uint2*>(lowp)[i] = packed;
        }
    }
    for (int64_t i = n4 * 4 + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += stride)
    {
        float gj = g[i];
        if (a.grad_scale != 1.0f)
        {
            gj = __fmul_rn(gj, a.grad_scale);
        }
        if (clip != 1.0f)
        {
            gj = __fmul_rn(gj, clip);
        }
        float w = master[i], mm = m[i], vv = v[i];
        adam_one(w, mm, vv, gj, a);
        master[i] = w;
        m[i] = mm;
        v[i] = vv;
        if (store_g)
        {
            g[i] = gj;
        }
        if (lowp != nullptr)
        {
            lowp[i] = __float2bfloat16_rn(w);
        }
    }
}

} // namespace
} // namespace veda::cuda

using namespace veda::cuda;

extern "C" size_t veda_sumsq_workspace(int64_t n)
{
    return static_cast<size_t>(sumsq_grid(n)) * sizeof(double);
}

extern "C" int veda_sumsq(const float* g, int64_t n, double* sumsq, int accumulate,
                          void* workspace, size_t workspace_bytes, veda_stream_t stream)
{
    VEDA_REQUIRE(n >= 0 && sumsq != nullptr, "bad arguments");
    VEDA_REQUIRE(workspace != nullptr && workspace_bytes >= veda_sumsq_workspace(n),
                 "workspace too small (see veda_sumsq_workspace)");
    VEDA_REQUIRE(n == 0 || g != nullptr, "null pointer");
    const int grid = sumsq_grid(n);
    double* partials = static_cast<double*>(workspace);
    if (n > 0)
    {
        const int rc = launch("veda_sumsq", sumsq_partial_kernel, dim3(grid), dim3(kThreads), 0, stream,
                              g, n, partials);
        if (rc != VEDA_OK)
        {
            return rc;
        }
    }
    return launch("veda_sumsq", sumsq_final_kernel, dim3(1), dim3(32), 0, stream,
                  static_cast<const double*>(partials), n > 0 ? grid : 0, sumsq, accumulate);
}

extern "C" int veda_clip_apply(float* g, int64_t n, const double* sumsq, float max_norm,
                               veda_stream_t stream)
{
    VEDA_REQUIRE(max_norm > 0.0f, "max_norm must be positive");
    VEDA_REQUIRE(n >= 0 && sumsq != nullptr, "bad arguments");
    if (n == 0)
    {
        return VEDA_OK;
    }
    clip_kernel<<<grid_for(n, 256), 256, 0, stream>>>(g, n, sumsq, max_norm);
    count_launch();
    return check_launch("veda_clip_apply");
}

namespace
{
int adamw_launch(float* master, float* m, float* v, float* g, void* lowp, int64_t n, float lr,
                 float beta1, float beta2, float eps, float weight_decay, double bias1, double bias2,
                 const double* bias_dev, const double* sumsq, float max_norm, float grad_scale,
                 int write_grad, veda_stream_t stream)
{
    VEDA_REQUIRE(lr >= 0.0f && eps > 0.0f && weight_decay >= 0.0f,
                 "learning rate, eps and weight decay must be positive");
    VEDA_REQUIRE(beta1 >= 0.0f && beta1 < 1.0f && beta2 >= 0.0f && beta2 < 1.0f,
                 "betas must lie in [0, 1)");
    VEDA_REQUIRE(bias_dev != nullptr || (bias1 > 0.0 && bias2 > 0.0), "bias corrections must be positive");
    VEDA_REQUIRE(sumsq == nullptr || max_norm > 0.0f, "max_norm must be positive");
    VEDA_REQUIRE(n >= 0, "bad size");
    if (n == 0)
    {
        return VEDA_OK;
    }
    VEDA_REQUIRE(master && m && v && g, "null pointer");
    const bool vec = aligned16(master) && aligned16(m) && aligned16(v) && aligned16(g) &&
                     (lowp == nullptr || (reinterpret_cast<uintptr_t>(lowp) & 7u) == 0);
    AdamArgs a{lr, beta1, beta2, eps, weight_decay, bias1, bias2, max_norm, grad_scale,
               write_grad};
    const unsigned grid = grid_for(vec ? n / 4 + 1 : n, kThreads, 4);
    return launch("veda_adamw_step", adamw_kernel, dim3(grid), dim3(kThreads), 0, stream, master, m, v, g,
                  static_cast<bf16*>(lowp), n, sumsq, a, bias_dev, vec);
}
} // namespace

extern "C" int veda_adamw_step(float* master, float* m, float* v, float* g, void* lowp, int64_t n,
                               float lr, float beta1, float beta2, float eps, float weight_decay,
                               double bias1, double bias2, const double* sumsq, float max_norm,
                               float grad_scale, int write_grad, veda_stream_t stream)
{
    return adamw_launch(master, m, v, g, lowp, n, lr, beta1, beta2, eps, weight_decay, bias1, bias2,
                        nullptr, sumsq, max_norm, grad_scale, write_grad, stream);
}

extern "C" int veda_adamw_step_dev(float* master, float* m, float* v, float* g, void* lowp,
                                   int64_t n, float lr, float beta1, float beta2, float eps,
                                   float weight_decay, const double* bias, const double* sumsq,
                                   float max_norm, float grad_scale, int write_grad,
                                   veda_stream_t stream)
{
    VEDA_REQUIRE(bias != nullptr, "null bias corrections");
    return adamw_launch(master, m, v, g, lowp, n, lr, beta1, beta2, eps, weight_decay, 0.0, 0.0,
                        bias, sumsq, max_norm, grad_scale, write_grad, stream);
}

extern "C" int veda_launch_count_add(int64_t n)
{
    count_launch(static_cast<uint64_t>(n));
    return VEDA_OK;
}
