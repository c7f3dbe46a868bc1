// The element-wise and per-lane ops of the fine-grained autograd API (the reference's
// veda::ops used by veda::autograd): broadcast add/mul, scalar mul, accumulate, strided copy,
// unbroadcast, sum, softmax, silu, argmax; plus fill, seeded normal fill and fp32->bf16.
// They keep the reference's arithmetic (fp32 with the same operation order per element) and
// are simple grid-stride kernels: the fused training path does not use them on its hot loop.
#include "common.cuh"

namespace veda::cuda
{
namespace
{

constexpr int kMaxRank = 8;

struct Dims
{
    int rank;
    int64_t shape[kMaxRank];
    int64_t sa[kMaxRank];
    int64_t sb[kMaxRank];
};

template <typename T>
__global__ void binary_kernel(int op, const T* __restrict__ a, const T* __restrict__ b,
                              T* __restrict__ out, Dims d, int64_t total)
{
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        int64_t rem = idx, oa = 0, ob = 0;
        for (int k = d.rank - 1; k >= 0; --k)
        {
            const int64_t c = rem % d.shape[k];
            rem /= d.shape[k];
            oa += c * d.sa[k];
            ob += c * d.sb[k];
        }
        const float x = to_f32(a[oa]), y = to_f32(b[ob]);
        out[idx] = from_f32<T>(op == 0 ? x + y : x * y);
    }
}

// Same-shape contiguous operands (the residual add): 16-byte vectors, no index arithmetic.
template <typename T>
__global__ void binary_dense_kernel(int op, const T* __restrict__ a, const T* __restrict__ b,
                                    T* __restrict__ out, int64_t n)
{
    constexpr int V = Vec16<T>::N;
    const int64_t nv = n / V;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nv;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        float x[V], y[V];
        load16(a + i * V, x);
        load16(b + i * V, y);
#pragma unroll
        for (int j = 0; j < V; ++j)
        {
            x[j] = op == 0 ? x[j] + y[j] : x[j] * y[j];
        }
        store16(out + i * V, x);
    }
    for (int64_t i = nv * V + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        const float x = to_f32(a[i]), y = to_f32(b[i]);
        out[i] = from_f32<T>(op == 0 ? x + y : x * y);
    }
}

template <typename T>
__global__ void scale_kernel(const T* __restrict__ x, float s, T* __restrict__ out, int64_t n)
{
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        out[i] = from_f32<T>(to_f32(x[i]) * s);
    }
}

template <typename D, typename S>
__global__ void accumulate_kernel(D* __restrict__ dst, const S* __restrict__ src, int64_t n)
{
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        dst[i] = from_f32<D>(to_f32(dst[i]) + to_f32(src[i]));
    }
}

template <typename D, typename S>
__global__ void copy_strided_kernel(const S* __restrict__ src, D* __restrict__ dst, Dims d,
                                    int64_t offset, int64_t total)
{
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        int64_t rem = idx, o = offset;
        for (int k = d.rank - 1; k >= 0; --k)
        {
            const int64_t c = rem % d.shape[k];
            rem /= d.shape[k];
            o += c * d.sa[k];
        }
        dst[idx] = from_f32<D>(to_f32(src[o]));
    }
}

// One thread per output element; reduced axes (target extent 1 where the source is larger) are
// walked in row-major order, the order detail::unbroadcast visits them (Variable.cpp:55-84).
// d.shape: source shape; d.sa: target extents (aligned); d.sb: source contiguous strides.
template <typename T>
__global__ void unbroadcast_kernel(const T* __restrict__ g, T* __restrict__ out, Dims d,
                                   int64_t out_total, int64_t reduce_total)
{
    for (int64_t o = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; o < out_total;
         o += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        // coordinates of o in the target (kept axes)
        int64_t base = 0, rem = o;
        for (int k = d.rank - 1; k >= 0; --k)
        {
            const int64_t ext = d.sa[k];
            const int64_t c = rem % ext;
            rem /= ext;
            if (ext != 1 || d.shape[k] == 1)
            {
                base += c * d.sb[k];
            }
        }
        float acc = 0.0f;
        for (int64_t r = 0; r < reduce_total; ++r)
        {
            int64_t rr = r, off = base;
            for (int k = d.rank - 1; k >= 0; --k)
            {
                if (d.sa[k] == 1 && d.shape[k] != 1)
                {
                    const int64_t c = rr % d.shape[k];
                    rr /= d.shape[k];
                    off += c * d.sb[k];
                }
            }
            acc += to_f32(g[off]);
        }
        out[o] = from_f32<T>(acc);
    }
}

template <typename T>
__global__ void sum_kernel(const T* __restrict__ x, int64_t n, float* out)
{
    __shared__ double part[32];
    double s = 0.0;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x)
    {
        s += static_cast<double>(to_f32(x[i]));
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
        for (int w = 0; w < static_cast<int>(blockDim.x / 32); ++w)
        {
            t += part[w];
        }
        *out = static_cast<float>(t);
    }
}

template <typename T>
__global__ void fill_kernel(T* __restrict__ x, float value, int64_t n)
{
    const T v = from_f32<T>(value);
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        x[i] = v;
    }
}

// softmax over contiguous lanes, one CTA per lane: max, sum of exp(x - max) (fp32), divide.
template <typename T>
__global__ void softmax_fwd_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t lanes,
                                   int64_t length)
{
    __shared__ float red[32];
    __shared__ float bcast;
    for (int64_t lane_i = blockIdx.x; lane_i < lanes; lane_i += gridDim.x)
    {
        const T* xr = x + lane_i * length;
        T* yr = y + lane_i * length;
        float m = -INFINITY;
        for (int64_t i = threadIdx.x; i < length; i += blockDim.x)
        {
            m = fmaxf(m, to_f32(xr[i]));
        }
        m = warp_max(m);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
        __syncthreads();
        if (threadIdx.x == 0)
        {
            float t = red[0];
            for (int w = 1; w < static_cast<int>(blockDim.x / 32); ++w) t = fmaxf(t, red[w]);
            bcast = t;
        }
        __syncthreads();
        m = bcast;
        __syncthreads();
        float s = 0.0f;
        for (int64_t i = threadIdx.x; i < length; i += blockDim.x)
        {
            s += expf(to_f32(xr[i]) - m);
        }
        s = warp_sum(s);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
        __syncthreads();
        if (threadIdx.x == 0)
        {
            float t = 0.0f;
            for (int w = 0; w < static_cast<int>(blockDim.x / 32); ++w) t += red[w];
            bcast = t;
        }
        __syncthreads();
        s = bcast;
        for (int64_t i = threadIdx.x; i < length; i += blockDim.x)
        {
            yr[i] = from_f32<T>(expf(to_f32(xr[i]) - m) / s);
        }
        __syncthreads();
    }
}

template <typename T>
__global__ void softmax_bwd_kernel(const T* __restrict__ y, const T* __restrict__ g,
                                   T* __restrict__ dx, int64_t lanes, int64_t length)
{
    __shared__ float red[32];
    __shared__ float bcast;
    for (int64_t lane_i = blockIdx.x; lane_i < lanes; lane_i += gridDim.x)
    {
        const T* yr = y + lane_i * length;
        const T* gr = g + lane_i * length;
        float w = 0.0f;
        for (int64_t i = threadIdx.x; i < length; i += blockDim.x)
        {
            w += to_f32(gr[i]) * to_f32(yr[i]);
        }
        w = warp_sum(w);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = w;
        __syncthreads();
        if (threadIdx.x == 0)
        {
            float t = 0.0f;
            for (int k = 0; k < static_cast<int>(blockDim.x / 32); ++k) t += red[k];
            bcast = t;
        }
        __syncthreads();
        w = bcast;
        for (int64_t i = threadIdx.x; i < length; i += blockDim.x)
        {
            dx[lane_i * length + i] = from_f32<T>(to_f32(yr[i]) * (to_f32(gr[i]) - w));
        }
        __syncthreads();
    }
}

template <typename T>
__global__ void silu_fwd_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n)
{
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        const float v = to_f32(x[i]);
        y[i] = from_f32<T>(v / (1.0f + expf(-v)));
    }
}

template <typename T>
__global__ void silu_bwd_kernel(const T* __restrict__ x, const T* __restrict__ g,
                                T* __restrict__ dx, int64_t n)
{
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        const float v = to_f32(x[i]);
        const float s = 1.0f / (1.0f + expf(-v));
        dx[i] = from_f32<T>(to_f32(g[i]) * s * (1.0f + v * (1.0f - s)));
    }
}

// tanh-GELU: 0.5 x (1 + tanh(c (x + 0.044715 x^3))), c = sqrt(2/pi).
constexpr float kGeluC = 0.7978845608028654f;
constexpr float kGeluCubic = 0.044715f;

template <typename T>
__global__ void gelu_fwd_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n)
{
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        const float v = to_f32(x[i]);
        y[i] = from_f32<T>(0.5f * v * (1.0f + tanhf(kGeluC * (v + kGeluCubic * v * v * v))));
    }
}

template <typename T>
__global__ void gelu_bwd_kernel(const T* __restrict__ x, const T* __restrict__ g,
                                T* __restrict__ dx, int64_t n)
{
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        const float v = to_f32(x[i]);
        const float u = kGeluC * (v + kGeluCubic * v * v * v);
        const float t = tanhf(u);
        const float d = 0.5f * (1.0f + t) +
                        0.5f * v * (1.0f - t * t) * kGeluC * (1.0f + 3.0f * kGeluCubic * v * v);
        dx[i] = from_f32<T>(to_f32(g[i]) * d);
    }
}

// Row argmax, ties to the lower index; NaN anywhere in the row flags the status.
template <typename T>
__global__ void argmax_kernel(const T* __restrict__ x, int64_t ld, int64_t rows, int64_t n,
                              int64_t* __restrict__ out, int* status)
{
    __shared__ float bv[32];
    __shared__ int64_t bi[32];
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x)
    {
        const T* xr = x + r * ld;
        float best = -INFINITY;
        int64_t idx = -1;
        bool nan = false;
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x)
        {
            const float v = to_f32(xr[i]);
            if (v != v)
            {
                nan = true;
            }
            else if (idx < 0 || v > best)
            {
                best = v;
                idx = i;
            }
        }
        if (__syncthreads_or(nan))
        {
            if (threadIdx.x == 0)
            {
                out[r] = -1;
                if (status != nullptr) *status = VEDA_ERR_INVALID_ARGUMENT;
            }
            continue;
        }
        for (int o = 16; o > 0; o >>= 1)
        {
            const float ov = __shfl_xor_sync(0xFFFFFFFFu, best, o);
            const int64_t oi = __shfl_xor_sync(0xFFFFFFFFu, idx, o);
            if (oi >= 0 && (idx < 0 || ov > best || (ov == best && oi < idx)))
            {
                best = ov;
                idx = oi;
            }
        }
        if ((threadIdx.x & 31) == 0)
        {
            bv[threadIdx.x >> 5] = best;
            bi[threadIdx.x >> 5] = idx;
        }
        __syncthreads();
        if (threadIdx.x == 0)
        {
            float b = bv[0];
            int64_t j = bi[0];
            for (int w = 1; w < static_cast<int>(blockDim.x / 32); ++w)
            {
                if (bi[w] >= 0 && (j < 0 || bv[w] > b || (bv[w] == b && bi[w] < j)))
                {
                    b = bv[w];
                    j = bi[w];
                }
            }
            out[r] = j;
        }
        __syncthreads();
    }
}

__device__ __forceinline__ uint64_t mix64(uint64_t z)
{
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

template <typename T>
__global__ void randn_kernel(T* __restrict__ x, int64_t n, float stddev, uint64_t seed)
{
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        const uint64_t h = mix64(seed * 0x2545F4914F6CDD1Dull ^ static_cast<uint64_t>(i));
        const float u1 = (static_cast<float>(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
        const float u2 = static_cast<float>((h >> 16) & 0xFFFFFFull) * (1.0f / 16777216.0f);
        const float z = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
        x[i] = from_f32<T>(z * stddev);
    }
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ src, bf16* __restrict__ dst, int64_t n)
{
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        dst[i] = __float2bfloat16_rn(src[i]);
    }
}

int fill_dims(Dims& d, const int64_t* shape, int rank, const int64_t* sa, const int64_t* sb,
              int64_t& total)
{
    if (rank < 0 || rank > kMaxRank)
    {
        return fail(VEDA_ERR_UNSUPPORTED, "rank above 8");
    }
    d.rank = rank;
    total = 1;
    for (int k = 0; k < rank; ++k)
    {
        if (shape[k] < 0)
        {
            return fail(VEDA_ERR_INVALID_ARGUMENT, "negative extent");
        }
        d.shape[k] = shape[k];
        d.sa[k] = sa ? sa[k] : 0;
        d.sb[k] = sb ? sb[k] : 0;
        total *= shape[k];
    }
    return VEDA_OK;
}

} // namespace
} // namespace veda::cuda

using namespace veda::cuda;

#define VEDA_DISPATCH(dtype, T, ...)                                                              \
    if ((dtype) == VEDA_BF16)                                                                     \
    {                                                                                             \
        using T = bf16;                                                                           \
        __VA_ARGS__;                                                                              \
    }                                                                                             \
    else                                                                                          \
    {                                                                                             \
        using T = float;                                                                          \
        __VA_ARGS__;                                                                              \
    }

extern "C" int veda_binary(int op, const void* a, const int64_t* a_strides, const void* b,
                           const int64_t* b_strides, void* out, const int64_t* shape, int rank,
                           int dtype, veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype) && (op == 0 || op == 1), "bad op or dtype");
    Dims d{};
    int64_t total = 0;
    int rc = fill_dims(d, shape, rank, a_strides, b_strides, total);
    if (rc != VEDA_OK) return rc;
    if (total == 0) return VEDA_OK;
    VEDA_REQUIRE(a && b && out, "null pointer");
    bool dense = aligned16(a) && aligned16(b) && aligned16(out);
    int64_t expect = 1;
    for (int k = rank - 1; k >= 0 && dense; --k)
    {
        dense = d.shape[k] == 1 || (d.sa[k] == expect && d.sb[k] == expect);
        expect *= d.shape[k];
    }
    if (dense)
    {
        const int64_t v = 16 / static_cast<int64_t>(dtype_size(dtype));
        VEDA_DISPATCH(dtype, T,
                      binary_dense_kernel<T><<<grid_for(total / v + 1, 256, 4), 256, 0, stream>>>(
                          op, static_cast<const T*>(a), static_cast<const T*>(b),
                          static_cast<T*>(out), total));
        count_launch();
        return check_launch("veda_binary");
    }
    VEDA_DISPATCH(dtype, T,
                  binary_kernel<T><<<grid_for(total, 256), 256, 0, stream>>>(
                      op, static_cast<const T*>(a), static_cast<const T*>(b),
                      static_cast<T*>(out), d, total));
    count_launch();
    return check_launch("veda_binary");
}

extern "C" int veda_scale(const void* x, float s, void* out, int64_t n, int dtype,
                          veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype) && n >= 0, "bad arguments");
    if (n == 0) return VEDA_OK;
    VEDA_REQUIRE(x && out, "null pointer");
    VEDA_DISPATCH(dtype, T,
                  scale_kernel<T><<<grid_for(n, 256), 256, 0, stream>>>(
                      static_cast<const T*>(x), s, static_cast<T*>(out), n));
    count_launch();
    return check_launch("veda_scale");
}

extern "C" int veda_accumulate(void* dst, int dtype_dst, const void* src, int dtype_src, int64_t n,
                               veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype_dst) && valid_dtype(dtype_src) && n >= 0, "bad arguments");
    if (n == 0) return VEDA_OK;
    VEDA_REQUIRE(dst && src, "null pointer");
    const unsigned grid = grid_for(n, 256);
    if (dtype_dst == VEDA_F32)
    {
        VEDA_DISPATCH(dtype_src, S,
                      accumulate_kernel<float, S><<<grid, 256, 0, stream>>>(
                          static_cast<float*>(dst), static_cast<const S*>(src), n));
    }
    else
    {
        VEDA_DISPATCH(dtype_src, S,
                      accumulate_kernel<bf16, S><<<grid, 256, 0, stream>>>(
                          static_cast<bf16*>(dst), static_cast<const S*>(src), n));
    }
    count_launch();
    return check_launch("veda_accumulate");
}

extern "C" int veda_copy_strided(const void* src, int dtype_src, const int64_t* src_strides,
                                 int64_t offset, void* dst, int dtype_dst, const int64_t* shape,
                                 int rank, veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype_src) && valid_dtype(dtype_dst), "unknown dtype");
    Dims d{};
    int64_t total = 0;
    int rc = fill_dims(d, shape, rank, src_strides, nullptr, total);
    if (rc != VEDA_OK) return rc;
    if (total == 0) return VEDA_OK;
    VEDA_REQUIRE(src && dst, "null pointer");
    const unsigned grid = grid_for(total, 256);
    if (dtype_dst == VEDA_F32)
    {
        VEDA_DISPATCH(dtype_src, S,
                      copy_strided_kernel<float, S><<<grid, 256, 0, stream>>>(
                          static_cast<const S*>(src), static_cast<float*>(dst), d, offset, total));
    }
    else
    {
        VEDA_DISPATCH(dtype_src, S,
                      copy_strided_kernel<bf16, S><<<grid, 256, 0, stream>>>(
                          static_cast<const S*>(src), static_cast<bf16*>(dst), d, offset, total));
    }
    count_launch();
    return check_launch("veda_copy_strided");
}

extern "C" int veda_unbroadcast(const void* g, const int64_t* shape, const int64_t* target,
                                int rank, void* out, int dtype, veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype), "unknown dtype");
    VEDA_REQUIRE(rank >= 0 && rank <= kMaxRank, "rank above 8");
    Dims d{};
    d.rank = rank;
    int64_t out_total = 1, reduce_total = 1, stride = 1;
    for (int k = rank - 1; k >= 0; --k)
    {
        VEDA_REQUIRE(target[k] == shape[k] || target[k] == 1, "target does not broadcast");
        d.shape[k] = shape[k];
        d.sa[k] = target[k];
        d.sb[k] = stride;
        stride *= shape[k];
        out_total *= target[k];
        if (target[k] == 1 && shape[k] != 1) reduce_total *= shape[k];
    }
    if (out_total == 0) return VEDA_OK;
    VEDA_REQUIRE(g && out, "null pointer");
    VEDA_DISPATCH(dtype, T,
                  unbroadcast_kernel<T><<<grid_for(out_total, 256), 256, 0, stream>>>(
                      static_cast<const T*>(g), static_cast<T*>(out), d, out_total,
                      reduce_total));
    count_launch();
    return check_launch("veda_unbroadcast");
}

extern "C" int veda_sum(const void* x, int64_t n, float* out, int dtype, veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype) && n >= 0 && out != nullptr, "bad arguments");
    VEDA_REQUIRE(n == 0 || x != nullptr, "null pointer");
    VEDA_DISPATCH(dtype, T,
                  sum_kernel<T><<<1, 1024, 0, stream>>>(static_cast<const T*>(x), n, out));
    count_launch();
    return check_launch("veda_sum");
}

extern "C" int veda_fill(void* x, float value, int64_t n, int dtype, veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype) && n >= 0, "bad arguments");
    if (n == 0) return VEDA_OK;
    VEDA_REQUIRE(x != nullptr, "null pointer");
    VEDA_DISPATCH(dtype, T,
                  fill_kernel<T><<<grid_for(n, 256), 256, 0, stream>>>(static_cast<T*>(x), value,
                                                                       n));
    count_launch();
    return check_launch("veda_fill");
}

extern "C" int veda_softmax_fwd(const void* x, void* y, int64_t lanes, int64_t length, int dtype,
                                veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype) && lanes >= 0 && length >= 0, "bad arguments");
    if (lanes == 0 || length == 0) return VEDA_OK;
    VEDA_REQUIRE(x && y, "null pointer");
    const unsigned grid = static_cast<unsigned>(
        lanes < static_cast<int64_t>(sm_count()) * 8 ? lanes : static_cast<int64_t>(sm_count()) * 8);
    VEDA_DISPATCH(dtype, T,
                  softmax_fwd_kernel<T><<<grid, 256, 0, stream>>>(
                      static_cast<const T*>(x), static_cast<T*>(y), lanes, length));
    count_launch();
    return check_launch("veda_softmax_fwd");
}

namespace veda::cuda
{
namespace
{
// log_softmax over the last dim (ops::log_softmax, src/libs/ops/Softmax.cpp:82-151): x - m -
// log(sum exp(x - m)) with m the lane's maximum; a lane that is -inf everywhere stays -inf (no
// inf - inf). One block per lane.
template <typename T>
__global__ void log_softmax_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t lanes,
                                   int64_t length)
{
    __shared__ float red[32];
    __shared__ float bcast;
    for (int64_t lane_i = blockIdx.x; lane_i < lanes; lane_i += gridDim.x)
    {
        const T* xr = x + lane_i * length;
        T* yr = y + lane_i * length;
        float m = -INFINITY;
        for (int64_t i = threadIdx.x; i < length; i += blockDim.x) m = fmaxf(m, to_f32(xr[i]));
        m = warp_max(m);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
        __syncthreads();
        if (threadIdx.x == 0)
        {
            float t = red[0];
            for (int w = 1; w < static_cast<int>(blockDim.x / 32); ++w) t = fmaxf(t, red[w]);
            bcast = t;
        }
        __syncthreads();
        m = bcast;
        __syncthreads();
        if (m == -INFINITY)
        {
            for (int64_t i = threadIdx.x; i < length; i += blockDim.x) yr[i] = from_f32<T>(-INFINITY);
            continue;
        }
        float s = 0.0f;
        for (int64_t i = threadIdx.x; i < length; i += blockDim.x) s += expf(to_f32(xr[i]) - m);
        s = warp_sum(s);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
        __syncthreads();
        if (threadIdx.x == 0)
        {
            float t = 0.0f;
            for (int w = 0; w < static_cast<int>(blockDim.x / 32); ++w) t += red[w];
            bcast = logf(t);
        }
        __syncthreads();
        const float log_sum = bcast;
        __syncthreads();
        for (int64_t i = threadIdx.x; i < length; i += blockDim.x)
        {
            yr[i] = from_f32<T>(to_f32(xr[i]) - m - log_sum);
        }
    }
}
} // namespace
} // namespace veda::cuda

extern "C" int veda_log_softmax_fwd(const void* x, void* y, int64_t lanes, int64_t length, int dtype,
                                    veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype) && lanes >= 0 && length >= 0, "bad arguments");
    if (lanes == 0 || length == 0) return VEDA_OK;
    VEDA_REQUIRE(x && y, "null pointer");
    const unsigned grid = static_cast<unsigned>(
        lanes < static_cast<int64_t>(sm_count()) * 8 ? lanes : static_cast<int64_t>(sm_count()) * 8);
    VEDA_DISPATCH(dtype, T,
                  log_softmax_kernel<T><<<grid, 256, 0, stream>>>(
                      static_cast<const T*>(x), static_cast<T*>(y), lanes, length));
    count_launch();
    return check_launch("veda_log_softmax_fwd");
}

extern "C" int veda_softmax_bwd(const void* y, const void* g, void* dx, int64_t lanes,
                                int64_t length, int dtype, veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype) && lanes >= 0 && length >= 0, "bad arguments");
    if (lanes == 0 || length == 0) return VEDA_OK;
    VEDA_REQUIRE(y && g && dx, "null pointer");
    const unsigned grid = static_cast<unsigned>(
        lanes < static_cast<int64_t>(sm_count()) * 8 ? lanes : static_cast<int64_t>(sm_count()) * 8);
    VEDA_DISPATCH(dtype, T,
                  softmax_bwd_kernel<T><<<grid, 256, 0, stream>>>(
                      static_cast<const T*>(y), static_cast<const T*>(g), static_cast<T*>(dx),
                      lanes, length));
    count_launch();
    return check_launch("veda_softmax_bwd");
}

extern "C" int veda_silu_fwd(const void* x, void* y, int64_t n, int dtype, veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype) && n >= 0, "bad arguments");
    if (n == 0) return VEDA_OK;
    VEDA_REQUIRE(x && y, "null pointer");
    VEDA_DISPATCH(dtype, T,
                  silu_fwd_kernel<T><<<grid_for(n, 256), 256, 0, stream>>>(
                      static_cast<const T*>(x), static_cast<T*>(y), n));
    count_launch();
    return check_launch("veda_silu_fwd");
}

extern "C" int veda_silu_bwd(const void* x, const void* g, void* dx, int64_t n, int dtype,
                             veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype) && n >= 0, "bad arguments");
    if (n == 0) return VEDA_OK;
    VEDA_REQUIRE(x && g && dx, "null pointer");
    VEDA_DISPATCH(dtype, T,
                  silu_bwd_kernel<T><<<grid_for(n, 256), 256, 0, stream>>>(
                      static_cast<const T*>(x), static_cast<const T*>(g), static_cast<T*>(dx), n));
    count_launch();
    return check_launch("veda_silu_bwd");
}

extern "C" int veda_gelu_fwd(const void* x, void* y, int64_t n, int dtype, veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype) && n >= 0, "bad arguments");
    if (n == 0) return VEDA_OK;
    VEDA_REQUIRE(x && y, "null pointer");
    VEDA_DISPATCH(dtype, T,
                  gelu_fwd_kernel<T><<<grid_for(n, 256), 256, 0, stream>>>(
                      static_cast<const T*>(x), static_cast<T*>(y), n));
    count_launch();
    return check_launch("veda_gelu_fwd");
}

extern "C" int veda_gelu_bwd(const void* x, const void* g, void* dx, int64_t n, int dtype,
                             veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype) && n >= 0, "bad arguments");
    if (n == 0) return VEDA_OK;
    VEDA_REQUIRE(x && g && dx, "null pointer");
    VEDA_DISPATCH(dtype, T,
                  gelu_bwd_kernel<T><<<grid_for(n, 256), 256, 0, stream>>>(
                      static_cast<const T*>(x), static_cast<const T*>(g), static_cast<T*>(dx), n));
    count_launch();
    return check_launch("veda_gelu_bwd");
}

extern "C" int veda_argmax(const void* x, int64_t ld, int64_t rows, int64_t n, int64_t* out,
                           int* status, int dtype, veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype) && rows >= 0 && n > 0 && ld >= n, "bad arguments");
    if (rows == 0) return VEDA_OK;
    VEDA_REQUIRE(x && out, "null pointer");
    const unsigned grid = static_cast<unsigned>(
        rows < static_cast<int64_t>(sm_count()) * 8 ? rows : static_cast<int64_t>(sm_count()) * 8);
    VEDA_DISPATCH(dtype, T,
                  argmax_kernel<T><<<grid, 256, 0, stream>>>(static_cast<const T*>(x), ld, rows,
                                                             n, out, status));
    count_launch();
    return check_launch("veda_argmax");
}

extern "C" int veda_randn(void* x, int64_t n, float stddev, uint64_t seed, int dtype,
                          veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype) && n >= 0, "bad arguments");
    if (n == 0) return VEDA_OK;
    VEDA_REQUIRE(x != nullptr, "null pointer");
    VEDA_DISPATCH(dtype, T,
                  randn_kernel<T><<<grid_for(n, 256), 256, 0, stream>>>(static_cast<T*>(x), n,
                                                                        stddev, seed));
    count_launch();
    return check_launch("veda_randn");
}

extern "C" int veda_f32_to_bf16(const float* src, void* dst, int64_t n, veda_stream_t stream)
{
    VEDA_REQUIRE(n >= 0, "bad size");
    if (n == 0) return VEDA_OK;
    VEDA_REQUIRE(src && dst, "null pointer");
    f32_to_bf16_kernel<<<grid_for(n, 256), 256, 0, stream>>>(src, static_cast<bf16*>(dst), n);
    count_launch();
    return check_launch("veda_f32_to_bf16");
}
