// Token-by-token generation on the device: the attention of one new query per head against a KV
// cache (src/libs/model/ScaledDotProductAttention.cpp:138-191 for one query row): softmax over
// every cached position (all precede or equal the query, so no mask), weighted sum of the cached
// values; GQA query head h reads KV head h / (H / Hkv). The greedy choice of the next token is
// veda_argmax (elementwise.cu).
#include "common.cuh"


namespace veda::cuda
{
namespace
{

constexpr int kDecodeWarps = 4;

// One CTA per query head: each warp takes every kDecodeWarps-th cached position, keeps an online
// (max, sum, weighted value) in fp32, and the warps are merged in order. Lane l owns dimensions
// l, l + 32, ... of the head.
template <typename T, int DL>
__global__ void __launch_bounds__(kDecodeWarps * 32)
attn_decode_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                   int64_t ldkv, int64_t len, const int64_t* __restrict__ pos, int heads, int kv_heads,
                   int head_dim, float scale, T* __restrict__ out)
{
    if (pos != nullptr)
    {
        len = *pos + 1;   // the query sits at position *pos and sees every position up to it
    }
    __shared__ float s_m[kDecodeWarps], s_l[kDecodeWarps], s_acc[kDecodeWarps][DL * 32];
    const int h = blockIdx.x;
    const int kvh = h / (heads / kv_heads);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float qv[DL], acc[DL];
#pragma unroll
    for (int i = 0; i < DL; ++i)
    {
        const int d = lane + 32 * i;
        qv[i] = d < head_dim ? to_f32(q[static_cast<int64_t>(h) * head_dim + d]) : 0.0f;
        acc[i] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;
    for (int64_t j = warp; j < len; j += kDecodeWarps)
    {
        const T* kr = k + j * ldkv + static_cast<int64_t>(kvh) * head_dim;
        const T* vr = v + j * ldkv + static_cast<int64_t>(kvh) * head_dim;
        float dot = 0.0f;
#pragma unroll
        for (int i = 0; i < DL; ++i)
        {
            const int d = lane + 32 * i;
            if (d < head_dim) dot += qv[i] * to_f32(kr[d]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xFFFFFFFFu, dot, o);
        const float s = dot * scale;
        const float mn = fmaxf(m, s);
        const float corr = expf(m - mn);   // 0 on the first position (m = -inf)
        const float p = expf(s - mn);
        l = l * corr + p;
#pragma unroll
        for (int i = 0; i < DL; ++i)
        {
            const int d = lane + 32 * i;
            acc[i] = acc[i] * corr + (d < head_dim ? p * to_f32(vr[d]) : 0.0f);
        }
        m = mn;
    }
    if (lane == 0)
    {
        s_m[warp] = m;
        s_l[warp] = l;
    }
#pragma unroll
    for (int i = 0; i < DL; ++i) s_acc[warp][lane + 32 * i] = acc[i];
    __syncthreads();
    if (warp == 0)
    {
        float gm = -INFINITY;
        for (int w = 0; w < kDecodeWarps; ++w) gm = fmaxf(gm, s_m[w]);
        float gl = 0.0f, o[DL];
#pragma unroll
        for (int i = 0; i < DL; ++i) o[i] = 0.0f;
        for (int w = 0; w < kDecodeWarps; ++w)
        {
            const float c = s_m[w] == -INFINITY ? 0.0f : expf(s_m[w] - gm);
            gl += s_l[w] * c;
#pragma unroll
            for (int i = 0; i < DL; ++i) o[i] += s_acc[w][lane + 32 * i] * c;
        }
#pragma unroll
        for (int i = 0; i < DL; ++i)
        {
            const int d = lane + 32 * i;
            if (d < head_dim) out[static_cast<int64_t>(h) * head_dim + d] = from_f32<T>(o[i] / gl);
        }
    }
}

} // namespace
} // namespace veda::cuda

using namespace veda::cuda;

namespace
{
int launch_decode(const void* q, const void* k, const void* v, int64_t ldkv, int64_t len,
                  const int64_t* pos, int64_t heads, int64_t kv_heads, int64_t head_dim, float scale,
                  void* out, int dtype, veda_stream_t stream)
{
    const int dl = static_cast<int>((head_dim + 31) / 32);
#define VEDA_DEC(T, DL)                                                                               \
    attn_decode_kernel<T, DL><<<static_cast<unsigned>(heads), kDecodeWarps * 32, 0, stream>>>(       \
        static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), ldkv, len, pos, \
        static_cast<int>(heads), static_cast<int>(kv_heads), static_cast<int>(head_dim), scale,      \
        static_cast<T*>(out))
#define VEDA_DEC_DL(T)                                                                                \
    switch (dl)                                                                                        \
    {                                                                                                  \
    case 1: VEDA_DEC(T, 1); break;                                                                     \
    case 2: VEDA_DEC(T, 2); break;                                                                     \
    case 3: VEDA_DEC(T, 3); break;                                                                     \
    case 4: VEDA_DEC(T, 4); break;                                                                     \
    case 5: VEDA_DEC(T, 5); break;                                                                     \
    case 6: VEDA_DEC(T, 6); break;                                                                     \
    case 7: VEDA_DEC(T, 7); break;                                                                     \
    default: VEDA_DEC(T, 8); break;                                                                    \
    }
    if (dtype == VEDA_BF16)
    {
        VEDA_DEC_DL(bf16)
    }
    else
    {
        VEDA_DEC_DL(float)
    }
#undef VEDA_DEC_DL
#undef VEDA_DEC
    count_launch();
    return check_launch("veda_attention_decode");
}
} // namespace

extern "C" int veda_attention_decode(const void* q, const void* k, const void* v, int64_t ldkv,
                                     int64_t len, int64_t heads, int64_t kv_heads, int64_t head_dim,
                                     float scale, void* out, int dtype, veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype), "unknown dtype");
    VEDA_REQUIRE(len > 0 && heads > 0 && kv_heads > 0 && heads % kv_heads == 0, "bad shape");
    VEDA_REQUIRE(head_dim > 0 && head_dim <= 256, "head_dim must lie in [1, 256]");
    VEDA_REQUIRE(ldkv >= kv_heads * head_dim, "bad cache leading dimension");
    VEDA_REQUIRE(q && k && v && out, "null pointer");
    return launch_decode(q, k, v, ldkv, len, nullptr, heads, kv_heads, head_dim, scale, out, dtype,
                         stream);
}

extern "C" int veda_attention_decode_at(const void* q, const void* k, const void* v, int64_t ldkv,
                                        const int64_t* pos, int64_t heads, int64_t kv_heads,
                                        int64_t head_dim, float scale, void* out, int dtype,
                                        veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype), "unknown dtype");
    VEDA_REQUIRE(heads > 0 && kv_heads > 0 && heads % kv_heads == 0, "bad shape");
    VEDA_REQUIRE(head_dim > 0 && head_dim <= 256, "head_dim must lie in [1, 256]");
    VEDA_REQUIRE(ldkv >= kv_heads * head_dim, "bad cache leading dimension");
    VEDA_REQUIRE(q && k && v && out && pos, "null pointer");
    return launch_decode(q, k, v, ldkv, 0, pos, heads, kv_heads, head_dim, scale, out, dtype, stream);
}

// One token's q, k, v at the position held in device memory: QK-norm (x / sqrt(mean(x^2) + eps)
// * gain, Model.cpp:173-178) and RoPE (half-split rotation by the table row of that position,
// Views.cpp:78-134) for every query head into q_out and every KV head into its cache row, and the
// values copied into theirs. Block b: query head b, KV head b - H, or value head b - H - Hkv.
template <typename T>
__global__ void __launch_bounds__(128)
decode_qkv_kernel(const T* __restrict__ qkv, const T* __restrict__ qgain, const T* __restrict__ kgain,
                  const float* __restrict__ cosv, const float* __restrict__ sinv,
                  const int64_t* __restrict__ pos, T* __restrict__ q_out, T* __restrict__ k_cache,
                  T* __restrict__ v_cache, int64_t ldkv, int heads, int kv_heads, int head_dim,
                  float eps)
{
    __shared__ float red[4];
    const int64_t p = *pos;
    const int b = blockIdx.x, tid = threadIdx.x;
    if (b >= heads + kv_heads)
    {
        const int vh = b - heads - kv_heads;
        const T* src = qkv + static_cast<int64_t>(heads + kv_heads + vh) * head_dim;
        T* dst = v_cache + p * ldkv + static_cast<int64_t>(vh) * head_dim;
        for (int d = tid; d < head_dim; d += blockDim.x) dst[d] = src[d];
        return;
    }
    const bool is_q = b < heads;
    const T* x = qkv + static_cast<int64_t>(b) * head_dim;   // q heads, then k heads, in order
    const T* gain = is_q ? qgain : kgain;
    float ss = 0.0f;
    for (int d = tid; d < head_dim; d += blockDim.x)
    {
        const float v = to_f32(x[d]);
        ss += v * v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    ss = 0.0f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) ss += red[w];
    const float r = sqrtf(ss / static_cast<float>(head_dim) + eps);   // x / r, as RMSNorm divides
    T* dst = is_q ? q_out + static_cast<int64_t>(b) * head_dim
                  : k_cache + p * ldkv + static_cast<int64_t>(b - heads) * head_dim;
    const int half = head_dim / 2;
    const float* cr = cosv + p * head_dim;
    const float* sr = sinv + p * head_dim;
    for (int d = tid; d < half; d += blockDim.x)
    {
        const float a = (to_f32(x[d]) / r) * to_f32(gain[d]);
        const float c = (to_f32(x[d + half]) / r) * to_f32(gain[d + half]);
        dst[d] = from_f32<T>(a * cr[d] - c * sr[d]);
        dst[d + half] = from_f32<T>(c * cr[d] + a * sr[d]);
    }
}

__global__ void advance_kernel(int64_t* pos)
{
    *pos += 1;
}

extern "C" int veda_decode_qkv_at(const void* qkv, const void* q_gain, const void* k_gain,
                                  const float* cos, const float* sin, const int64_t* pos,
                                  void* q_out, void* k_cache, void* v_cache, int64_t ldkv,
                                  int64_t heads, int64_t kv_heads, int64_t head_dim, float eps,
                                  int dtype, veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype), "unknown dtype");
    VEDA_REQUIRE(heads > 0 && kv_heads > 0 && head_dim > 0 && head_dim % 2 == 0, "bad shape");
    VEDA_REQUIRE(ldkv >= kv_heads * head_dim, "bad cache leading dimension");
    VEDA_REQUIRE(qkv && q_gain && k_gain && cos && sin && pos && q_out && k_cache && v_cache,
                 "null pointer");
    const unsigned blocks = static_cast<unsigned>(heads + 2 * kv_heads);
#define VEDA_QKV(T)                                                                                   \
    decode_qkv_kernel<T><<<blocks, 128, 0, stream>>>(                                                 \
        static_cast<const T*>(qkv), static_cast<const T*>(q_gain), static_cast<const T*>(k_gain), cos, \
        sin, pos, static_cast<T*>(q_out), static_cast<T*>(k_cache), static_cast<T*>(v_cache), ldkv,   \
        static_cast<int>(heads), static_cast<int>(kv_heads), static_cast<int>(head_dim), eps)
    if (dtype == VEDA_BF16) VEDA_QKV(bf16); else VEDA_QKV(float);
#undef VEDA_QKV
    count_launch();
    return check_launch("veda_decode_qkv_at");
}

extern "C" int veda_decode_advance(int64_t* pos, veda_stream_t stream)
{
    VEDA_REQUIRE(pos != nullptr, "null pointer");
    advance_kernel<<<1, 1, 0, stream>>>(pos);
    count_launch();
    return check_launch("veda_decode_advance");
}

// ---- the decode step's Linear layers at one row --------------------------------------------
// y[n] = sum_k x[k] * w[n, k] (matmul_nt, Variable.cpp:325, for a single activation row). Every weight
// byte is read once and nothing is reused, so the bound is HBM bandwidth, not the tensor cores: a
// warp owns R weight rows, each lane streams 16-byte pieces of them (L1 bypassed) against the
// activation staged in shared memory, accumulates in fp32 with fmaf in piece order, and the warp
// reduces the row sums and rounds each to the output dtype once. kGemvUnroll pieces per row are
// loaded before any is used, so R * kGemvUnroll 16-byte loads per lane are in flight.
namespace veda::cuda
{
namespace
{
constexpr int kGemvWarps = 8;
constexpr int kGemvUnroll = 4;
constexpr int64_t kGemvSmem = 48 * 1024;   // the activation row, staged whole

__device__ __forceinline__ uint4 load_stream16(const void* p)
{
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p));
    return v;
}

template <typename T>
__device__ __forceinline__ void unpack16(const uint4 raw, float (&out)[16 / sizeof(T)])
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

__device__ __forceinline__ float silu_gate(float g) { return g * __fdividef(1.0f, 1.0f + __expf(-g)); }

// SWIGLU: the warp's two rows are gate row j and up row n + j of the fused [2n, k] weight, and the
// output is h[j] = silu(g) * u on the values rounded to the dtype (the separate Linear then SwiGLU
// of Model.cpp:198-204, same arithmetic as veda_swiglu_fwd).
template <typename T, int R, bool SWIGLU, bool VEC>
__global__ void __launch_bounds__(kGemvWarps * 32)
gemv_kernel(const T* __restrict__ x, const T* __restrict__ w, int64_t ldw, T* __restrict__ y, int n, int k)
{
    extern __shared__ __align__(16) unsigned char gemv_smem[];
    T* xs = reinterpret_cast<T*>(gemv_smem);
    constexpr int E = 16 / sizeof(T);
    if constexpr (VEC)
    {
        for (int i = threadIdx.x * E; i < k; i += blockDim.x * E)
            *reinterpret_cast<uint4*>(xs + i) = *reinterpret_cast<const uint4*>(x + i);
    }
    else
    {
        for (int i = threadIdx.x; i < k; i += blockDim.x) xs[i] = x[i];
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int per_warp = SWIGLU ? 1 : R;
    const int base = (blockIdx.x * kGemvWarps + warp) * per_warp;
    if (base >= n) return;
    const T* rows[R];
#pragma unroll
    for (int r = 0; r < R; ++r)
    {
        const int row = SWIGLU ? base : min(base + r, n - 1);   // a row past n repeats the last one
        rows[r] = w + (static_cast<int64_t>(row) + (SWIGLU ? static_cast<int64_t>(r) * n : 0)) * ldw;
    }
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.0f;
    if constexpr (VEC)
    {
        for (int c0 = lane * E; c0 < k; c0 += 32 * E * kGemvUnroll)
        {
            uint4 wv[kGemvUnroll][R];
#pragma unroll
            for (int u = 0; u < kGemvUnroll; ++u)
            {
                const int c = c0 + u * 32 * E;
#pragma unroll
                for (int r = 0; r < R; ++r)
                    if (c < k) wv[u][r] = load_stream16(rows[r] + c);
            }
#pragma unroll
            for (int u = 0; u < kGemvUnroll; ++u)
            {
                const int c = c0 + u * 32 * E;
                if (c < k)
                {
                    float xv[E];
                    load16(xs + c, xv);
#pragma unroll
                    for (int r = 0; r < R; ++r)
                    {
                        float wf[E];
                        unpack16<T>(wv[u][r], wf);
#pragma unroll
                        for (int j = 0; j < E; ++j) acc[r] = fmaf(xv[j], wf[j], acc[r]);
                    }
                }
            }
        }
    }
    else
    {
        for (int c = lane; c < k; c += 32)
        {
            const float xv = to_f32(xs[c]);
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r] = fmaf(xv, to_f32(rows[r][c]), acc[r]);
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = warp_sum(acc[r]);
    if (lane != 0) return;
    if constexpr (SWIGLU)
    {
        const float g = to_f32(from_f32<T>(acc[0])), u = to_f32(from_f32<T>(acc[1]));
        y[base] = from_f32<T>(silu_gate(g) * u);
    }
    else
    {
#pragma unroll
        for (int r = 0; r < R; ++r)
            if (base + r < n) y[base + r] = from_f32<T>(acc[r]);
    }
}

template <typename T, int R, bool SWIGLU>
void launch_gemv(const void* x, const void* w, int64_t ldw, void* y, int64_t n, int64_t k, bool vec,
                 cudaStream_t stream)
{
    constexpr int per_warp = SWIGLU ? 1 : R;
    const auto blocks = static_cast<unsigned>((n + kGemvWarps * per_warp - 1) / (kGemvWarps * per_warp));
    const size_t smem = static_cast<size_t>(k) * sizeof(T);
    const auto xp = static_cast<const T*>(x);
    const auto wp = static_cast<const T*>(w);
    const auto yp = static_cast<T*>(y);
    if (vec)
        gemv_kernel<T, R, SWIGLU, true><<<blocks, kGemvWarps * 32, smem, stream>>>(
            xp, wp, ldw, yp, static_cast<int>(n), static_cast<int>(k));
    else
        gemv_kernel<T, R, SWIGLU, false><<<blocks, kGemvWarps * 32, smem, stream>>>(
            xp, wp, ldw, yp, static_cast<int>(n), static_cast<int>(k));
}

int gemv_checks(const void* x, const void* w, int64_t ldw, const void* y, int64_t n, int64_t k, int dtype)
{
    VEDA_REQUIRE(valid_dtype(dtype), "unknown dtype");
    VEDA_REQUIRE(x && w && y, "null pointer");
    VEDA_REQUIRE(n > 0 && k > 0 && n < (1ll << 30), "bad shape");
    VEDA_REQUIRE(ldw >= k, "bad weight leading dimension");
    VEDA_REQUIRE(k * static_cast<int64_t>(dtype_size(dtype)) <= kGemvSmem,
                 "the activation row exceeds the 48 KB staged in shared memory");
    return 0;
}

bool gemv_vec(const void* x, const void* w, int64_t ldw, int64_t k, int dtype)
{
    const int64_t e = 16 / static_cast<int64_t>(dtype_size(dtype));
    return aligned16(x) && aligned16(w) && k % e == 0 && ldw % e == 0;
}
} // namespace
} // namespace veda::cuda

extern "C" int veda_gemv_nt(const void* x, const void* w, int64_t ldw, void* y, int64_t n, int64_t k,
                            int dtype, veda_stream_t stream)
{
    if (const int rc = gemv_checks(x, w, ldw, y, n, k, dtype)) return rc;
    const bool vec = gemv_vec(x, w, ldw, k, dtype);
    // two rows a warp once there are enough rows to fill the SMs with them
    const bool two = n >= 8192;
    if (dtype == VEDA_BF16)
    {
        if (two) launch_gemv<bf16, 2, false>(x, w, ldw, y, n, k, vec, stream);
        else launch_gemv<bf16, 1, false>(x, w, ldw, y, n, k, vec, stream);
    }
    else
    {
        if (two) launch_gemv<float, 2, false>(x, w, ldw, y, n, k, vec, stream);
        else launch_gemv<float, 1, false>(x, w, ldw, y, n, k, vec, stream);
    }
    count_launch();
    return check_launch("veda_gemv_nt");
}

extern "C" int veda_gemv_swiglu(const void* x, const void* w_gate_up, int64_t ldw, void* h, int64_t f,
                                int64_t k, int dtype, veda_stream_t stream)
{
    if (const int rc = gemv_checks(x, w_gate_up, ldw, h, f, k, dtype)) return rc;
    const bool vec = gemv_vec(x, w_gate_up, ldw, k, dtype);
    if (dtype == VEDA_BF16) launch_gemv<bf16, 2, true>(x, w_gate_up, ldw, h, f, k, vec, stream);
    else launch_gemv<float, 2, true>(x, w_gate_up, ldw, h, f, k, vec, stream);
    count_launch();
    return check_launch("veda_gemv_swiglu");
}
