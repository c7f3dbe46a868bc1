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
                   int64_t ldkv, int64_t len, int heads, int kv_heads, int head_dim, float scale,
                   T* __restrict__ out)
{
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

extern "C" int veda_attention_decode(const void* q, const void* k, const void* v, int64_t ldkv,
                                     int64_t len, int64_t heads, int64_t kv_heads, int64_t head_dim,
                                     float scale, void* out, int dtype, veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype), "unknown dtype");
    VEDA_REQUIRE(len > 0 && heads > 0 && kv_heads > 0 && heads % kv_heads == 0, "bad shape");
    VEDA_REQUIRE(head_dim > 0 && head_dim <= 256, "head_dim must lie in [1, 256]");
    VEDA_REQUIRE(ldkv >= kv_heads * head_dim, "bad cache leading dimension");
    VEDA_REQUIRE(q && k && v && out, "null pointer");
    const int dl = static_cast<int>((head_dim + 31) / 32);
#define VEDA_DEC(T, DL)                                                                               \
    attn_decode_kernel<T, DL><<<static_cast<unsigned>(heads), kDecodeWarps * 32, 0, stream>>>(       \
        static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), ldkv, len,      \
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
