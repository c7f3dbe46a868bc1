// Token-by-token generation on the device. The attention of one new query per head against a KV
// cache (src/libs/model/ScaledDotProductAttention.cpp:138-191 for one query row): softmax over
// every cached position (all precede or equal the query, so no mask), weighted sum of the cached
// values; GQA query head h reads KV head h / (H / Hkv). Then the kernels of one recorded decode
// step: one-row GEMVs for the Linear layers (the pre-norm, SwiGLU or the greedy argmax fused in),
// the token's q/k/v handling fused with a split-position attention, and the position increment.
#include "common.cuh"

#include <algorithm>


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
constexpr int kGemvBlocksPerSm = 4;   // registers capped at 64 a thread
// The activation row (and the norm's gain) staged whole in dynamic shared memory: 48 KB a block
// can have without opting in to more, less 1 KB for the kernels' own static arrays (at most 112
// bytes), so every accepted size launches.
constexpr int64_t kGemvSmem = 47 * 1024;

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
// NORM: the activation is RMSNorm(s) * gamma of the residual row s = x (+ r), computed by every
// block into its shared copy (the pre-norm of Model.cpp:242-249 ahead of its Linear layer): s is
// rounded to the dtype as the residual add stores it, and block 0 writes it to sum_out; the sum of
// squares is taken by all threads in a fixed order, y = (s / rms) * gamma rounded once.
// PICK: the greedy choice over the outputs as well (argmax of the rounded values, ties to the lower
// index, a NaN anywhere an error: Sampling.cpp:97-113): each block's best goes to `part`, and the
// last block to finish (atomic arrival count, no block waits) reduces them into *token.
struct GemvPick
{
    int64_t* token = nullptr;
    int* status = nullptr;
    unsigned* counter = nullptr;
    float* val = nullptr;   // per block
    int* idx = nullptr;     // per block; -2 marks a NaN
};

// (v, i) is the better candidate than (bv, bi): larger, or equal with the lower index.
__device__ __forceinline__ bool better(float v, int i, float bv, int bi)
{
    return i >= 0 && (bi < 0 || v > bv || (v == bv && i < bi));
}

// Blocks loop over tiles of kGemvWarps * (rows per warp) rows, so a grid of a few blocks per SM
// pays the activation staging (and the norm) once per block however large n is.
// KS > 1 (16-byte path only): KS consecutive warps share a row group, warp part p taking the
// 16-byte pieces p, p + KS, ... of each row, their sums added in part order through shared memory;
// fewer dependent load rounds per row where k is long (o and down projections).
template <typename T, int R, bool SWIGLU, bool VEC, bool NORM, bool PICK = false, int KS = 1>
__global__ void __launch_bounds__(kGemvWarps * 32, kGemvBlocksPerSm)
gemv_kernel(const T* __restrict__ x, const T* __restrict__ w, int64_t ldw, T* __restrict__ y, int n, int k,
            const T* __restrict__ r_in, const T* __restrict__ gamma, T* __restrict__ sum_out, float eps,
            GemvPick pick = GemvPick{})
{
    extern __shared__ __align__(16) unsigned char gemv_smem[];
    T* xs = reinterpret_cast<T*>(gemv_smem);
    constexpr int E = 16 / sizeof(T);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int per_warp = SWIGLU ? 1 : R;   // output rows of a row group
    constexpr int groups = kGemvWarps / KS;
    constexpr int tile_rows = groups * per_warp;
    const int group = warp / KS, part = warp % KS;
    constexpr int PSTEP = KS * 32 * E;          // elements from one of a warp's pieces to its next
    const int tiles = (n + tile_rows - 1) / tile_rows;
    auto row_ptrs = [&](int base, const T* (&rows)[R]) {
#pragma unroll
        for (int r = 0; r < R; ++r)
        {
            const int row = min(SWIGLU ? base : base + r, n - 1);   // a row past n repeats the last one
            rows[r] = w + (static_cast<int64_t>(row) + (SWIGLU ? static_cast<int64_t>(r) * n : 0)) * ldw;
        }
    };
    auto load_pieces = [&](const T* const (&rows)[R], int c0, uint4 (&wv)[kGemvUnroll][R]) {
#pragma unroll
        for (int u = 0; u < kGemvUnroll; ++u)
        {
            const int c = c0 + u * PSTEP;
#pragma unroll
            for (int r = 0; r < R; ++r)
                if (c < k) wv[u][r] = load_stream16(rows[r] + c);
        }
    };
    // The first pieces of this block's first rows do not depend on the activation: their loads are
    // issued before it is staged, so the HBM latency overlaps the staging (and the norm). A warp
    // past n computes a copy of row n - 1 and drops it.
    uint4 wv0[kGemvUnroll][R];
    if constexpr (VEC)
    {
        const T* rows0[R];
        row_ptrs((blockIdx.x * groups + group) * per_warp, rows0);
        load_pieces(rows0, lane * E + part * 32 * E, wv0);
    }
    if constexpr (NORM)
    {
        __shared__ float inv_s;
        __shared__ float ss_s[kGemvWarps];
        T* gs = xs + k;   // the gain, staged with the row so its loads overlap the row's
        // sum of squares: each thread over the elements it stages, then across the warp, then the
        // warps in order (fixed, so every block computes the same value)
        float ss = 0.0f;
        for (int i = threadIdx.x; i < k; i += blockDim.x)
        {
            float v = to_f32(x[i]);
            if (r_in != nullptr) v += to_f32(r_in[i]);
            gs[i] = gamma[i];
            const T t = from_f32<T>(v);
            xs[i] = t;
            if (blockIdx.x == 0 && sum_out != nullptr) sum_out[i] = t;
            const float tv = to_f32(t);
            ss += tv * tv;
        }
        ss = warp_sum(ss);
        if (lane == 0) ss_s[warp] = ss;
        __syncthreads();
        if (threadIdx.x == 0)
        {
            float total = 0.0f;
            for (int q = 0; q < kGemvWarps; ++q) total += ss_s[q];
            inv_s = 1.0f / sqrtf(total / static_cast<float>(k) + eps);
        }
        __syncthreads();
        const float inv = inv_s;
        for (int i = threadIdx.x; i < k; i += blockDim.x)
            xs[i] = from_f32<T>((to_f32(xs[i]) * inv) * to_f32(gs[i]));
    }
    else if constexpr (VEC)
    {
        for (int i = threadIdx.x * E; i < k; i += blockDim.x * E)
            *reinterpret_cast<uint4*>(xs + i) = *reinterpret_cast<const uint4*>(x + i);
    }
    else
    {
        for (int i = threadIdx.x; i < k; i += blockDim.x) xs[i] = x[i];
    }
    __syncthreads();

    float best = -INFINITY;   // PICK: this warp's best output so far, rows in ascending order
    int best_i = -1;
    bool nan = false;
    float acc[R];
    auto consume = [&](const uint4 (&wv)[kGemvUnroll][R], int c0) {
#pragma unroll
        for (int u = 0; u < kGemvUnroll; ++u)
        {
            const int c = c0 + u * PSTEP;
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
    };
    // the pieces of a tile's rows from c0 on (16-byte pieces), or every element (VEC false)
    auto dot_from = [&](const T* const (&rows)[R], int c0) {
        if constexpr (VEC)
        {
            for (; c0 < k; c0 += PSTEP * kGemvUnroll)
            {
                uint4 wv[kGemvUnroll][R];
                load_pieces(rows, c0, wv);
                consume(wv, c0);
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
    };
    __shared__ float ks_s[KS > 1 ? kGemvWarps : 1][R];
    auto finish = [&](int base) {
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = warp_sum(acc[r]);
        if constexpr (KS > 1)
        {
            if (lane == 0)
            {
#pragma unroll
                for (int r = 0; r < R; ++r) ks_s[warp][r] = acc[r];
            }
            __syncthreads();
            if (part == 0)
            {
#pragma unroll
                for (int r = 0; r < R; ++r)
                {
                    acc[r] = ks_s[warp][r];
                    for (int q = 1; q < KS; ++q) acc[r] += ks_s[warp + q][r];
                }
            }
            __syncthreads();   // ks_s is free for the next tile
            if (part != 0) return;
        }
        if (lane != 0 || base >= n) return;
        if constexpr (SWIGLU)
        {
            const float g = to_f32(from_f32<T>(acc[0])), u = to_f32(from_f32<T>(acc[1]));
            y[base] = from_f32<T>(silu_gate(g) * u);
        }
        else
        {
#pragma unroll
            for (int r = 0; r < R; ++r)
            {
                if (base + r < n)
                {
                    const T t = from_f32<T>(acc[r]);
                    y[base + r] = t;
                    if constexpr (PICK)
                    {
                        const float v = to_f32(t);
                        if (v != v) nan = true;
                        else if (better(v, base + r, best, best_i)) { best = v; best_i = base + r; }
                    }
                }
            }
        }
    };
    {
        // the block's first tile, its first pieces already loaded
        const int base = (blockIdx.x * groups + group) * per_warp;
        const T* rows[R];
        row_ptrs(base, rows);
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = 0.0f;
        if constexpr (VEC)
        {
            consume(wv0, lane * E + part * 32 * E);
            dot_from(rows, lane * E + part * 32 * E + PSTEP * kGemvUnroll);
        }
        else
        {
            dot_from(rows, 0);
        }
        finish(base);
    }
    for (int tile = blockIdx.x + gridDim.x; tile < tiles; tile += gridDim.x)
    {
        const int base = (tile * groups + group) * per_warp;
        const T* rows[R];
        row_ptrs(base, rows);
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = 0.0f;
        dot_from(rows, VEC ? lane * E + part * 32 * E : 0);
        finish(base);
    }
    if constexpr (PICK)
    {
        __shared__ float pv_s[kGemvWarps];
        __shared__ int pi_s[kGemvWarps];
        __shared__ bool last_s;
        if (lane == 0)
        {
            pv_s[warp] = best;
            pi_s[warp] = best_i;
        }
        const bool block_nan = __syncthreads_or(nan);
        if (threadIdx.x == 0)
        {
            float b = -INFINITY;
            int j = -1;
            for (int q = 0; q < kGemvWarps; ++q)
                if (better(pv_s[q], pi_s[q], b, j)) { b = pv_s[q]; j = pi_s[q]; }
            pick.val[blockIdx.x] = b;
            pick.idx[blockIdx.x] = block_nan ? -2 : j;
            __threadfence();
            last_s = atomicAdd(pick.counter, 1u) == gridDim.x - 1;
        }
        __syncthreads();
        if (!last_s) return;
        __threadfence();
        float b = -INFINITY;
        int j = -1;
        bool bad = false;
        for (int q = threadIdx.x; q < static_cast<int>(gridDim.x); q += blockDim.x)
        {
            const int qi = __ldcg(pick.idx + q);
            const float qv = __ldcg(pick.val + q);
            if (qi == -2) bad = true;
            else if (better(qv, qi, b, j)) { b = qv; j = qi; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
        {
            const float ov = __shfl_xor_sync(0xFFFFFFFFu, b, o);
            const int oi = __shfl_xor_sync(0xFFFFFFFFu, j, o);
            if (better(ov, oi, b, j)) { b = ov; j = oi; }
        }
        if (lane == 0)
        {
            pv_s[warp] = b;
            pi_s[warp] = j;
        }
        bad = __syncthreads_or(bad);
        if (threadIdx.x == 0)
        {
            for (int q = 1; q < kGemvWarps; ++q)
                if (better(pv_s[q], pi_s[q], pv_s[0], pi_s[0])) { pv_s[0] = pv_s[q]; pi_s[0] = pi_s[q]; }
            *pick.token = bad ? -1 : pi_s[0];
            if (bad && pick.status != nullptr) *pick.status = VEDA_ERR_INVALID_ARGUMENT;
            *pick.counter = 0u;   // ready for the next call
        }
    }
}

// Blocks of a launch over n rows, per_warp rows a warp: one per tile up to kGemvBlocksPerSm per SM
// (the blocks the kernel's launch bounds keep resident at once), tiles beyond that looped over.
int64_t gemv_grid(int64_t n, int per_warp, int ks = 1)
{
    const int64_t tile_rows = static_cast<int64_t>(kGemvWarps / ks) * per_warp;
    const int64_t tiles = (n + tile_rows - 1) / tile_rows;
    return std::min<int64_t>(tiles, static_cast<int64_t>(sm_count()) * kGemvBlocksPerSm);
}

// Warps a row group is split across: one per round of kGemvUnroll 16-byte pieces a lane would
// otherwise load one after another (1024 bf16 or 512 fp32 elements a round), up to 4.
int gemv_split(int64_t k, int dtype)
{
    const int64_t per_round = 32 * kGemvUnroll * (16 / static_cast<int64_t>(dtype_size(dtype)));
    const int64_t rounds = (k + per_round - 1) / per_round;
    return rounds >= 3 ? 4 : static_cast<int>(rounds);
}

// The pre-norm operands of a NORM launch (all null for a plain one).
struct GemvNorm
{
    const void* r = nullptr;
    const void* gamma = nullptr;
    void* sum = nullptr;
    float eps = 0.0f;
};

template <typename T, int R, bool SWIGLU>
void launch_gemv(const void* x, const void* w, int64_t ldw, void* y, int64_t n, int64_t k, bool vec,
                 const GemvNorm* norm, cudaStream_t stream)
{
    constexpr int per_warp = SWIGLU ? 1 : R;
    const int ks = vec ? gemv_split(k, sizeof(T) == 2 ? VEDA_BF16 : VEDA_F32) : 1;
    const auto blocks = static_cast<unsigned>(gemv_grid(n, per_warp, ks));
    const size_t smem = static_cast<size_t>(k) * sizeof(T) * (norm != nullptr ? 2 : 1);
    const auto xp = static_cast<const T*>(x);
    const auto wp = static_cast<const T*>(w);
    const auto yp = static_cast<T*>(y);
    const auto ni = static_cast<int>(n), ki = static_cast<int>(k);
    const auto rp = norm ? static_cast<const T*>(norm->r) : nullptr;
    const auto gp = norm ? static_cast<const T*>(norm->gamma) : nullptr;
    const auto sp = norm ? static_cast<T*>(norm->sum) : nullptr;
    const float eps = norm ? norm->eps : 0.0f;
#define VEDA_GEMV(V, N, KS)                                                                            \
    gemv_kernel<T, R, SWIGLU, V, N, false, KS><<<blocks, kGemvWarps * 32, smem, stream>>>(xp, wp, ldw, yp, \
                                                                                         ni, ki, rp, gp,   \
                                                                                         sp, eps)
#define VEDA_GEMV_KS(N)                                                                                \
    if (!vec) VEDA_GEMV(false, N, 1);                                                                  \
    else if (ks == 4) VEDA_GEMV(true, N, 4);                                                           \
    else if (ks == 2) VEDA_GEMV(true, N, 2);                                                           \
    else VEDA_GEMV(true, N, 1)
    if (norm != nullptr)
    {
        VEDA_GEMV_KS(true);
    }
    else
    {
        VEDA_GEMV_KS(false);
    }
#undef VEDA_GEMV_KS
#undef VEDA_GEMV
}

// ---- the decode step's attention, fused with the q/k/v handling of its token ---------------
// CTAs (KV head, slice of the positions) serve the G = H / Hkv query heads that read the KV head
// (Dh = 128). Warps first take QK-norm + RoPE of those query heads (into shared memory, rounded to
// the dtype as the projection output would be stored); the CTA whose slice holds *pos also
// normalises and rotates the KV head's new key into cache row *pos and copies its value row. Then
// the 2 * WARPS half-warps walk the slice's positions, lane l of a half-warp holding dimensions
// [8l, 8l + 8), U positions per half-warp loaded before any is used, each keeping an online
// softmax state per query head in fp32; half-warps merge through shuffles, warps through shared
// memory, slices through the workspace (the last CTA of the KV head to finish). Every cached key
// and value is read once per KV head instead of once per query head. WARPS and U: 16 and 4 for
// G <= 2 (128 positions in flight per CTA), fewer where G's per-head registers need the room.
constexpr int kFusedDim = 128;

template <typename T>
struct Raw8
{
    uint4 v[sizeof(T) / 2];   // 8 elements: one 16-byte vector (bf16) or two (fp32)
};

template <typename T>
__device__ __forceinline__ Raw8<T> load_raw8(const T* p)
{
    Raw8<T> r;
#pragma unroll
    for (int i = 0; i < static_cast<int>(sizeof(T) / 2); ++i) r.v[i] = reinterpret_cast<const uint4*>(p)[i];
    return r;
}

template <typename T>
__device__ __forceinline__ void unpack_raw8(const Raw8<T>& r, float (&o)[8])
{
    if constexpr (sizeof(T) == 2)
    {
        unpack16<T>(r.v[0], o);
    }
    else
    {
        float a[4], b[4];
        unpack16<T>(r.v[0], a);
        unpack16<T>(r.v[1], b);
#pragma unroll
        for (int i = 0; i < 4; ++i)
        {
            o[i] = a[i];
            o[4 + i] = b[i];
        }
    }
}

template <typename T, int G, int WARPS, int U>
__global__ void __launch_bounds__(WARPS * 32)
decode_attn_fused_kernel(const T* __restrict__ qkv, const T* __restrict__ qgain, const T* __restrict__ kgain,
                         const float* __restrict__ cosv, const float* __restrict__ sinv,
                         const int64_t* __restrict__ pos, T* __restrict__ k_cache, T* __restrict__ v_cache,
                         int64_t ldkv, int kv_heads, float eps, float scale, T* __restrict__ out,
                         int64_t capacity, int64_t chunk, float* __restrict__ part,
                         unsigned* __restrict__ counters)
{
    constexpr int D = kFusedDim;
    constexpr int S = WARPS * 2;   // half-warps, each a stride-S slice of the positions
    __shared__ __align__(16) float q_s[G][D];
    __shared__ float m_s[WARPS][G], l_s[WARPS][G];
    __shared__ __align__(16) float acc_s[WARPS][G][D];
    __shared__ bool last_s;
    const int64_t p = *pos;
    if (p < 0 || p >= capacity) return;   // a position outside the cache writes nothing
    const int kvh = blockIdx.x;
    const int heads = kv_heads * G;
    // this CTA's slice of the positions 0..p; the slice holding p also writes the new key and value
    const int split = blockIdx.y;
    const int64_t lo = static_cast<int64_t>(split) * chunk;
    if (lo > p) return;
    const int64_t hi = min(lo + chunk, p + 1);
    const int active = static_cast<int>(p / chunk) + 1;
    const bool owner = split == active - 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // item g < G: query head kvh * G + g; item G: the key; item G + 1: the value
    for (int item = warp; item < G + 2; item += WARPS)
    {
        if (item >= G && !owner) continue;
        if (item == G + 1)
        {
            const T* src = qkv + static_cast<int64_t>(heads + kv_heads + kvh) * D;
            T* dst = v_cache + p * ldkv + static_cast<int64_t>(kvh) * D;
            for (int d = lane; d < D; d += 32) dst[d] = src[d];
            continue;
        }
        const bool is_q = item < G;
        const T* src = qkv + static_cast<int64_t>(is_q ? kvh * G + item : heads + kvh) * D;
        const T* gain = is_q ? qgain : kgain;
        // every load of the item first (row, gain, and the rotation's table row), then the math
        float xv[4], gv[4], cv[2], sv[2], ss = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i)
        {
            xv[i] = to_f32(src[lane + 32 * i]);
            gv[i] = to_f32(gain[lane + 32 * i]);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i)
        {
            cv[i] = cosv[p * D + lane + 32 * i];
            sv[i] = sinv[p * D + lane + 32 * i];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) ss += xv[i] * xv[i];
        ss = warp_sum(ss);
        const float r = sqrtf(ss / static_cast<float>(D) + eps);   // x / r, as RMSNorm divides
        float a[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = (xv[i] / r) * gv[i];
        // half-split rotation: dimension d < 64 pairs with d + 64 (lane + 32 i with lane + 32 (i + 2))
        float o[4];
#pragma unroll
        for (int i = 0; i < 2; ++i)
        {
            o[i] = a[i] * cv[i] - a[i + 2] * sv[i];
            o[i + 2] = a[i + 2] * cv[i] + a[i] * sv[i];
        }
        if (is_q)
        {
#pragma unroll
            for (int i = 0; i < 4; ++i) q_s[item][lane + 32 * i] = to_f32(from_f32<T>(o[i]));
        }
        else
        {
            T* dst = k_cache + p * ldkv + static_cast<int64_t>(kvh) * D;
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = from_f32<T>(o[i]);
        }
    }
    __syncthreads();   // the new key and value rows and the queries are visible to the whole block

    const int hw = lane >> 4, hl = lane & 15;
    const unsigned half = 0xFFFFu << (16 * hw);
    const int slot = warp * 2 + hw;
    const int d0 = hl * 8;
    float qf[G][8], m[G], l[G], acc[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g)
    {
#pragma unroll
        for (int i = 0; i < 8; ++i)
        {
            qf[g][i] = q_s[g][d0 + i];
            acc[g][i] = 0.0f;
        }
        m[g] = -INFINITY;
        l[g] = 0.0f;
    }
    const T* kb = k_cache + static_cast<int64_t>(kvh) * D + d0;
    const T* vb = v_cache + static_cast<int64_t>(kvh) * D + d0;
    auto step = [&](const Raw8<T>& kr, const Raw8<T>& vr) {
        float kf[8], vf[8], dot[G];
        unpack_raw8<T>(kr, kf);
#pragma unroll
        for (int g = 0; g < G; ++g)
        {
            dot[g] = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) dot[g] += qf[g][i] * kf[i];
        }
#pragma unroll
        for (int g = 0; g < G; ++g)
        {
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) dot[g] += __shfl_xor_sync(half, dot[g], o);
        }
        unpack_raw8<T>(vr, vf);
#pragma unroll
        for (int g = 0; g < G; ++g)
        {
            const float sc = dot[g] * scale;
            const float mn = fmaxf(m[g], sc);
            const float corr = expf(m[g] - mn);   // 0 on the first position (m = -inf)
            const float pe = expf(sc - mn);
            l[g] = l[g] * corr + pe;
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[g][i] = acc[g][i] * corr + pe * vf[i];
            m[g] = mn;
        }
    };
    for (int64_t j0 = lo + slot; j0 < hi; j0 += U * S)
    {
        Raw8<T> kr[U], vr[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
        {
            const int64_t j = j0 + u * S;
            if (j < hi)
            {
                kr[u] = load_raw8(kb + j * ldkv);
                vr[u] = load_raw8(vb + j * ldkv);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (j0 + u * S < hi) step(kr[u], vr[u]);
    }

    // merge the two half-warps of each warp, then the warps
#pragma unroll
    for (int g = 0; g < G; ++g)
    {
        const float m2 = __shfl_xor_sync(0xFFFFFFFFu, m[g], 16);
        const float l2 = __shfl_xor_sync(0xFFFFFFFFu, l[g], 16);
        const float mx = fmaxf(m[g], m2);
        const float c1 = m[g] == -INFINITY ? 0.0f : expf(m[g] - mx);
        const float c2 = m2 == -INFINITY ? 0.0f : expf(m2 - mx);
        l[g] = l[g] * c1 + l2 * c2;
#pragma unroll
        for (int i = 0; i < 8; ++i)
        {
            const float a2 = __shfl_xor_sync(0xFFFFFFFFu, acc[g][i], 16);
            acc[g][i] = acc[g][i] * c1 + a2 * c2;
        }
        m[g] = mx;
        if (hw == 0)
        {
#pragma unroll
            for (int i = 0; i < 8; ++i) acc_s[warp][g][d0 + i] = acc[g][i];
            if (hl == 0)
            {
                m_s[warp][g] = m[g];
                l_s[warp][g] = l[g];
            }
        }
    }
    __syncthreads();
    // the CTA's (max, sum, unnormalised output) per query head and dimension; one slice: the result
    constexpr int PS = D + 2;   // a partial: max, sum, then D outputs
    for (int t = threadIdx.x; t < G * D; t += blockDim.x)
    {
        const int g = t / D, d = t % D;
        float mx = -INFINITY;
        for (int w = 0; w < WARPS; ++w) mx = fmaxf(mx, m_s[w][g]);
        float ls = 0.0f, o = 0.0f;
        for (int w = 0; w < WARPS; ++w)
        {
            const float c = m_s[w][g] == -INFINITY ? 0.0f : expf(m_s[w][g] - mx);
            ls += l_s[w][g] * c;
            o += acc_s[w][g][d] * c;
        }
        if (active == 1)
        {
            out[static_cast<int64_t>(kvh * G + g) * D + d] = from_f32<T>(o / ls);
        }
        else
        {
            float* pr = part + ((static_cast<int64_t>(kvh) * gridDim.y + split) * G + g) * PS;
            pr[2 + d] = o;
            if (d == 0)
            {
                pr[0] = mx;
                pr[1] = ls;
            }
        }
    }
    if (active == 1) return;
    // The last slice of this KV head to finish merges them all (no CTA waits on another): each
    // CTA's partials are made visible device-wide before its arrival is counted.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last_s = atomicAdd(&counters[kvh], 1u) == static_cast<unsigned>(active - 1);
    __syncthreads();
    if (!last_s) return;
    __threadfence();
    for (int t = threadIdx.x; t < G * D; t += blockDim.x)
    {
        const int g = t / D, d = t % D;
        const float* pr = part + (static_cast<int64_t>(kvh) * gridDim.y * G + g) * PS;
        const int64_t stride = static_cast<int64_t>(G) * PS;   // from one slice to the next
        float mx = -INFINITY;
        for (int sp = 0; sp < active; ++sp) mx = fmaxf(mx, __ldcg(pr + sp * stride));
        float ls = 0.0f, o = 0.0f;
        for (int sp = 0; sp < active; ++sp)
        {
            const float c = expf(__ldcg(pr + sp * stride) - mx);   // every slice has >= 1 position
            ls += __ldcg(pr + sp * stride + 1) * c;
            o += __ldcg(pr + sp * stride + 2 + d) * c;
        }
        out[static_cast<int64_t>(kvh * G + g) * D + d] = from_f32<T>(o / ls);
    }
    if (threadIdx.x == 0) counters[kvh] = 0u;   // ready for the next call
}

template <typename T, int R>
void launch_gemv_pick(const void* x, const void* w, int64_t ldw, void* y, int64_t n, int64_t k, bool vec,
                      const GemvNorm& norm, const GemvPick& pick, cudaStream_t stream)
{
    const auto blocks = static_cast<unsigned>(gemv_grid(n, R));
    const size_t smem = static_cast<size_t>(k) * sizeof(T) * 2;   // the row and the gain
    const auto ni = static_cast<int>(n), ki = static_cast<int>(k);
#define VEDA_GEMV_PICK(V)                                                                               \
    gemv_kernel<T, R, false, V, true, true><<<blocks, kGemvWarps * 32, smem, stream>>>(                 \
        static_cast<const T*>(x), static_cast<const T*>(w), ldw, static_cast<T*>(y), ni, ki,            \
        static_cast<const T*>(norm.r), static_cast<const T*>(norm.gamma), static_cast<T*>(norm.sum),    \
        norm.eps, pick)
    if (vec) VEDA_GEMV_PICK(true);
    else VEDA_GEMV_PICK(false);
#undef VEDA_GEMV_PICK
}

int64_t pick_blocks(int64_t n) { return gemv_grid(n, n >= 8192 ? 2 : 1); }

int gemv_checks(const void* x, const void* w, int64_t ldw, const void* y, int64_t n, int64_t k, int dtype)
{
    VEDA_REQUIRE(valid_dtype(dtype), "unknown dtype");
    VEDA_REQUIRE(x && w && y, "null pointer");
    VEDA_REQUIRE(n > 0 && k > 0 && n < (1ll << 30), "bad shape");
    VEDA_REQUIRE(ldw >= k, "bad weight leading dimension");
    VEDA_REQUIRE(k * static_cast<int64_t>(dtype_size(dtype)) <= kGemvSmem,
                 "the activation row exceeds the 47 KB staged in shared memory");
    return 0;
}

bool gemv_vec(const void* x, const void* w, int64_t ldw, int64_t k, int dtype)
{
    const int64_t e = 16 / static_cast<int64_t>(dtype_size(dtype));
    return (x == nullptr || aligned16(x)) && aligned16(w) && k % e == 0 && ldw % e == 0;
}

int gemv_dispatch(const void* x, const void* w, int64_t ldw, void* y, int64_t n, int64_t k, int dtype,
                  bool swiglu, const GemvNorm* norm, cudaStream_t stream)
{
    const bool vec = gemv_vec(norm ? nullptr : x, w, ldw, k, dtype);
    // two rows a warp once there are enough rows to fill the SMs with them
    const bool two = n >= 8192;
    if (dtype == VEDA_BF16)
    {
        if (swiglu) launch_gemv<bf16, 2, true>(x, w, ldw, y, n, k, vec, norm, stream);
        else if (two) launch_gemv<bf16, 2, false>(x, w, ldw, y, n, k, vec, norm, stream);
        else launch_gemv<bf16, 1, false>(x, w, ldw, y, n, k, vec, norm, stream);
    }
    else
    {
        if (swiglu) launch_gemv<float, 2, true>(x, w, ldw, y, n, k, vec, norm, stream);
        else if (two) launch_gemv<float, 2, false>(x, w, ldw, y, n, k, vec, norm, stream);
        else launch_gemv<float, 1, false>(x, w, ldw, y, n, k, vec, norm, stream);
    }
    count_launch();
    return 0;
}

int norm_checks(const void* x, const void* r, const void* gamma, const void* sum, int64_t k, int dtype)
{
    VEDA_REQUIRE(gamma != nullptr, "null pointer");
    VEDA_REQUIRE(2 * k * static_cast<int64_t>(dtype_size(dtype)) <= kGemvSmem,
                 "the activation row and its gain exceed the 47 KB staged in shared memory");
    VEDA_REQUIRE(sum == nullptr || (sum != x && sum != r), "sum must not alias x or r (block 0 writes it "
                                                          "while the others read them)");
    return 0;
}
} // namespace
} // namespace veda::cuda

extern "C" int veda_gemv_nt(const void* x, const void* w, int64_t ldw, void* y, int64_t n, int64_t k,
                            int dtype, veda_stream_t stream)
{
    if (const int rc = gemv_checks(x, w, ldw, y, n, k, dtype)) return rc;
    gemv_dispatch(x, w, ldw, y, n, k, dtype, false, nullptr, stream);
    return check_launch("veda_gemv_nt");
}

extern "C" int veda_gemv_swiglu(const void* x, const void* w_gate_up, int64_t ldw, void* h, int64_t f,
                                int64_t k, int dtype, veda_stream_t stream)
{
    if (const int rc = gemv_checks(x, w_gate_up, ldw, h, f, k, dtype)) return rc;
    gemv_dispatch(x, w_gate_up, ldw, h, f, k, dtype, true, nullptr, stream);
    return check_launch("veda_gemv_swiglu");
}

extern "C" int veda_gemv_rmsnorm(const void* x, const void* r, const void* gamma, float eps, void* sum,
                                 const void* w, int64_t ldw, void* y, int64_t n, int64_t k, int dtype,
                                 veda_stream_t stream)
{
    if (const int rc = gemv_checks(x, w, ldw, y, n, k, dtype)) return rc;
    if (const int rc = norm_checks(x, r, gamma, sum, k, dtype)) return rc;
    const GemvNorm norm{r, gamma, sum, eps};
    gemv_dispatch(x, w, ldw, y, n, k, dtype, false, &norm, stream);
    return check_launch("veda_gemv_rmsnorm");
}

extern "C" int veda_gemv_rmsnorm_swiglu(const void* x, const void* r, const void* gamma, float eps, void* sum,
                                        const void* w_gate_up, int64_t ldw, void* h, int64_t f, int64_t k,
                                        int dtype, veda_stream_t stream)
{
    if (const int rc = gemv_checks(x, w_gate_up, ldw, h, f, k, dtype)) return rc;
    if (const int rc = norm_checks(x, r, gamma, sum, k, dtype)) return rc;
    const GemvNorm norm{r, gamma, sum, eps};
    gemv_dispatch(x, w_gate_up, ldw, h, f, k, dtype, true, &norm, stream);
    return check_launch("veda_gemv_rmsnorm_swiglu");
}

namespace
{
// Positions per CTA slice for a cache of `capacity` rows: the whole cache up to 256 rows (two
// rounds of loads for 16 warps cost less than merging slices), else 128 (one round), or more so
// that at most 64 slices cover it.
int64_t decode_chunk(int64_t capacity)
{
    if (capacity <= 256) return 256;
    const int64_t c = (capacity + 63) / 64;
    return std::max<int64_t>(128, (c + 63) / 64 * 64);
}

int64_t decode_workspace(int64_t heads, int64_t kv_heads, int64_t capacity)
{
    const int64_t splits = (capacity + decode_chunk(capacity) - 1) / decode_chunk(capacity);
    const int64_t counters = (kv_heads * 4 + 255) / 256 * 256;
    return counters + kv_heads * splits * (heads / kv_heads) * (kFusedDim + 2) * 4;
}
} // namespace

extern "C" int64_t veda_decode_attention_workspace(int64_t heads, int64_t kv_heads, int64_t capacity)
{
    if (heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0 || capacity <= 0) return -1;
    return decode_workspace(heads, kv_heads, capacity);
}

extern "C" int veda_decode_attention_at(const void* qkv, const void* q_gain, const void* k_gain,
                                        const float* cos, const float* sin, const int64_t* pos, void* k_cache,
                                        void* v_cache, int64_t ldkv, int64_t capacity, int64_t heads,
                                        int64_t kv_heads, int64_t head_dim, float eps, float scale, void* out,
                                        void* workspace, int64_t workspace_bytes, int dtype, veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype), "unknown dtype");
    VEDA_REQUIRE(qkv && q_gain && k_gain && cos && sin && pos && k_cache && v_cache && out && workspace,
                 "null pointer");
    VEDA_REQUIRE(heads > 0 && kv_heads > 0 && heads % kv_heads == 0 && heads < (1 << 20), "bad shape");
    VEDA_REQUIRE(capacity > 0 && capacity < (1ll << 40), "bad cache capacity");
    VEDA_REQUIRE(ldkv >= kv_heads * head_dim, "bad cache leading dimension");
    const int64_t g = heads / kv_heads;
    if (head_dim != kFusedDim || !(g == 1 || g == 2 || g == 4 || g == 8) || ldkv % 8 != 0 ||
        !aligned16(k_cache) || !aligned16(v_cache))
    {
        return fail(VEDA_ERR_UNSUPPORTED, "veda_decode_attention_at: head_dim 128, 1/2/4/8 query heads per "
                                          "KV head and 16-byte aligned cache rows");
    }
    VEDA_REQUIRE(aligned16(workspace) && workspace_bytes >= decode_workspace(heads, kv_heads, capacity),
                 "workspace smaller than veda_decode_attention_workspace or not 16-byte aligned");
    const int64_t chunk = decode_chunk(capacity);
    const dim3 grid(static_cast<unsigned>(kv_heads), static_cast<unsigned>((capacity + chunk - 1) / chunk));
    auto* counters = static_cast<unsigned*>(workspace);
    auto* part = reinterpret_cast<float*>(static_cast<char*>(workspace) + (kv_heads * 4 + 255) / 256 * 256);
#define VEDA_FUSED(T, G, WARPS, U)                                                                        \
    decode_attn_fused_kernel<T, G, WARPS, U><<<grid, WARPS * 32, 0, stream>>>(                            \
        static_cast<const T*>(qkv), static_cast<const T*>(q_gain), static_cast<const T*>(k_gain), cos, sin, \
        pos, static_cast<T*>(k_cache), static_cast<T*>(v_cache), ldkv, static_cast<int>(kv_heads), eps,   \
        scale, static_cast<T*>(out), capacity, chunk, part, counters)
#define VEDA_FUSED_G(T)                                                                                   \
    switch (g)                                                                                             \
    {                                                                                                      \
    case 1: VEDA_FUSED(T, 1, 16, 4); break;                                                                \
    case 2: VEDA_FUSED(T, 2, 16, 4); break;                                                                \
    case 4: VEDA_FUSED(T, 4, 8, 4); break;                                                                 \
    default: VEDA_FUSED(T, 8, 8, 2); break;                                                                \
    }
    if (dtype == VEDA_BF16)
    {
        VEDA_FUSED_G(bf16)
    }
    else
    {
        VEDA_FUSED_G(float)
    }
#undef VEDA_FUSED_G
#undef VEDA_FUSED
    count_launch();
    return check_launch("veda_decode_attention_at");
}

extern "C" int64_t veda_gemv_argmax_workspace(int64_t n)
{
    if (n <= 0 || n >= (1ll << 30)) return -1;
    return 256 + pick_blocks(n) * 8;
}

extern "C" int veda_gemv_rmsnorm_argmax(const void* x, const void* r, const void* gamma, float eps, void* sum,
                                        const void* w, int64_t ldw, void* y, int64_t n, int64_t k,
                                        int64_t* token, int* status, void* workspace, int64_t workspace_bytes,
                                        int dtype, veda_stream_t stream)
{
    if (const int rc = gemv_checks(x, w, ldw, y, n, k, dtype)) return rc;
    if (const int rc = norm_checks(x, r, gamma, sum, k, dtype)) return rc;
    VEDA_REQUIRE(token != nullptr && workspace != nullptr, "null pointer");
    VEDA_REQUIRE(aligned16(workspace) && workspace_bytes >= 256 + pick_blocks(n) * 8,
                 "workspace smaller than veda_gemv_argmax_workspace or not 16-byte aligned");
    const GemvNorm norm{r, gamma, sum, eps};
    GemvPick pick;
    pick.token = token;
    pick.status = status;
    pick.counter = static_cast<unsigned*>(workspace);
    pick.val = reinterpret_cast<float*>(static_cast<char*>(workspace) + 256);
    pick.idx = reinterpret_cast<int*>(static_cast<char*>(workspace) + 256 + pick_blocks(n) * 4);
    const bool vec = gemv_vec(nullptr, w, ldw, k, dtype);
    if (dtype == VEDA_BF16)
    {
        if (n >= 8192) launch_gemv_pick<bf16, 2>(x, w, ldw, y, n, k, vec, norm, pick, stream);
        else launch_gemv_pick<bf16, 1>(x, w, ldw, y, n, k, vec, norm, pick, stream);
    }
    else
    {
        if (n >= 8192) launch_gemv_pick<float, 2>(x, w, ldw, y, n, k, vec, norm, pick, stream);
        else launch_gemv_pick<float, 1>(x, w, ldw, y, n, k, vec, norm, pick, stream);
    }
    count_launch();
    return check_launch("veda_gemv_rmsnorm_argmax");
}
