// Causal GQA attention forward and backward: C ABI front end and the warp-per-row kernels.
//
// Semantics are those of the composition in src/libs/train/Model.cpp:182-189 — scores =
// (q k^T) * scale, causal mask, softmax over keys, context = P v — with the KV head of query head
// h being h / (H / Hkv) (src/libs/model/Attention.cpp:191). The backward recomputes P from the
// saved log-sum-exp and forms dS = P * (dP - D), D = rowsum(dO * O), which equals the reference's
// softmax backward y * (G - sum G y) (src/libs/autograd/NonLinear.cpp:123-133) because
// sum_j dP_ij P_ij = dO_i . O_i.
//
// Two implementations sit behind the entry points:
//   * attention_tc.cu — bf16, head_dim 128: tcgen05 / TMEM kernels (forward; fused backward, or
//     the bit-reproducible two-kernel backward under veda_attention_set_deterministic(1));
//   * this file — any dtype and head_dim <= 256: one warp per query (forward, dQ) or per key
//     (dK, dV), fp32 accumulation, keys visited in ascending order. It is the fp32 path used for
//     fp32 parity and serves bf16 shapes the tensor maps cannot describe (sequence lengths that
//     are not a multiple of 8, operands not 16-byte aligned).
#include "attention.cuh"

#include <algorithm>

namespace veda::cuda
{
namespace
{

constexpr int kMaxPerLane = 8;   // head_dim <= 256

struct AttnShape
{
    int64_t B, T, H, Hkv, Dh;
    int64_t ldq, ldk, ldv, ldo;
    float scale;
    int causal;
};

template <typename T>
__device__ __forceinline__ void load_row(const T* p, int dh, float (&r)[kMaxPerLane])
{
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int e = 0; e < kMaxPerLane; ++e)
    {
        const int d = lane + 32 * e;
        r[e] = d < dh ? to_f32(p[d]) : 0.0f;
    }
}

__device__ __forceinline__ float dot_row(const float (&a)[kMaxPerLane], const float (&b)[kMaxPerLane])
{
    float s = 0.0f;
#pragma unroll
    for (int e = 0; e < kMaxPerLane; ++e)
    {
        s += a[e] * b[e];
    }
    return warp_sum(s);
}

// One warp per (b, h, i): online softmax over keys 0..i (or all keys without the mask).
template <typename T>
__global__ void simple_fwd_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                  const T* __restrict__ v, T* __restrict__ o, float* __restrict__ lse,
                                  AttnShape s)
{
    const int lane = threadIdx.x & 31;
    const int64_t rows = s.B * s.H * s.T;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int dh = static_cast<int>(s.Dh);
    const int64_t rep = s.H / s.Hkv;
    for (int64_t r = warp; r < rows; r += warps)
    {
        const int64_t i = r % s.T;
        const int64_t h = (r / s.T) % s.H;
        const int64_t b = r / (s.T * s.H);
        const int64_t kvh = h / rep;
        float qr[kMaxPerLane], acc[kMaxPerLane];
        load_row(q + (b * s.T + i) * s.ldq + h * s.Dh, dh, qr);
#pragma unroll
        for (int e = 0; e < kMaxPerLane; ++e) acc[e] = 0.0f;
        float m = -INFINITY, l = 0.0f;
        const int64_t last = s.causal ? i : s.T - 1;
        for (int64_t j = 0; j <= last; ++j)
        {
            float kr[kMaxPerLane], vr[kMaxPerLane];
            load_row(k + (b * s.T + j) * s.ldk + kvh * s.Dh, dh, kr);
            const float sc = dot_row(qr, kr) * s.scale;
            load_row(v + (b * s.T + j) * s.ldv + kvh * s.Dh, dh, vr);
            if (sc > m)
            {
                const float corr = m == -INFINITY ? 0.0f : expf(m - sc);
                l = l * corr + 1.0f;
#pragma unroll
                for (int e = 0; e < kMaxPerLane; ++e) acc[e] = acc[e] * corr + vr[e];
                m = sc;
            }
            else
            {
                const float p = expf(sc - m);
                l += p;
#pragma unroll
                for (int e = 0; e < kMaxPerLane; ++e) acc[e] += p * vr[e];
            }
        }
        T* orow = o + (b * s.T + i) * s.ldo + h * s.Dh;
#pragma unroll
        for (int e = 0; e < kMaxPerLane; ++e)
        {
            const int d = lane + 32 * e;
            if (d < dh) orow[d] = from_f32<T>(acc[e] / l);
        }
        if (lane == 0) lse[(b * s.H + h) * s.T + i] = m + logf(l);
    }
}

// D[b,h,i] = sum_d dO * O
template <typename T>
__global__ void rowdot_kernel(const T* __restrict__ o, int64_t ldo, const T* __restrict__ dout,
                              int64_t lddo, float* __restrict__ dvec, AttnShape s)
{
    const int64_t rows = s.B * s.H * s.T;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    for (int64_t r = warp; r < rows; r += warps)
    {
        const int64_t i = r % s.T;
        const int64_t h = (r / s.T) % s.H;
        const int64_t b = r / (s.T * s.H);
        float a[kMaxPerLane], g[kMaxPerLane];
        load_row(o + (b * s.T + i) * ldo + h * s.Dh, static_cast<int>(s.Dh), a);
        load_row(dout + (b * s.T + i) * lddo + h * s.Dh, static_cast<int>(s.Dh), g);
        const float d = dot_row(a, g);
        if ((threadIdx.x & 31) == 0) dvec[(b * s.H + h) * s.T + i] = d;
    }
}

// One warp per (b, h, i): dQ_i = scale * sum_j P_ij (dP_ij - D_i) k_j.
template <typename T>
__global__ void simple_dq_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                 const T* __restrict__ v, const T* __restrict__ dout, int64_t lddo,
                                 const float* __restrict__ lse, const float* __restrict__ dvec,
                                 T* __restrict__ dq, int64_t lddq, AttnShape s)
{
    const int lane = threadIdx.x & 31;
    const int64_t rows = s.B * s.H * s.T;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int dh = static_cast<int>(s.Dh);
    const int64_t rep = s.H / s.Hkv;
    for (int64_t r = warp; r < rows; r += warps)
    {
        const int64_t i = r % s.T;
        const int64_t h = (r / s.T) % s.H;
        const int64_t b = r / (s.T * s.H);
        const int64_t kvh = h / rep;
        float qr[kMaxPerLane], gr[kMaxPerLane], acc[kMaxPerLane];
        load_row(q + (b * s.T + i) * s.ldq + h * s.Dh, dh, qr);
        load_row(dout + (b * s.T + i) * lddo + h * s.Dh, dh, gr);
#pragma unroll
        for (int e = 0; e < kMaxPerLane; ++e) acc[e] = 0.0f;
        const float L = lse[(b * s.H + h) * s.T + i];
        const float D = dvec[(b * s.H + h) * s.T + i];
        const int64_t last = s.causal ? i : s.T - 1;
        for (int64_t j = 0; j <= last; ++j)
        {
            float kr[kMaxPerLane], vr[kMaxPerLane];
            load_row(k + (b * s.T + j) * s.ldk + kvh * s.Dh, dh, kr);
            load_row(v + (b * s.T + j) * s.ldv + kvh * s.Dh, dh, vr);
            const float p = expf(dot_row(qr, kr) * s.scale - L);
            const float ds = p * (dot_row(gr, vr) - D);
#pragma unroll
            for (int e = 0; e < kMaxPerLane; ++e) acc[e] += ds * kr[e];
        }
        T* out = dq + (b * s.T + i) * lddq + h * s.Dh;
#pragma unroll
        for (int e = 0; e < kMaxPerLane; ++e)
        {
            const int d = lane + 32 * e;
            if (d < dh) out[d] = from_f32<T>(acc[e] * s.scale);
        }
    }
}

// One warp per (b, kv head, j): dK_j, dV_j summed over the group's query heads and queries i >= j.
template <typename T>
__global__ void simple_dkv_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                  const T* __restrict__ v, const T* __restrict__ dout, int64_t lddo,
                                  const float* __restrict__ lse, const float* __restrict__ dvec,
                                  T* __restrict__ dk, int64_t lddk, T* __restrict__ dv,
                                  int64_t lddv, AttnShape s)
{
    const int lane = threadIdx.x & 31;
    const int64_t rows = s.B * s.Hkv * s.T;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int dh = static_cast<int>(s.Dh);
    const int64_t rep = s.H / s.Hkv;
    for (int64_t r = warp; r < rows; r += warps)
    {
        const int64_t j = r % s.T;
        const int64_t kvh = (r / s.T) % s.Hkv;
        const int64_t b = r / (s.T * s.Hkv);
        float kr[kMaxPerLane], vr[kMaxPerLane], ak[kMaxPerLane], av[kMaxPerLane];
        load_row(k + (b * s.T + j) * s.ldk + kvh * s.Dh, dh, kr);
        load_row(v + (b * s.T + j) * s.ldv + kvh * s.Dh, dh, vr);
#pragma unroll
        for (int e = 0; e < kMaxPerLane; ++e) ak[e] = av[e] = 0.0f;
        for (int64_t h = kvh * rep; h < (kvh + 1) * rep; ++h)
        {
            for (int64_t i = s.causal ? j : 0; i < s.T; ++i)
            {
                float qr[kMaxPerLane], gr[kMaxPerLane];
                load_row(q + (b * s.T + i) * s.ldq + h * s.Dh, dh, qr);
                load_row(dout + (b * s.T + i) * lddo + h * s.Dh, dh, gr);
                const float L = lse[(b * s.H + h) * s.T + i];
                const float D = dvec[(b * s.H + h) * s.T + i];
                const float p = expf(dot_row(qr, kr) * s.scale - L);
                const float ds = p * (dot_row(gr, vr) - D);
#pragma unroll
                for (int e = 0; e < kMaxPerLane; ++e)
                {
                    av[e] += p * gr[e];
                    ak[e] += ds * qr[e];
                }
            }
        }
        T* ko = dk + (b * s.T + j) * lddk + kvh * s.Dh;
        T* vo = dv + (b * s.T + j) * lddv + kvh * s.Dh;
#pragma unroll
        for (int e = 0; e < kMaxPerLane; ++e)
        {
            const int d = lane + 32 * e;
            if (d < dh)
            {
                ko[d] = from_f32<T>(ak[e] * s.scale);
                vo[d] = from_f32<T>(av[e]);
            }
        }
    }
}

int checks(int64_t B, int64_t T, int64_t H, int64_t Hkv, int64_t Dh, int64_t ldq, int64_t ldk,
           int64_t ldv, int64_t ldo, int dtype)
{
    VEDA_REQUIRE(valid_dtype(dtype), "unknown dtype");
    VEDA_REQUIRE(B >= 0 && T >= 0 && H > 0 && Hkv > 0 && Dh > 0, "bad shape");
    VEDA_REQUIRE(H % Hkv == 0, "heads must be a multiple of kv_heads");
    VEDA_REQUIRE(Dh <= 32 * kMaxPerLane, "head_dim above 256");
    VEDA_REQUIRE(ldq >= H * Dh && ldo >= H * Dh && ldk >= Hkv * Dh && ldv >= Hkv * Dh,
                 "leading dimension smaller than heads * head_dim");
    return VEDA_OK;
}

} // namespace
} // namespace veda::cuda

using namespace veda::cuda;

extern "C" size_t veda_attention_bwd_workspace(int64_t batch, int64_t seq_len, int64_t heads,
                                               int64_t kv_heads, int64_t head_dim, int dtype)
{
    // D = rowsum(dO * O) [B, H, T] fp32, plus what the tensor-core backward keeps between its
    // launches: the fused path's fp32 dQ accumulator, or the deterministic path's dS^T.
    (void)kv_heads;
    size_t bytes = (static_cast<size_t>(batch * heads * seq_len) * sizeof(float) + 255) &
                   ~static_cast<size_t>(255);
    if (tc_supported(head_dim, dtype))
    {
        bytes += tc_bwd_extra_workspace(batch, seq_len, heads);
    }
    return (bytes + 255) & ~static_cast<size_t>(255);
}

extern "C" int veda_attention_fwd(const void* q, int64_t ldq, const void* k, int64_t ldk,
                                  const void* v, int64_t ldv, void* o, int64_t ldo, float* lse,
                                  int64_t batch, int64_t seq_len, int64_t heads, int64_t kv_heads,
                                  int64_t head_dim, float scale, int causal, int dtype,
                                  veda_stream_t stream)
{
    int rc = checks(batch, seq_len, heads, kv_heads, head_dim, ldq, ldk, ldv, ldo, dtype);
    if (rc != VEDA_OK) return rc;
    if (batch == 0 || seq_len == 0) return VEDA_OK;
    VEDA_REQUIRE(q && k && v && o && lse, "null pointer");
    if (tc_supported(head_dim, dtype) && tc_aligned(q, ldq, k, ldk, v, ldv, o, ldo))
    {
        const int rc2 = attn_tc_fwd(q, ldq, k, ldk, v, ldv, o, ldo, lse, batch, seq_len, heads,
                                    kv_heads, scale, causal, stream);
        if (rc2 != -1)
        {
            return rc2;
        }
    }
    AttnShape s{batch, seq_len, heads, kv_heads, head_dim, ldq, ldk, ldv, ldo, scale, causal};
    const unsigned grid = grid_for(batch * heads * seq_len * 32, 256);
    if (dtype == VEDA_BF16)
        simple_fwd_kernel<bf16><<<grid, 256, 0, stream>>>(
            static_cast<const bf16*>(q), static_cast<const bf16*>(k), static_cast<const bf16*>(v),
            static_cast<bf16*>(o), lse, s);
    else
        simple_fwd_kernel<float><<<grid, 256, 0, stream>>>(
            static_cast<const float*>(q), static_cast<const float*>(k),
            static_cast<const float*>(v), static_cast<float*>(o), lse, s);
    count_launch();
    return check_launch("veda_attention_fwd");
}

extern "C" int veda_attention_bwd(const void* q, int64_t ldq, const void* k, int64_t ldk,
                                  const void* v, int64_t ldv, const void* o, int64_t ldo,
                                  const void* dout, int64_t lddo, const float* lse, void* dq,
                                  int64_t lddq, void* dk, int64_t lddk, void* dv, int64_t lddv,
                                  void* workspace, size_t workspace_bytes, int64_t batch,
                                  int64_t seq_len, int64_t heads, int64_t kv_heads,
                                  int64_t head_dim, float scale, int causal, int dtype,
                                  veda_stream_t stream)
{
    int rc = checks(batch, seq_len, heads, kv_heads, head_dim, ldq, ldk, ldv, ldo, dtype);
    if (rc != VEDA_OK) return rc;
    VEDA_REQUIRE(lddo >= heads * head_dim && lddq >= heads * head_dim &&
                     lddk >= kv_heads * head_dim && lddv >= kv_heads * head_dim,
                 "gradient leading dimension too small");
    if (batch == 0 || seq_len == 0) return VEDA_OK;
    VEDA_REQUIRE(q && k && v && o && dout && lse && dq && dk && dv, "null pointer");
    VEDA_REQUIRE(workspace != nullptr &&
                     workspace_bytes >= veda_attention_bwd_workspace(batch, seq_len, heads,
                                                                     kv_heads, head_dim, dtype),
                 "workspace too small (see veda_attention_bwd_workspace)");
    float* dvec = static_cast<float*>(workspace);
    if (tc_supported(head_dim, dtype) && tc_aligned(q, ldq, k, ldk, v, ldv, o, ldo) &&
        tc_aligned(dout, lddo, dq, lddq, dk, lddk, dv, lddv))
    {
        char* extra = static_cast<char*>(workspace) +
                      ((static_cast<size_t>(batch * heads * seq_len) * sizeof(float) + 255) & ~static_cast<size_t>(255));
        const int rc2 = attn_tc_bwd(q, ldq, k, ldk, v, ldv, o, ldo, dout, lddo, lse, dq, lddq, dk,
                                    lddk, dv, lddv, dvec, extra, batch, seq_len, heads, kv_heads,
                                    scale, causal, stream);
        if (rc2 != -1)
        {
            return rc2;
        }
    }
    AttnShape s{batch, seq_len, heads, kv_heads, head_dim, ldq, ldk, ldv, ldo, scale, causal};
    const unsigned gq = grid_for(batch * heads * seq_len * 32, 256);
    const unsigned gk = grid_for(batch * kv_heads * seq_len * 32, 256);
    if (dtype == VEDA_BF16)
    {
        rowdot_kernel<bf16><<<gq, 256, 0, stream>>>(static_cast<const bf16*>(o), ldo,
                                                    static_cast<const bf16*>(dout), lddo, dvec, s);
        simple_dq_kernel<bf16><<<gq, 256, 0, stream>>>(
            static_cast<const bf16*>(q), static_cast<const bf16*>(k), static_cast<const bf16*>(v),
            static_cast<const bf16*>(dout), lddo, lse, dvec, static_cast<bf16*>(dq), lddq, s);
        simple_dkv_kernel<bf16><<<gk, 256, 0, stream>>>(
            static_cast<const bf16*>(q), static_cast<const bf16*>(k), static_cast<const bf16*>(v),
            static_cast<const bf16*>(dout), lddo, lse, dvec, static_cast<bf16*>(dk), lddk,
            static_cast<bf16*>(dv), lddv, s);
    }
    else
    {
        rowdot_kernel<float><<<gq, 256, 0, stream>>>(static_cast<const float*>(o), ldo,
                                                     static_cast<const float*>(dout), lddo, dvec, s);
        simple_dq_kernel<float><<<gq, 256, 0, stream>>>(
            static_cast<const float*>(q), static_cast<const float*>(k),
            static_cast<const float*>(v), static_cast<const float*>(dout), lddo, lse, dvec,
            static_cast<float*>(dq), lddq, s);
        simple_dkv_kernel<float><<<gk, 256, 0, stream>>>(
            static_cast<const float*>(q), static_cast<const float*>(k),
            static_cast<const float*>(v), static_cast<const float*>(dout), lddo, lse, dvec,
            static_cast<float*>(dk), lddk, static_cast<float*>(dv), lddv, s);
    }
    count_launch(3);
    return check_launch("veda_attention_bwd");
}

extern "C" size_t veda_attention_bwd_dq_offset(int64_t batch, int64_t seq_len, int64_t heads)
{
    return (static_cast<size_t>(batch * heads * seq_len) * sizeof(float) + 255) &
           ~static_cast<size_t>(255);
}

extern "C" int veda_attention_bwd_dq_f32(const void* q, int64_t ldq, const void* k, int64_t ldk,
                                         const void* v, int64_t ldv, const void* o, int64_t ldo,
                                         const void* dout, int64_t lddo, const float* lse, void* dk,
                                         int64_t lddk, void* dv, int64_t lddv, void* workspace,
                                         size_t workspace_bytes, int64_t batch, int64_t seq_len,
                                         int64_t heads, int64_t kv_heads, int64_t head_dim,
                                         float scale, int causal, int dtype, veda_stream_t stream)
{
    int rc = checks(batch, seq_len, heads, kv_heads, head_dim, ldq, ldk, ldv, ldo, dtype);
    if (rc != VEDA_OK) return rc;
    VEDA_REQUIRE(lddo >= heads * head_dim && lddk >= kv_heads * head_dim &&
                     lddv >= kv_heads * head_dim,
                 "gradient leading dimension too small");
    if (batch == 0 || seq_len == 0) return VEDA_OK;
    VEDA_REQUIRE(q && k && v && o && dout && lse && dk && dv, "null pointer");
    VEDA_REQUIRE(workspace != nullptr &&
                     workspace_bytes >= veda_attention_bwd_workspace(batch, seq_len, heads,
                                                                     kv_heads, head_dim, dtype),
                 "workspace too small (see veda_attention_bwd_workspace)");
    if (!tc_supported(head_dim, dtype) || attention_deterministic() != 0 ||
        !tc_aligned(q, ldq, k, ldk, v, ldv, o, ldo) || !tc_aligned(dout, lddo, dk, lddk, dv, lddv, dk, lddk))
    {
        return fail(VEDA_ERR_UNSUPPORTED,
                    "veda_attention_bwd_dq_f32: only the fused tensor-core backward (bf16, head_dim "
                    "128, 16-byte aligned operands, not the deterministic mode) keeps dQ in fp32");
    }
    float* dvec = static_cast<float*>(workspace);
    char* extra = static_cast<char*>(workspace) + veda_attention_bwd_dq_offset(batch, seq_len, heads);
    const int rc2 = attn_tc_bwd(q, ldq, k, ldk, v, ldv, o, ldo, dout, lddo, lse, nullptr, 0, dk, lddk,
                                dv, lddv, dvec, extra, batch, seq_len, heads, kv_heads, scale,
                                causal, stream);
    if (rc2 == -1)
    {
        return fail(VEDA_ERR_UNSUPPORTED, "veda_attention_bwd_dq_f32: the shape needs the general kernels");
    }
    return rc2;
}

extern "C" int veda_attention_set_deterministic(int on)
{
    return veda::cuda::g_attn_deterministic.exchange(on ? 1 : 0);
}
