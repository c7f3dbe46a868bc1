// Internal interface between the attention front end (attention.cu) and the tcgen05 kernels
// (attention_tc.cu).
#pragma once

#include "common.cuh"

#include <atomic>

namespace veda::cuda
{

// The tensor-core kernels cover bf16 with head_dim 128.
inline bool tc_supported(int64_t head_dim, int dtype)
{
    return dtype == VEDA_BF16 && head_dim == 128;
}

inline bool tc_aligned(const void* a, int64_t lda, const void* b, int64_t ldb, const void* c,
                       int64_t ldc, const void* d, int64_t ldd)
{
    return aligned16(a) && aligned16(b) && aligned16(c) && aligned16(d) && lda % 8 == 0 &&
           ldb % 8 == 0 && ldc % 8 == 0 && ldd % 8 == 0;
}

// Workspace the tcgen05 backward needs after D: the fused path's fp32 dQ accumulator
// [B*T][H*128], or the deterministic path's dS^T [B*H][T][T] bf16; then -LSE log2(e).
size_t tc_bwd_extra_workspace(int64_t B, int64_t T, int64_t H);

// tcgen05 kernels (bf16, head_dim 128, 16-byte aligned operands); return -1 when a tensor map
// cannot be built for the shape (the caller then runs the generic kernels). attn_tc_bwd with
// dq == nullptr (fused kernel only, -1 in the deterministic mode) leaves dQ / scale in the fp32
// accumulator at the start of `extra` instead of rounding it into dq.
int attn_tc_fwd(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                void* o, int64_t ldo, float* lse, int64_t B, int64_t T, int64_t H, int64_t Hkv,
                float scale, int causal, cudaStream_t s);
int attn_tc_bwd(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                const void* o, int64_t ldo, const void* dout, int64_t lddo, const float* lse,
                void* dq, int64_t lddq, void* dk, int64_t lddk, void* dv, int64_t lddv, float* dvec,
                void* extra, int64_t B, int64_t T, int64_t H, int64_t Hkv, float scale, int causal,
                cudaStream_t s);

// 1: the backward uses the two-kernel path whose dQ is bit-reproducible (dS^T through HBM);
// 0 (the default): the fused kernel. Process-wide.
extern std::atomic<int> g_attn_deterministic;
int attention_deterministic();

} // namespace veda::cuda
