// Internal interface between the attention front end (attention.cu) and the tiled tensor-core
// kernels (attention_flash.cu).
#pragma once

#include "common.cuh"

namespace veda::cuda
{

// The tiled kernels cover bf16 with head_dim 128.
extern const bool kFlashReady;
inline bool flash_supported(int64_t head_dim, int dtype)
{
    return kFlashReady && dtype == VEDA_BF16 && head_dim == 128;
}

inline bool flash_aligned(const void* a, int64_t lda, const void* b, int64_t ldb, const void* c,
                          int64_t ldc, const void* d, int64_t ldd)
{
    return aligned16(a) && aligned16(b) && aligned16(c) && aligned16(d) && lda % 8 == 0 &&
           ldb % 8 == 0 && ldc % 8 == 0 && ldd % 8 == 0;
}

size_t flash_bwd_extra_workspace(int64_t B, int64_t T, int64_t H, int64_t Hkv, int64_t Dh);
// The tcgen05 backward keeps dS^T for every (batch, head) as bf16 [T x T] between its two kernels.
size_t tc_bwd_extra_workspace(int64_t B, int64_t T, int64_t H);

// tcgen05 kernels (attention_tc.cu): same contract as flash_fwd / flash_bwd (bf16, head_dim 128,
// 16-byte aligned operands); return -1 when a tensor map cannot be built (caller falls back).
int attn_tc_fwd(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                void* o, int64_t ldo, float* lse, int64_t B, int64_t T, int64_t H, int64_t Hkv,
                float scale, int causal, cudaStream_t s);
int attn_tc_bwd(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                const void* o, int64_t ldo, const void* dout, int64_t lddo, const float* lse,
                void* dq, int64_t lddq, void* dk, int64_t lddk, void* dv, int64_t lddv, float* dvec,
                void* extra, int64_t B, int64_t T, int64_t H, int64_t Hkv, float scale, int causal,
                cudaStream_t s);
// Which tiled implementation serves bf16 / head_dim 128: 1 tcgen05 (default), 0 mma.sync.
int attention_tc_enabled();

int flash_fwd(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
              void* o, int64_t ldo, float* lse, int64_t B, int64_t T, int64_t H, int64_t Hkv,
              float scale, int causal, cudaStream_t s);

int flash_bwd(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
              const void* o, int64_t ldo, const void* dout, int64_t lddo, const float* lse,
              void* dq, int64_t lddq, void* dk, int64_t lddk, void* dv, int64_t lddv, float* dvec,
              void* extra, int64_t B, int64_t T, int64_t H, int64_t Hkv, float scale, int causal,
              cudaStream_t s);

} // namespace veda::cuda
