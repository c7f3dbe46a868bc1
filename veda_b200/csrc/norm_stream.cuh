// Internal interface of the streaming RMSNorm kernels (norm_stream.cu) used by norm.cu.
#pragma once

#include "common.cuh"

namespace veda::cuda
{

// bf16 RMSNorm forward for rows of n = 256, 512, 1024 or 2048 elements (16-byte aligned rows).
// With r non-null the rows normalised are x + r (rounded to bf16), which are also written to
// sum. Returns -1 without launching when the shape is not one of these (the caller uses another
// kernel).
int rms_fwd_stream(const bf16* x, int64_t ldx, const bf16* r, int64_t ldr, const bf16* gamma,
                   bf16* y, int64_t ldy, bf16* sum, int64_t lds, int64_t rows, int64_t n, float eps,
                   cudaStream_t s);

// bf16 RMSNorm backward for n = 256, 512 or 1024. `partials` (may be null) receives one n-float row of the
// gain gradient per block, for the caller to sum in block order; at most `max_blocks` blocks are
// used and the number used is returned in *blocks. Returns -1 without launching when not
// applicable.
int rms_bwd_stream(const bf16* x, int64_t ldx, const bf16* gamma, const bf16* dy, int64_t lddy,
                   const bf16* dresid, int64_t ldr, bf16* dx, int64_t lddx, float* partials,
                   int max_blocks, int64_t rows, int64_t n, float eps, cudaStream_t s, int* blocks);

} // namespace veda::cuda
