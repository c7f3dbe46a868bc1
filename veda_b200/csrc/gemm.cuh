// Internal interface between the GEMM front end (gemm_sm100.cu) and the CUDA-core GEMM.
#pragma once

#include "common.cuh"

namespace veda::cuda
{

enum GemmOp
{
    kNT = 0,   // A[M,K] B[N,K]
    kNN = 1,   // A[M,K] B[K,N]
    kTN = 2    // A[K,M] B[K,N]
};

// CUDA-core GEMM (any dtype, any alignment, batched with element strides). For fp32 operands the
// k loop runs in ascending order with separately rounded multiply and add, the arithmetic of
// ops::matmul's multiply_block (src/libs/ops/Matmul.cpp:47-74), so a 2-D fp32 product equals the
// CPU's bit for bit.
int simt_gemm(int op, int64_t batch, int64_t M, int64_t N, int64_t K, const void* A, int64_t lda,
              int64_t sa, const void* B, int64_t ldb, int64_t sb, void* C, int64_t ldc,
              int64_t sc, int dtype_ab, int dtype_c, float alpha, float beta, cudaStream_t s);

} // namespace veda::cuda
