// CUDA-core GEMM: the fp32 path (exact arithmetic of the reference's matmul loop) and the
// fallback for bf16 shapes the tensor-core kernel's TMA descriptors cannot describe.
// 64x64 output tile per 256-thread CTA, 4x4 outputs per thread, K staged 16 at a time.
#include "gemm.cuh"

namespace veda::cuda
{
namespace
{

constexpr int TM = 64, TN = 64, TK = 16;

template <typename TA, typename TC, int OP>
__global__ void __launch_bounds__(256)
simt_gemm_kernel(const TA* __restrict__ A, int64_t lda, int64_t sa, const TA* __restrict__ B,
                 int64_t ldb, int64_t sb, TC* __restrict__ C, int64_t ldc, int64_t sc, int M,
                 int N, int K, float alpha, float beta)
{
    __shared__ float as[TK][TM + 1];
    __shared__ float bs[TK][TN + 1];
    const int64_t z = blockIdx.z;
    A += z * sa;
    B += z * sb;
    C += z * sc;
    const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

    for (int k0 = 0; k0 < K; k0 += TK)
    {
        for (int e = threadIdx.x; e < TM * TK; e += 256)
        {
            int m, k;
            if (OP == kTN)
            {
                k = e / TM;
                m = e % TM;   // A[k, m]: m contiguous
            }
            else
            {
                m = e / TK;
                k = e % TK;   // A[m, k]: k contiguous
            }
            const int gm = m0 + m, gk = k0 + k;
            float v = 0.0f;
            if (gm < M && gk < K)
            {
                v = to_f32(OP == kTN ? A[static_cast<int64_t>(gk) * lda + gm]
                                     : A[static_cast<int64_t>(gm) * lda + gk]);
            }
            as[k][m] = v;
        }
        for (int e = threadIdx.x; e < TN * TK; e += 256)
        {
            int n, k;
            if (OP == kNT)
            {
                n = e / TK;
                k = e % TK;   // B[n, k]
            }
            else
            {
                k = e / TN;
                n = e % TN;   // B[k, n]
            }
            const int gn = n0 + n, gk = k0 + k;
            float v = 0.0f;
            if (gn < N && gk < K)
            {
                v = to_f32(OP == kNT ? B[static_cast<int64_t>(gn) * ldb + gk]
                                     : B[static_cast<int64_t>(gk) * ldb + gn]);
            }
            bs[k][n] = v;
        }
        __syncthreads();
        const int kmax = K - k0 < TK ? K - k0 : TK;
        for (int k = 0; k < kmax; ++k)
        {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
            {
                a[i] = as[k][ty + 16 * i];
                b[i] = bs[k][tx + 16 * i];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], b[j]));
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        const int gm = m0 + ty + 16 * i;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j)
        {
            const int gn = n0 + tx + 16 * j;
            if (gn >= N) continue;
            TC* c = C + static_cast<int64_t>(gm) * ldc + gn;
            float v = alpha == 1.0f ? acc[i][j] : alpha * acc[i][j];
            if (beta != 0.0f)
            {
                v = beta == 1.0f ? to_f32(*c) + v : beta * to_f32(*c) + v;
            }
            *c = from_f32<TC>(v);
        }
    }
}

template <typename TA, typename TC>
int launch(int op, int64_t batch, int64_t M, int64_t N, int64_t K, const void* A, int64_t lda,
           int64_t sa, const void* B, int64_t ldb, int64_t sb, void* C, int64_t ldc, int64_t sc,
           float alpha, float beta, cudaStream_t s)
{
    const dim3 grid(static_cast<unsigned>((N + TN - 1) / TN), static_cast<unsigned>((M + TM - 1) / TM),
                    static_cast<unsigned>(batch));
    const TA* a = static_cast<const TA*>(A);
    const TA* b = static_cast<const TA*>(B);
    TC* c = static_cast<TC*>(C);
    const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
    if (op == kNT)
        simt_gemm_kernel<TA, TC, kNT><<<grid, 256, 0, s>>>(a, lda, sa, b, ldb, sb, c, ldc, sc, m, n, k, alpha, beta);
    else if (op == kNN)
        simt_gemm_kernel<TA, TC, kNN><<<grid, 256, 0, s>>>(a, lda, sa, b, ldb, sb, c, ldc, sc, m, n, k, alpha, beta);
    else
        simt_gemm_kernel<TA, TC, kTN><<<grid, 256, 0, s>>>(a, lda, sa, b, ldb, sb, c, ldc, sc, m, n, k, alpha, beta);
    count_launch();
    return check_launch("simt_gemm");
}

} // namespace

int simt_gemm(int op, int64_t batch, int64_t M, int64_t N, int64_t K, const void* A, int64_t lda,
              int64_t sa, const void* B, int64_t ldb, int64_t sb, void* C, int64_t ldc,
              int64_t sc, int dtype_ab, int dtype_c, float alpha, float beta, cudaStream_t s)
{
    if (M > (1ll << 30) || N > (1ll << 30) || K > (1ll << 30) || batch > 65535)
    {
        return fail(VEDA_ERR_UNSUPPORTED, "simt_gemm: extent too large");
    }
    if (dtype_ab == VEDA_F32)
    {
        return dtype_c == VEDA_F32
                   ? launch<float, float>(op, batch, M, N, K, A, lda, sa, B, ldb, sb, C, ldc, sc, alpha, beta, s)
                   : launch<float, bf16>(op, batch, M, N, K, A, lda, sa, B, ldb, sb, C, ldc, sc, alpha, beta, s);
    }
    return dtype_c == VEDA_F32
               ? launch<bf16, float>(op, batch, M, N, K, A, lda, sa, B, ldb, sb, C, ldc, sc, alpha, beta, s)
               : launch<bf16, bf16>(op, batch, M, N, K, A, lda, sa, B, ldb, sb, C, ldc, sc, alpha, beta, s);
}

} // namespace veda::cuda
