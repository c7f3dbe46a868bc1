// bf16 GEMM on the 5th-generation tensor cores (tcgen05.mma, accumulators in TMEM), fed by TMA.
//
// The Linear/LM-head products of the training step: forward y = x W^T (NT), input gradient
// dX = dY W (NN) and weight gradient dW = dY^T X (TN) — ops::matmul / ops::matmul_nt as used by
// autograd::matmul_nt's forward and backward (src/libs/autograd/Variable.cpp:325-346). The
// reference runs a scalar fp32 i-j-k loop (src/libs/ops/Matmul.cpp:47-74); here operands are bf16,
// products accumulate in fp32 in TMEM, and the epilogue writes bf16 or fp32 (fp32 with beta = 1
// accumulates into a gradient, the leaf accumulation of Variable.cpp:27-38).
//
// Kernel structure (one CTA per SM, persistent over output tiles of 128 x BN):
//   warp 0     TMA producer: one thread streams 128x64 A and BNx64 B bf16 tiles into a
//              STAGES-deep ring of 128-byte-swizzled shared-memory buffers (no multicast);
//   warp 1     MMA issuer: allocates 2*BN TMEM columns (two accumulators), one thread issues
//              tcgen05.mma (M=128, N=BN, K=16) and signals stage release / tile completion with
//              tcgen05.commit onto mbarriers;
//   warps 2-5  epilogue: tcgen05.ld 32 lanes x 32 columns at a time, alpha/beta, convert, store;
//              the other accumulator is being filled meanwhile.
// Operand layouts: A and B are each either K-major (the reduction dim contiguous) or MN-major; the
// shared-memory descriptors and the instruction descriptor's major bits say which, so NT, NN and
// TN all run without a transpose pass. Split-K (fp32 output only) adds partial tiles with fp32
// vector atomics, so small weight-gradient GEMMs still fill all 148 SMs.
// Every mbarrier wait is bounded; a wait that gives up records VEDA_ERR_TIMEOUT in the library's
// device status word (veda_kernel_status) and the kernel runs to completion.
#include "gemm.cuh"
#include "swiglu_math.cuh"
#include "tc_common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

namespace veda::cuda
{
int* device_status_ptr();

namespace
{

constexpr int BM = 128;
constexpr int BK = 64;               // 64 bf16 = 128 bytes: one swizzle row
constexpr int kThreads = 192;        // 6 warps

template <int BN>
struct Cfg
{
    static constexpr int STAGES = BN == 256 ? 4 : 6;
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256 + 4 * 2 * 32 * 128;
};

struct Params
{
    int M, N, K;
    int num_m, num_n, kblocks, splits, kb_per_split;
    void* C;
    int64_t ldc;
    float alpha, beta;
    int out_f32;      // 1: fp32 C, 0: bf16 C
    int atomic;       // 1: split-K partial tiles are added with fp32 atomics
    int vec_ok;       // C base and ldc allow 16-byte stores
    int out_mode;     // 0: stores from registers; 1: TMA store; 2: TMA reduce-add (fp32 C)
    int* status;
    // SwiGLU epilogues of the paired kernel (EPI 1 and 2): the width F of gate and of up, which
    // sit side by side in one [M, 2F] buffer; EPI 2 reads them from gu
    int F;
    const bf16* gu;
    int64_t ldgu;
};

// Per-warp output staging: two 4 KB tiles of 32 rows x 128 bytes (128-byte swizzle), so the
// epilogue writes C with coalesced TMA stores instead of one 16-byte store per row and thread.
constexpr int kStageTile = 32 * 128;
constexpr int kOutStaging = 4 * 2 * kStageTile;   // 4 epilogue warps, double-buffered

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y)
{
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(tc::smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
}

// Element-wise atomic add of a shared tile onto global memory (fp32).
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* src, int x, int y)
{
    asm volatile(
        "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(tc::smem_u32(src)), "r"(x), "r"(y)
        : "memory");
}

using namespace tc;

// Output tile order: groups of 16 M-tiles sweep all N-tiles, so an A row-panel stays in L2.
__device__ __forceinline__ void unit_coords(int u, const Params& p, int& mb, int& nb, int& split)
{
    const int tiles = p.num_m * p.num_n;
    split = u / tiles;
    const int t = u - split * tiles;
    constexpr int G = 16;
    const int group = t / (G * p.num_n);
    const int first = group * G;
    const int gm = min(p.num_m - first, G);
    const int in = t - group * G * p.num_n;
    mb = first + in % gm;
    nb = in / gm;
}

template <int BN>
__device__ __forceinline__ void store_chunk(const Params& p, int row, int col0, const uint32_t (&r)[32])
{
    if (row >= p.M)
    {
        return;
    }
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j)
    {
        v[j] = __uint_as_float(r[j]);
        if (p.alpha != 1.0f)
        {
            v[j] *= p.alpha;
        }
    }
    const bool full = col0 + 32 <= p.N && p.vec_ok;
    if (p.out_f32)
    {
        float* c = static_cast<float*>(p.C) + static_cast<int64_t>(row) * p.ldc + col0;
        if (full)
        {
            if (p.atomic)
            {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                {
                    atomicAdd(reinterpret_cast<float4*>(c + j), make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
                }
                return;
            }
#pragma unroll
            for (int j = 0; j < 32; j += 4)
            {
                float4 o = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                if (p.beta != 0.0f)
                {
                    const float4 old = *reinterpret_cast<const float4*>(c + j);
                    o.x += p.beta * old.x;
                    o.y += p.beta * old.y;
                    o.z += p.beta * old.z;
                    o.w += p.beta * old.w;
                }
                *reinterpret_cast<float4*>(c + j) = o;
            }
            return;
        }
        for (int j = 0; j < 32; ++j)
        {
            if (col0 + j < p.N)
            {
                if (p.atomic)
                {
                    atomicAdd(c + j, v[j]);
                }
                else
                {
                    c[j] = p.beta != 0.0f ? v[j] + p.beta * c[j] : v[j];
                }
            }
        }
        return;
    }
    bf16* c = static_cast<bf16*>(p.C) + static_cast<int64_t>(row) * p.ldc + col0;
    if (full)
    {
#pragma unroll
        for (int j = 0; j < 32; j += 8)
        {
            float o[8];
#pragma unroll
            for (int q = 0; q < 8; ++q)
            {
                o[q] = v[j + q];
            }
            if (p.beta != 0.0f)
            {
                float old[8];
                load16(c + j, old);
#pragma unroll
                for (int q = 0; q < 8; ++q)
                {
                    o[q] += p.beta * old[q];
                }
            }
            store16(c + j, o);
        }
        return;
    }
    for (int j = 0; j < 32; ++j)
    {
        if (col0 + j < p.N)
        {
            const float o = p.beta != 0.0f ? v[j] + p.beta * __bfloat162float(c[j]) : v[j];
            c[j] = __float2bfloat16_rn(o);
        }
    }
}

// TMA epilogue of one warp: its 32 accumulator rows (TMEM lanes) x NCOLS columns, from TMEM
// through a swizzled staging tile to C (store, or fp32 reduce-add for split-K / beta = 1).
// `row0`, `col0`: C coordinates of the warp's first row and the tile's first column; `nstore`
// counts this warp's bulk groups (staging buffers alternate; one group may stay in flight).
template <int NCOLS>
__device__ __forceinline__ void epilogue_tma(const Params& p, const CUtensorMap* mc, uint32_t taddr,
                                             int row0, int col0, uint8_t* staging, uint32_t& nstore,
                                             int lane)
{
    if (row0 >= p.M)
    {
        return;
    }
    const int chunk = p.out_f32 ? 32 : 64;   // columns per 128-byte staging row
    for (int c = 0; c < NCOLS; c += chunk)
    {
        if (col0 + c >= p.N)
        {
            break;
        }
        uint8_t* buf = staging + (nstore & 1) * kStageTile;
        if (nstore >= 2)
        {
            if (lane == 0)
            {
                bulk_wait_group_read<1>();   // the group that last used `buf` has read it
            }
            __syncwarp();
        }
        uint32_t r0[32];
        tmem_ld32(taddr + static_cast<uint32_t>(c), r0);
        uint8_t* row = buf + lane * 128;
        if (p.out_f32)
        {
#pragma unroll
            for (int k = 0; k < 8; ++k)
            {
                float4 o = make_float4(__uint_as_float(r0[4 * k]), __uint_as_float(r0[4 * k + 1]),
                                       __uint_as_float(r0[4 * k + 2]), __uint_as_float(r0[4 * k + 3]));
                if (p.alpha != 1.0f)
                {
                    o.x *= p.alpha;
                    o.y *= p.alpha;
                    o.z *= p.alpha;
                    o.w *= p.alpha;
                }
                *reinterpret_cast<float4*>(row + ((k ^ (lane & 7)) << 4)) = o;
            }
        }
        else
        {
            uint32_t r1[32];
            tmem_ld32(taddr + static_cast<uint32_t>(c + 32), r1);
#pragma unroll
            for (int k = 0; k < 8; ++k)
            {
                const uint32_t* src = k < 4 ? &r0[8 * k] : &r1[8 * (k - 4)];
                uint32_t w[4];
#pragma unroll
                for (int q = 0; q < 4; ++q)
                {
                    float a = __uint_as_float(src[2 * q]), b = __uint_as_float(src[2 * q + 1]);
                    if (p.alpha != 1.0f)
                    {
                        a *= p.alpha;
                        b *= p.alpha;
                    }
                    const __nv_bfloat162 t = __floats2bfloat162_rn(a, b);
                    w[q] = *reinterpret_cast<const uint32_t*>(&t);
                }
                *reinterpret_cast<uint4*>(row + ((k ^ (lane & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
            }
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0)
        {
            if (p.out_mode == 2)
            {
                tma_reduce_add_2d(mc, buf, col0 + c, row0);
            }
            else
            {
                tma_store_2d(mc, buf, col0 + c, row0);
            }
            bulk_commit_group();
        }
        ++nstore;
    }
}

template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
               const __grid_constant__ CUtensorMap tma_c, const Params p)
{
    using C_ = Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* sa = smem;
    uint8_t* sb = smem + C_::STAGES * C_::A_BYTES;
    uint8_t* staging = sb + C_::STAGES * C_::B_BYTES;   // epilogue staging tiles
    uint64_t* full = reinterpret_cast<uint64_t*>(staging + kOutStaging);
    uint64_t* empty = full + C_::STAGES;
    uint64_t* tfull = empty + C_::STAGES;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0)
    {
        *abort = 0;
        for (int s = 0; s < C_::STAGES; ++s)
        {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b)
        {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4);
        }
        mbar_fence_init();
    }
    if (warp == 1)
    {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(C_::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    dep_wait();   // A, B and C belong to the kernels before this one
    dep_release();

    const int units = p.num_m * p.num_n * p.splits;

    if (warp == 0 && lane == 0)
    {
        tma_prefetch(&tma_a);
        tma_prefetch(&tma_b);
        int stage = 0;
        uint32_t phase = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x)
        {
            int mb, nb, split;
            unit_coords(u, p, mb, nb, split);
            const int kb0 = split * p.kb_per_split;
            const int kb1 = min(p.kblocks, kb0 + p.kb_per_split);
            for (int kb = kb0; kb < kb1; ++kb)
            {
                mbar_wait(&empty[stage], phase ^ 1, p.status, abort);
                mbar_expect_tx(&full[stage], C_::STAGE_BYTES);
                uint8_t* a_dst = sa + stage * C_::A_BYTES;
                uint8_t* b_dst = sb + stage * C_::B_BYTES;
                if constexpr (!A_MN)
                {
                    tma_load_2d(a_dst, &tma_a, &full[stage], kb * BK, mb * BM);
                }
                else
                {
#pragma unroll
                    for (int j = 0; j < BM / 64; ++j)
                    {
                        tma_load_2d(a_dst + j * (BK * 128), &tma_a, &full[stage], mb * BM + j * 64,
                                    kb * BK);
                    }
                }
                if constexpr (!B_MN)
                {
                    tma_load_2d(b_dst, &tma_b, &full[stage], kb * BK, nb * BN);
                }
                else
                {
#pragma unroll
                    for (int j = 0; j < BN / 64; ++j)
                    {
                        tma_load_2d(b_dst + j * (BK * 128), &tma_b, &full[stage], nb * BN + j * 64,
                                    kb * BK);
                    }
                }
                if (++stage == C_::STAGES)
                {
                    stage = 0;
                    phase ^= 1;
                }
            }
        }
    }
    else if (warp == 1 && lane == 0)
    {
        constexpr uint32_t idesc = instr_desc(BM, BN, A_MN, B_MN);
        int stage = 0;
        uint32_t phase = 0;
        int it = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x, ++it)
        {
            int mb, nb, split;
            unit_coords(u, p, mb, nb, split);
            const int kb0 = split * p.kb_per_split;
            const int kb1 = min(p.kblocks, kb0 + p.kb_per_split);
            const int buf = it & 1;
            const uint32_t tphase = (it >> 1) & 1;
            mbar_wait(&tempty[buf], tphase ^ 1, p.status, abort);
            fence_after();
            const uint32_t d = tmem + static_cast<uint32_t>(buf * BN);
            for (int kb = kb0; kb < kb1; ++kb)
            {
                mbar_wait(&full[stage], phase, p.status, abort);
                fence_after();
                const uint32_t a_base = smem_u32(sa + stage * C_::A_BYTES);
                const uint32_t b_base = smem_u32(sb + stage * C_::B_BYTES);
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk)
                {
                    const uint64_t ad = A_MN ? smem_desc(a_base + kk * 2048, BK * 128, 1024)
                                             : smem_desc(a_base + kk * 32, 16, 1024);
                    const uint64_t bd = B_MN ? smem_desc(b_base + kk * 2048, BK * 128, 1024)
                                             : smem_desc(b_base + kk * 32, 16, 1024);
                    mma(d, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
                }
                commit(&empty[stage]);
                if (++stage == C_::STAGES)
                {
                    stage = 0;
                    phase ^= 1;
                }
            }
            commit(&tfull[buf]);
        }
    }
    else if (warp >= 2)
    {
        const int quarter = warp & 3;
        uint32_t nstore = 0;
        int it = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x, ++it)
        {
            int mb, nb, split;
            unit_coords(u, p, mb, nb, split);
            const int buf = it & 1;
            const uint32_t tphase = (it >> 1) & 1;
            mbar_wait(&tfull[buf], tphase, p.status, abort);
            fence_after();
            const int row = mb * BM + quarter * 32 + lane;
            const uint32_t base = tmem + static_cast<uint32_t>(buf * BN) +
                                  (static_cast<uint32_t>(quarter * 32) << 16);
            if (p.out_mode != 0)
            {
                epilogue_tma<BN>(p, &tma_c, base, mb * BM + quarter * 32, nb * BN,
                                 staging + (warp - 2) * 2 * kStageTile, nstore, lane);
            }
            else
            {
#pragma unroll 1
                for (int c = 0; c < BN; c += 32)
                {
                    uint32_t r[32];
                    tmem_ld32(base + static_cast<uint32_t>(c), r);
                    store_chunk<BN>(p, row, nb * BN + c, r);
                }
            }
            fence_before();
            __syncwarp();
            if (lane == 0)
            {
                mbar_arrive(&tempty[buf]);
            }
        }
    }
    if (warp >= 2 && lane == 0)
    {
        bulk_wait_group<0>();   // staged output fully written before the CTA's memory goes
    }
    fence_before();
    __syncthreads();
    if (warp == 1)
    {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(C_::TMEM_COLS));
    }
}

// ---- paired-CTA kernel ------------------------------------------------------------------------
// A cluster of two CTAs on one TPC computes a 256 x 256 output tile with tcgen05.mma.cta_group::2
// (M = 256, N = 256, K = 16) issued by the even CTA: each CTA stages its own 128 rows of A and its
// own 128 columns of B (a 128 x 128 layout per CTA, exactly the single-CTA operand layout), and the
// tensor cores of the pair read both halves. Per k-block each SM then streams 32 KB instead of the
// 48 KB a 128 x 256 tile needs, and six stages fit in shared memory. Each CTA's TMEM receives its
// 128 rows of the tile (two 256-column accumulators); each CTA's epilogue stores its rows.
// Loads carry no multicast: each CTA loads only its own operand halves. The odd CTA's loads
// complete on the even CTA's stage barrier (the .cta_group::2 form of the TMA load, which may
// signal the peer's barrier); tcgen05.commit signals stage release and tile completion to the
// barriers of both CTAs; the odd CTA's epilogue releases an accumulator on the even CTA's barrier.
// ---- SwiGLU epilogues of the paired kernel ----------------------------------------------------
__device__ __forceinline__ uint32_t pack_bf16(float a, float b)
{
    const __nv_bfloat162 t = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&t);
}
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Writes this lane's row (64 bf16 as 32 packed words) of a 32 x 128-byte staging tile and stores
// the tile to (x, y) of `map`; the staging buffers alternate as in epilogue_tma.
__device__ __forceinline__ void stage_store(const CUtensorMap* map, const uint32_t (&w)[32], int x, int y,
                                            uint8_t* staging, uint32_t& nstore, int lane)
{
    uint8_t* buf = staging + (nstore & 1) * kStageTile;
    if (nstore >= 2)
    {
        if (lane == 0)
        {
            bulk_wait_group_read<1>();
        }
        __syncwarp();
    }
    uint8_t* row = buf + lane * 128;
#pragma unroll
    for (int k = 0; k < 8; ++k)
    {
        *reinterpret_cast<uint4*>(row + ((k ^ (lane & 7)) << 4)) =
            make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
    }
    fence_proxy_async();
    __syncwarp();
    if (lane == 0)
    {
        tma_store_2d(map, buf, x, y);
        bulk_commit_group();
    }
    ++nstore;
}

// EPI 1, one warp's 32 rows: accumulator columns 0-127 are gate columns gcol.. of the [M, 2F]
// output and 128-255 the up columns F + gcol..; writes both (bf16) and h = silu(gate) * up,
// computed from the bf16-rounded gate and up as the stand-alone SwiGLU reads them, into H.
__device__ __forceinline__ void epilogue_swiglu(const Params& p, const CUtensorMap* mc,
                                                const CUtensorMap* mh, uint32_t taddr, int row0,
                                                int gcol, uint8_t* staging, uint32_t& nstore, int lane)
{
    if (row0 >= p.M)
    {
        return;
    }
#pragma unroll 1
    for (int c = 0; c < 128; c += 64)
    {
        uint32_t gw[32], uw[32], hw[32];
#pragma unroll
        for (int half = 0; half < 2; ++half)
        {
            uint32_t a[32], b[32];
            tmem_ld32(taddr + static_cast<uint32_t>(c + half * 32), a);
            tmem_ld32(taddr + static_cast<uint32_t>(128 + c + half * 32), b);
#pragma unroll
            for (int q = 0; q < 16; ++q)
            {
                const uint32_t g2 = pack_bf16(__uint_as_float(a[2 * q]), __uint_as_float(a[2 * q + 1]));
                const uint32_t u2 = pack_bf16(__uint_as_float(b[2 * q]), __uint_as_float(b[2 * q + 1]));
                gw[half * 16 + q] = g2;
                uw[half * 16 + q] = u2;
                hw[half * 16 + q] = pack_bf16(swiglu_value(bf16_lo(g2), bf16_lo(u2)),
                                              swiglu_value(bf16_hi(g2), bf16_hi(u2)));
            }
        }
        stage_store(mc, gw, gcol + c, row0, staging, nstore, lane);
        stage_store(mc, uw, p.F + gcol + c, row0, staging, nstore, lane);
        stage_store(mh, hw, gcol + c, row0, staging, nstore, lane);
    }
}

// EPI 2 staging: per warp four 2 KB tiles of 32 rows x 64 bytes (32 bf16) with the 64-byte swizzle
// (row r's 16-byte segment s at s ^ ((r >> 1) & 3)), gate and up of two 32-column chunks, so one
// chunk's gate and up load while the other's are computed; dg and du overwrite them in place.
constexpr int kChunkTile = 32 * 64;

__device__ __forceinline__ uint32_t swz64(int r, int s)
{
    return static_cast<uint32_t>(r * 64 + ((s ^ ((r >> 1) & 3)) << 4));
}

// Asynchronous copy of a warp's 32 rows x 32 bf16 of `src` (row stride ld) into a staging tile:
// four 16-byte copies a lane, each instruction eight whole 64-byte rows; rows at or past M are
// filled with zeros.
__device__ __forceinline__ void copy_chunk_async(uint8_t* tile, const bf16* src, int64_t ld, int row0,
                                                 int M, int lane)
{
    const int seg = lane & 3;
#pragma unroll
    for (int k = 0; k < 4; ++k)
    {
        const int r = 8 * k + (lane >> 2);
        const bool in = row0 + r < M;
        const int row = in ? row0 + r : M - 1;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(tile + swz64(r, seg))),
                     "l"(src + static_cast<int64_t>(row) * ld + seg * 8), "r"(in ? 16u : 0u)
                     : "memory");
    }
}

// Gate and up of chunk j (columns col0 + 32 j) into the warp's tile pair j & 1, as one group.
__device__ __forceinline__ void dswiglu_load(const Params& p, int row0, int col0, int j, uint8_t* staging,
                                             int lane)
{
    uint8_t* const pair = staging + (j & 1) * 2 * kChunkTile;
    copy_chunk_async(pair, p.gu + col0 + 32 * j, p.ldgu, row0, p.M, lane);
    copy_chunk_async(pair + kChunkTile, p.gu + p.F + col0 + 32 * j, p.ldgu, row0, p.M, lane);
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// EPI 2, before the unit's accumulator is ready: once the last unit's stores have read the
// staging tiles, chunks 0 and 1 start loading.
__device__ __forceinline__ void dswiglu_start(const Params& p, int row0, int col0, uint8_t* staging,
                                              uint32_t nstore, int lane)
{
    if (row0 >= p.M)
    {
        return;
    }
    if (nstore > 0)
    {
        if (lane == 0)
        {
            bulk_wait_group_read<0>();
        }
        __syncwarp();
    }
    dswiglu_load(p, row0, col0, 0, staging, lane);
    dswiglu_load(p, row0, col0, 1, staging, lane);
}

// EPI 2, one warp's 32 rows x 128 columns (col0..) of the [M, F] intermediate, whose dh the
// accumulator at taddr holds, in four chunks of 32 columns: dh rounded to bf16 (as the stand-alone
// path stores it) with gate and up of the same rows and columns (p.gu) gives dg and du, written
// into C, the [M, 2F] gradient of gate|up, at col0 and F + col0 (C's map: 32 x 32 boxes, 64-byte
// swizzle). Chunk j + 2 loads into the tiles of chunk j once chunk j's stores have read them.
__device__ __forceinline__ void epilogue_dswiglu(const Params& p, const CUtensorMap* mc, uint32_t taddr,
                                                 int row0, int col0, uint8_t* staging,
                                                 uint32_t& nstore, int lane)
{
    if (row0 >= p.M)
    {
        return;
    }
#pragma unroll 1
    for (int j = 0; j < 4; ++j)
    {
        if (j < 3)
        {
            asm volatile("cp.async.wait_group 1;" ::: "memory");   // chunk j's group is complete
        }
        else
        {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncwarp();   // every lane's copies (other lanes' rows) are visible to the warp
        uint8_t* const tg = staging + (j & 1) * 2 * kChunkTile;
        uint8_t* const tu = tg + kChunkTile;
        uint32_t d[32];
        tmem_ld32(taddr + static_cast<uint32_t>(32 * j), d);
#pragma unroll
        for (int k = 0; k < 4; ++k)
        {
            uint4* const gk = reinterpret_cast<uint4*>(tg + swz64(lane, k));
            uint4* const uk = reinterpret_cast<uint4*>(tu + swz64(lane, k));
            const uint4 gv = *gk, uv = *uk;
            const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
            const uint32_t uw[4] = {uv.x, uv.y, uv.z, uv.w};
            uint32_t og[4], ou[4];
#pragma unroll
            for (int q = 0; q < 4; ++q)
            {
                const uint32_t d2 = pack_bf16(__uint_as_float(d[8 * k + 2 * q]), __uint_as_float(d[8 * k + 2 * q + 1]));
                uint64_t dg2, du2;
                swiglu_grads2(pk(bf16_lo(gw[q]), bf16_hi(gw[q])), pk(bf16_lo(uw[q]), bf16_hi(uw[q])),
                              pk(bf16_lo(d2), bf16_hi(d2)), dg2, du2);
                float dg0, dg1, du0, du1;
                upk(dg2, dg0, dg1);
                upk(du2, du0, du1);
                og[q] = pack_bf16(dg0, dg1);
                ou[q] = pack_bf16(du0, du1);
            }
            *gk = make_uint4(og[0], og[1], og[2], og[3]);
            *uk = make_uint4(ou[0], ou[1], ou[2], ou[3]);
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0)
        {
            tma_store_2d(mc, tg, col0 + 32 * j, row0);
            tma_store_2d(mc, tu, p.F + col0 + 32 * j, row0);
            bulk_commit_group();
        }
        ++nstore;
        if (j + 2 < 4)
        {
            if (lane == 0)
            {
                bulk_wait_group_read<0>();   // the stores just issued have read the pair
            }
            __syncwarp();
            dswiglu_load(p, row0, col0, j + 2, staging, lane);
        }
    }
}

// The paired kernel's shape per epilogue: EPI 2 (SwiGLU's backward, the heaviest epilogue) runs
// eight epilogue warps, two per scheduler, each on half of the tile's columns, and one pipeline
// stage less to stage their tiles; the others run four (eight measured slower for EPI 1).
template <int EPI>
struct Cfg2
{
    static constexpr int EPI_WARPS = EPI == 2 ? 8 : 4;
    static constexpr int THREADS = 64 + 32 * EPI_WARPS;
    static constexpr int STAGES = EPI == 2 ? 5 : 6;
    static constexpr int A_BYTES = 128 * BK * 2;   // this CTA's 128 rows of A
    static constexpr int B_BYTES = 128 * BK * 2;   // this CTA's 128 columns of B
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = 512;
    static constexpr int STAGING = EPI_WARPS * 2 * kStageTile;
    static constexpr int SMEM = STAGES * STAGE_BYTES + STAGING + 1024 + 256;
};

__device__ __forceinline__ uint32_t cluster_rank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// shared::cluster address of the same shared variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank)
{
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync()
{
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// TMA tile load whose completion may be signalled on the peer CTA's barrier (no multicast).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster,
                                                 int x, int y)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Arrives (once the issuing thread's MMAs complete) on the barrier at this offset in both CTAs.
__device__ __forceinline__ void commit_pair(uint64_t* bar)
{
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;" ::"r"(smem_u32(bar)),
        "h"(static_cast<uint16_t>(3))
        : "memory");
}

template <bool A_MN, bool B_MN, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Cfg2<EPI>::THREADS, 1)
tc_gemm2_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                const __grid_constant__ CUtensorMap tma_c, const __grid_constant__ CUtensorMap tma_h,
                const Params p)
{
    using C_ = Cfg2<EPI>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* sa = smem;
    uint8_t* sb = smem + C_::STAGES * C_::A_BYTES;
    uint8_t* staging = sb + C_::STAGES * C_::B_BYTES;   // epilogue staging tiles
    uint64_t* full = reinterpret_cast<uint64_t*>(staging + C_::STAGING);
    uint64_t* empty = full + C_::STAGES;
    uint64_t* tfull = empty + C_::STAGES;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();     // 0: issues the MMAs; 1: its peer
    const int cid = static_cast<int>(blockIdx.x >> 1);
    const int nclusters = static_cast<int>(gridDim.x >> 1);

    if (threadIdx.x == 0)
    {
        *abort = 0;
        for (int s = 0; s < C_::STAGES; ++s)
        {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b)
        {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 2 * C_::EPI_WARPS);   // the epilogue warps of both CTAs
        }
        mbar_fence_init();
    }
    if (warp == 1)
    {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(C_::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    fence_before();
    __syncthreads();
    cluster_sync();   // both CTAs' barriers are initialised before any cross-CTA signal
    fence_after();
    const uint32_t tmem = *tmem_slot;
    dep_wait();   // A, B and C belong to the kernels before this one
    dep_release();

    const int units = p.num_m * p.num_n * p.splits;

    if (warp == 0 && lane == 0)
    {
        tma_prefetch(&tma_a);
        tma_prefetch(&tma_b);
        int stage = 0;
        uint32_t phase = 0;
        for (int u = cid; u < units; u += nclusters)
        {
            int mb, nb, split;
            unit_coords(u, p, mb, nb, split);
            const int kb0 = split * p.kb_per_split;
            const int kb1 = min(p.kblocks, kb0 + p.kb_per_split);
            const int row0 = mb * 256 + static_cast<int>(rank) * 128;
            // EPI 1: the tile's B columns are 128 gate rows of W (this CTA's half at rank 0) and
            // the 128 matching up rows, F further on (rank 1)
            const int col0 = EPI == 1 ? (rank == 0 ? nb * 128 : p.F + nb * 128)
                                      : nb * 256 + static_cast<int>(rank) * 128;
            for (int kb = kb0; kb < kb1; ++kb)
            {
                mbar_wait(&empty[stage], phase ^ 1, p.status, abort);
                if (rank == 0)
                {
                    mbar_expect_tx(&full[stage], 2 * C_::STAGE_BYTES);   // both CTAs' halves
                }
                const uint32_t bar = peer_addr(&full[stage], 0);
                uint8_t* a_dst = sa + stage * C_::A_BYTES;
                uint8_t* b_dst = sb + stage * C_::B_BYTES;
                if constexpr (!A_MN)
                {
                    tma_load_2d_pair(a_dst, &tma_a, bar, kb * BK, row0);
                }
                else
                {
#pragma unroll
                    for (int j = 0; j < 2; ++j)
                    {
                        tma_load_2d_pair(a_dst + j * (BK * 128), &tma_a, bar, row0 + j * 64, kb * BK);
                    }
                }
                if constexpr (!B_MN)
                {
                    tma_load_2d_pair(b_dst, &tma_b, bar, kb * BK, col0);
                }
                else
                {
#pragma unroll
                    for (int j = 0; j < 2; ++j)
                    {
                        tma_load_2d_pair(b_dst + j * (BK * 128), &tma_b, bar, col0 + j * 64, kb * BK);
                    }
                }
                if (++stage == C_::STAGES)
                {
                    stage = 0;
                    phase ^= 1;
                }
            }
        }
    }
    else if (warp == 1 && lane == 0 && rank == 0)
    {
        constexpr uint32_t idesc = instr_desc(256, 256, A_MN, B_MN);
        int stage = 0;
        uint32_t phase = 0;
        int it = 0;
        for (int u = cid; u < units; u += nclusters, ++it)
        {
            int mb, nb, split;
            unit_coords(u, p, mb, nb, split);
            const int kb0 = split * p.kb_per_split;
            const int kb1 = min(p.kblocks, kb0 + p.kb_per_split);
            const int buf = it & 1;
            const uint32_t tphase = (it >> 1) & 1;
            mbar_wait(&tempty[buf], tphase ^ 1, p.status, abort);
            fence_after();
            const uint32_t d = tmem + static_cast<uint32_t>(buf * 256);
            for (int kb = kb0; kb < kb1; ++kb)
            {
                mbar_wait(&full[stage], phase, p.status, abort);
                fence_after();
                const uint32_t a_base = smem_u32(sa + stage * C_::A_BYTES);
                const uint32_t b_base = smem_u32(sb + stage * C_::B_BYTES);
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk)
                {
                    const uint64_t ad = A_MN ? smem_desc(a_base + kk * 2048, BK * 128, 1024)
                                             : smem_desc(a_base + kk * 32, 16, 1024);
                    const uint64_t bd = B_MN ? smem_desc(b_base + kk * 2048, BK * 128, 1024)
                                             : smem_desc(b_base + kk * 32, 16, 1024);
                    mma_pair(d, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
                }
                commit_pair(&empty[stage]);
                if (++stage == C_::STAGES)
                {
                    stage = 0;
                    phase ^= 1;
                }
            }
            commit_pair(&tfull[buf]);
        }
    }
    else if (warp >= 2)
    {
        const int quarter = warp & 3;
        // EPI 2: warps 2-5 take the tile's columns 0-127, warps 6-9 columns 128-255
        const int chalf = (warp - 2) >> 2;
        const uint32_t release = peer_addr(&tempty[0], 0);   // the even CTA's tempty[0]
        uint8_t* const wstage = staging + (warp - 2) * 2 * kStageTile;
        uint32_t nstore = 0;
        int it = 0;
        for (int u = cid; u < units; u += nclusters, ++it)
        {
            int mb, nb, split;
            unit_coords(u, p, mb, nb, split);
            const int buf = it & 1;
            const uint32_t tphase = (it >> 1) & 1;
            const int row = mb * 256 + static_cast<int>(rank) * 128 + quarter * 32 + lane;
            if constexpr (EPI == 2)
            {
                // gate and up of the first two chunks load while the products finish
                dswiglu_start(p, row - lane, nb * 256 + chalf * 128, wstage, nstore, lane);
            }
            mbar_wait(&tfull[buf], tphase, p.status, abort);
            fence_after();
            const uint32_t base = tmem + static_cast<uint32_t>(buf * 256) +
                                  (static_cast<uint32_t>(quarter * 32) << 16);
            if constexpr (EPI == 1)
            {
                epilogue_swiglu(p, &tma_c, &tma_h, base, row - lane, nb * 128, wstage, nstore, lane);
            }
            else if constexpr (EPI == 2)
            {
                epilogue_dswiglu(p, &tma_c, base + static_cast<uint32_t>(chalf * 128), row - lane,
                                 nb * 256 + chalf * 128, wstage, nstore, lane);
            }
            else if (p.out_mode != 0)
            {
                epilogue_tma<256>(p, &tma_c, base, row - lane, nb * 256, wstage, nstore, lane);
            }
            else
            {
#pragma unroll 1
                for (int c = 0; c < 256; c += 32)
                {
                    uint32_t r[32];
                    tmem_ld32(base + static_cast<uint32_t>(c), r);
                    store_chunk<256>(p, row, nb * 256 + c, r);
                }
            }
            fence_before();
            __syncwarp();
            if (lane == 0)
            {
                asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(
                                 release + static_cast<uint32_t>(buf * 8))
                             : "memory");
            }
        }
    }
    if (warp >= 2 && lane == 0)
    {
        bulk_wait_group<0>();   // staged output fully written before the CTA's memory goes
    }
    fence_before();
    __syncthreads();
    cluster_sync();   // no CTA leaves while its peer may still read its operands or barriers
    if (warp == 1)
    {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(C_::TMEM_COLS));
    }
}

// ---- host ------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                             &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
        {
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        }
    });
    return fn;
}

// 2-D bf16 tensor map over a row-major matrix with `inner` contiguous elements per row.
bool make_map(CUtensorMap* map, const void* base, int64_t inner, int64_t outer, int64_t ld,
              uint32_t box_inner, uint32_t box_outer)
{
    auto fn = encode_fn();
    if (fn == nullptr)
    {
        return false;
    }
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int BN, bool A_MN, bool B_MN>
int launch_tc(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const Params& p,
              int grid, cudaStream_t s)
{
    auto kernel = tc_gemm_kernel<BN, A_MN, B_MN>;
    static int configured_device = -1;
    int device = 0;
    cudaGetDevice(&device);
    if (configured_device != device)
    {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<BN>::SMEM);
        configured_device = device;
    }
    return launch("veda_gemm (tcgen05)", kernel, dim3(grid), dim3(kThreads), Cfg<BN>::SMEM, s, ma, mb,
                  mc, p);
}

// Launches the paired-CTA kernel on `clusters` clusters of two; -1 if clusters cannot be
// scheduled (the caller then uses the single-CTA kernel).
template <bool A_MN, bool B_MN, int EPI = 0>
int launch_tc2(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const Params& p,
               int clusters, cudaStream_t s, const CUtensorMap* mh = nullptr)
{
    auto kernel = tc_gemm2_kernel<A_MN, B_MN, EPI>;
    return launch("veda_gemm (tcgen05, CTA pair)", kernel, dim3(2 * clusters), dim3(Cfg2<EPI>::THREADS),
                  Cfg2<EPI>::SMEM, s, ma, mb, mc, mh != nullptr ? *mh : mc, p);
}

// How many two-CTA clusters of the paired kernel fit on the device at once (0: none).
template <bool A_MN, bool B_MN, int EPI = 0>
int pair_clusters()
{
    static int cached_device = -1, cached = 0;
    int device = 0;
    cudaGetDevice(&device);
    if (cached_device != device)
    {
        auto kernel = tc_gemm2_kernel<A_MN, B_MN, EPI>;
        cached = 0;
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg2<EPI>::SMEM) ==
            cudaSuccess)
        {
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(2 * (sm_count() / 2));
            cfg.blockDim = dim3(Cfg2<EPI>::THREADS);
            cfg.dynamicSmemBytes = Cfg2<EPI>::SMEM;
            cudaLaunchAttribute attr{};
            attr.id = cudaLaunchAttributeClusterDimension;
            attr.val.clusterDim.x = 2;
            attr.val.clusterDim.y = 1;
            attr.val.clusterDim.z = 1;
            cfg.attrs = &attr;
            cfg.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) == cudaSuccess)
            {
                cached = n;
            }
            cudaGetLastError();
        }
        cached_device = device;
    }
    return cached;
}

// The paired kernel serves M, N >= 256 unless VEDA_GEMM_SINGLE_CTA=1.
bool pair_enabled()
{
    static const bool enabled = [] {
        const char* v = std::getenv("VEDA_GEMM_SINGLE_CTA");
        return !(v != nullptr && v[0] == '1');
    }();
    return enabled;
}

// How the epilogue writes C: TMA store (beta = 0), TMA fp32 reduce-add (split-K partial tiles, or
// beta = 1 accumulation into fp32), else per-thread stores from registers (general beta, bf16
// accumulation, or a C whose base / row pitch a tensor map cannot describe). Builds the C map.
int output_mode(Params& p, CUtensorMap* mc, void* C, int64_t M, int64_t N, int64_t ldc, float beta)
{
    p.out_mode = 0;
    if (!p.vec_ok)
    {
        return 0;
    }
    int mode = 0;
    if (p.atomic)
    {
        mode = p.out_f32 ? 2 : 0;
    }
    else if (beta == 0.0f)
    {
        mode = 1;
    }
    else if (beta == 1.0f && p.out_f32)
    {
        mode = 2;
    }
    if (mode == 0)
    {
        return 0;
    }
    auto fn = encode_fn();
    if (fn == nullptr)
    {
        return 0;
    }
    const size_t es = p.out_f32 ? 4 : 2;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldc) * es};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / es), 32};
    const cuuint32_t estr[2] = {1, 1};
    if (fn(mc, p.out_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, C,
           dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    {
        return 0;
    }
    p.out_mode = mode;
    return mode;
}

// Picks a split-K factor (fp32 output only) that best fills whole waves of `slots` workers (SMs,
// or CTA pairs): the fraction of worker-time doing useful tiles, less a small charge per extra
// split for its atomic traffic.
int choose_splits(int tiles, int kblocks, bool allowed, int slots)
{
    const int sms = slots;
    if (!allowed)
    {
        return 1;
    }
    int best = 1;
    double best_score = -1.0;
    for (int s = 1; s <= 8; ++s)
    {
        const int per = (kblocks + s - 1) / s;
        if (s > 1 && (per < 8 || (s - 1) * per >= kblocks))
        {
            break;
        }
        const int units = tiles * s;
        const int waves = (units + sms - 1) / sms;
        const double score = static_cast<double>(units) / (waves * sms) - 0.03 * (s - 1);
        if (score > best_score)
        {
            best_score = score;
            best = s;
        }
    }
    return best;
}

// 256 x 256 tiles on CTA pairs; -1 when the pair kernel cannot run (tensor maps, clusters, or a
// split-K that needs a general beta), so the caller uses the single-CTA kernel.
int tc_gemm_pair(int op, int64_t M, int64_t N, int64_t K, const void* A, int64_t lda, const void* B,
                 int64_t ldb, void* C, int64_t ldc, int dtype_c, float alpha, float beta,
                 cudaStream_t s)
{
    const bool a_mn = op == kTN;
    const bool b_mn = op != kNT;
    const int clusters_max = std::min(op == kNT ? pair_clusters<false, false>()
                                      : op == kNN ? pair_clusters<false, true>()
                                                  : pair_clusters<true, true>(),
                                      compute_sms() / 2);
    if (clusters_max < 1)
    {
        return -1;
    }
    CUtensorMap ma, mb;
    // each CTA loads a 128-row (or, MN-major, 2 x 64-column) piece of its own half
    bool ok = a_mn ? make_map(&ma, A, M, K, lda, 64, 64) : make_map(&ma, A, K, M, lda, 64, 128);
    ok = ok && (b_mn ? make_map(&mb, B, N, K, ldb, 64, 64) : make_map(&mb, B, K, N, ldb, 64, 128));
    if (!ok)
    {
        return -1;
    }
    Params p{};
    p.M = static_cast<int>(M);
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.num_m = static_cast<int>((M + 255) / 256);
    p.num_n = static_cast<int>((N + 255) / 256);
    p.kblocks = static_cast<int>((K + BK - 1) / BK);
    p.C = C;
    p.ldc = ldc;
    p.alpha = alpha;
    p.beta = beta;
    p.out_f32 = dtype_c == VEDA_F32;
    p.vec_ok = aligned16(C) && (ldc % (dtype_c == VEDA_F32 ? 4 : 8)) == 0;
    p.status = device_status_ptr();
    const int tiles = p.num_m * p.num_n;
    p.splits = choose_splits(tiles, p.kblocks, p.out_f32 != 0, clusters_max);
    p.kb_per_split = (p.kblocks + p.splits - 1) / p.splits;
    p.atomic = p.splits > 1;
    if (p.atomic)
    {
        if (beta != 0.0f && beta != 1.0f)
        {
            return -1;
        }
        if (beta == 0.0f && cudaMemset2DAsync(C, ldc * 4, 0, N * 4, M, s) != cudaSuccess)
        {
            return fail(VEDA_ERR_CUDA, "veda_gemm: clearing C for split-K failed");
        }
        p.beta = 0.0f;
    }
    CUtensorMap mc{};
    output_mode(p, &mc, C, M, N, ldc, beta);
    const int clusters = std::min(tiles * p.splits, clusters_max);
    if (op == kNT) return launch_tc2<false, false>(ma, mb, mc, p, clusters, s);
    if (op == kNN) return launch_tc2<false, true>(ma, mb, mc, p, clusters, s);
    return launch_tc2<true, true>(ma, mb, mc, p, clusters, s);
}

// bf16 store map of the epilogue: 64-column x 32-row boxes with the 128-byte swizzle, or (narrow)
// 32-column boxes with the 64-byte swizzle.
bool make_store_map(CUtensorMap* map, void* base, int64_t inner, int64_t outer, int64_t ld,
                    bool narrow = false)
{
    auto fn = encode_fn();
    if (fn == nullptr)
    {
        return false;
    }
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
    const cuuint32_t box[2] = {narrow ? 32u : 64u, 32};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE,
              narrow ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool swiglu_shapes_ok(int64_t rows, int64_t F, int64_t D, int64_t tile)
{
    return pair_enabled() && rows >= 256 && rows < (1ll << 31) && F >= tile && F % tile == 0 &&
           2 * F < (1ll << 31) && D >= 16 && D % 8 == 0 && D < (1ll << 31);
}

// The gate|up projection with SwiGLU in its epilogue (paired kernel, EPI 1): gu[rows, 2F] =
// x[rows, D] W[2F, D]^T (W's rows 0..F-1 gate, F..2F-1 up) and h[rows, F] = silu(gate) * up.
// Each tile pairs 128 gate columns with the 128 matching up columns. -1: not for this kernel.
int gemm_swiglu_fwd_tc(int64_t rows, int64_t F, int64_t D, const void* x, int64_t ldx, const void* w,
                       int64_t ldw, void* gu, int64_t ldgu, void* h, int64_t ldh, cudaStream_t s)
{
    if (!swiglu_shapes_ok(rows, F, D, 128) || !aligned16(x) || !aligned16(w) || !aligned16(gu) ||
        !aligned16(h) || ldx % 8 != 0 || ldw % 8 != 0 || ldgu % 8 != 0 || ldh % 8 != 0)
    {
        return -1;
    }
    const int clusters_max = std::min(pair_clusters<false, false, 1>(), compute_sms() / 2);
    CUtensorMap ma, mb, mc, mh;
    if (clusters_max < 1 || !make_map(&ma, x, D, rows, ldx, 64, 128) ||
        !make_map(&mb, w, D, 2 * F, ldw, 64, 128) || !make_store_map(&mc, gu, 2 * F, rows, ldgu) ||
        !make_store_map(&mh, h, F, rows, ldh))
    {
        return -1;
    }
    Params p{};
    p.M = static_cast<int>(rows);
    p.N = static_cast<int>(2 * F);
    p.K = static_cast<int>(D);
    p.num_m = static_cast<int>((rows + 255) / 256);
    p.num_n = static_cast<int>(F / 128);
    p.kblocks = static_cast<int>((D + BK - 1) / BK);
    p.splits = 1;
    p.kb_per_split = p.kblocks;
    p.C = gu;
    p.ldc = ldgu;
    p.alpha = 1.0f;
    p.vec_ok = 1;
    p.out_mode = 1;
    p.status = device_status_ptr();
    p.F = static_cast<int>(F);
    const int tiles = p.num_m * p.num_n;
    return launch_tc2<false, false, 1>(ma, mb, mc, p, std::min(tiles, clusters_max), s, &mh);
}

// The down projection's input gradient with SwiGLU's backward in its epilogue (paired kernel,
// EPI 2): dh = dy[rows, D] W[D, F] stays in TMEM; with gate and up from gu[rows, 2F] the
// epilogue writes dgu[rows, 2F] = (dgate | dup). -1: not for this kernel.
int gemm_swiglu_bwd_tc(int64_t rows, int64_t F, int64_t D, const void* dy, int64_t lddy, const void* w,
                       int64_t ldw, const void* gu, int64_t ldgu, void* dgu, int64_t lddgu, cudaStream_t s)
{
    if (!swiglu_shapes_ok(rows, F, D, 256) || !aligned16(dy) || !aligned16(w) || !aligned16(gu) ||
        !aligned16(dgu) || lddy % 8 != 0 || ldw % 8 != 0 || ldgu % 8 != 0 || lddgu % 8 != 0)
    {
        return -1;
    }
    const int clusters_max = std::min(pair_clusters<false, true, 2>(), compute_sms() / 2);
    CUtensorMap ma, mb, mc;
    if (clusters_max < 1 || !make_map(&ma, dy, D, rows, lddy, 64, 128) ||
        !make_map(&mb, w, F, D, ldw, 64, 64) || !make_store_map(&mc, dgu, 2 * F, rows, lddgu, true))
    {
        return -1;
    }
    Params p{};
    p.M = static_cast<int>(rows);
    p.N = static_cast<int>(F);
    p.K = static_cast<int>(D);
    p.num_m = static_cast<int>((rows + 255) / 256);
    p.num_n = static_cast<int>(F / 256);
    p.kblocks = static_cast<int>((D + BK - 1) / BK);
    p.splits = 1;
    p.kb_per_split = p.kblocks;
    p.C = dgu;
    p.ldc = lddgu;
    p.alpha = 1.0f;
    p.vec_ok = 1;
    p.out_mode = 1;
    p.status = device_status_ptr();
    p.F = static_cast<int>(F);
    p.gu = static_cast<const bf16*>(gu);
    p.ldgu = ldgu;
    const int tiles = p.num_m * p.num_n;
    return launch_tc2<false, true, 2>(ma, mb, mc, p, std::min(tiles, clusters_max), s);
}

int tc_gemm(int op, int64_t M, int64_t N, int64_t K, const void* A, int64_t lda, const void* B,
            int64_t ldb, void* C, int64_t ldc, int dtype_c, float alpha, float beta, cudaStream_t s)
{
    const bool a_mn = op == kTN;
    const bool b_mn = op != kNT;
    if (M >= 256 && N >= 256 && pair_enabled())
    {
        const int rc = tc_gemm_pair(op, M, N, K, A, lda, B, ldb, C, ldc, dtype_c, alpha, beta, s);
        if (rc != -1)
        {
            return rc;
        }
    }
    const int BN = N >= 256 ? 256 : 128;
    CUtensorMap ma, mb;
    bool ok = a_mn ? make_map(&ma, A, M, K, lda, 64, 64) : make_map(&ma, A, K, M, lda, 64, BM);
    ok = ok && (b_mn ? make_map(&mb, B, N, K, ldb, 64, 64)
                     : make_map(&mb, B, K, N, ldb, 64, static_cast<uint32_t>(BN)));
    if (!ok)
    {
        return -1;   // caller falls back
    }
    Params p{};
    p.M = static_cast<int>(M);
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.num_m = static_cast<int>((M + BM - 1) / BM);
    p.num_n = static_cast<int>((N + BN - 1) / BN);
    p.kblocks = static_cast<int>((K + BK - 1) / BK);
    p.C = C;
    p.ldc = ldc;
    p.alpha = alpha;
    p.beta = beta;
    p.out_f32 = dtype_c == VEDA_F32;
    p.vec_ok = aligned16(C) && (ldc % (dtype_c == VEDA_F32 ? 4 : 8)) == 0;
    p.status = device_status_ptr();
    const int tiles = p.num_m * p.num_n;
    p.splits = choose_splits(tiles, p.kblocks, p.out_f32 != 0, compute_sms());
    p.kb_per_split = (p.kblocks + p.splits - 1) / p.splits;
    p.atomic = p.splits > 1;
    if (p.atomic)
    {
        // partial tiles are added onto C: first bring C to beta * C
        if (beta == 0.0f)
        {
            if (cudaMemset2DAsync(C, ldc * 4, 0, N * 4, M, s) != cudaSuccess)
            {
                return fail(VEDA_ERR_CUDA, "veda_gemm: clearing C for split-K failed");
            }
        }
        else if (beta != 1.0f)
        {
            return -1;   // general beta with split-K: let the caller use one split
        }
        p.beta = 0.0f;
    }
    CUtensorMap mc{};
    output_mode(p, &mc, C, M, N, ldc, beta);
    const int units = tiles * p.splits;
    const int grid = std::min(units, compute_sms());
    const bool big = BN == 256;
    if (op == kNT)
        return big ? launch_tc<256, false, false>(ma, mb, mc, p, grid, s)
                   : launch_tc<128, false, false>(ma, mb, mc, p, grid, s);
    if (op == kNN)
        return big ? launch_tc<256, false, true>(ma, mb, mc, p, grid, s)
                   : launch_tc<128, false, true>(ma, mb, mc, p, grid, s);
    return big ? launch_tc<256, true, true>(ma, mb, mc, p, grid, s)
               : launch_tc<128, true, true>(ma, mb, mc, p, grid, s);
}

bool tc_eligible(int op, int64_t M, int64_t N, int64_t K, const void* A, int64_t lda,
                 const void* B, int64_t ldb)
{
    (void)op;
    return M >= 1 && N >= 16 && K >= 16 && M < (1ll << 31) && N < (1ll << 31) &&
           K < (1ll << 31) && aligned16(A) && aligned16(B) && lda % 8 == 0 && ldb % 8 == 0;
}

int gemm_dispatch(int op, int64_t batch, int64_t M, int64_t N, int64_t K, const void* A,
                  int64_t lda, int64_t sa, const void* B, int64_t ldb, int64_t sb, void* C,
                  int64_t ldc, int64_t sc, int dtype_ab, int dtype_c, float alpha, float beta,
                  cudaStream_t s)
{
    VEDA_REQUIRE(valid_dtype(dtype_ab) && valid_dtype(dtype_c), "unknown dtype");
    VEDA_REQUIRE(op >= 0 && op <= 2, "unknown op");
    VEDA_REQUIRE(batch >= 0 && M >= 0 && N >= 0 && K >= 0, "negative extent");
    const int64_t a_rows = op == kTN ? K : M, a_cols = op == kTN ? M : K;
    const int64_t b_rows = op == kNT ? N : K, b_cols = op == kNT ? K : N;
    VEDA_REQUIRE(a_rows == 0 || lda >= a_cols, "lda smaller than the row length of A");
    VEDA_REQUIRE(b_rows == 0 || ldb >= b_cols, "ldb smaller than the row length of B");
    VEDA_REQUIRE(M == 0 || ldc >= N, "ldc smaller than N");
    (void)b_rows;
    if (batch == 0 || M == 0 || N == 0)
    {
        return VEDA_OK;
    }
    VEDA_REQUIRE(A != nullptr && B != nullptr && C != nullptr, "null pointer");
    if (K == 0)
    {
        // the empty sum is 0 (Matmul.cpp:63): C = beta * C
        for (int64_t z = 0; z < batch; ++z)
        {
            char* c = static_cast<char*>(C) + z * sc * static_cast<int64_t>(dtype_size(dtype_c));
            for (int64_t r = 0; r < M; ++r)
            {
                const int rc = veda_scale(c + r * ldc * static_cast<int64_t>(dtype_size(dtype_c)),
                                          beta, c + r * ldc * static_cast<int64_t>(dtype_size(dtype_c)),
                                          N, dtype_c, s);
                if (rc != VEDA_OK) return rc;
            }
        }
        return VEDA_OK;
    }
    if (dtype_ab == VEDA_BF16 && tc_eligible(op, M, N, K, A, lda, B, ldb))
    {
        const size_t es = 2, ec = dtype_size(dtype_c);
        bool all = true;
        for (int64_t z = 0; z < batch && all; ++z)
        {
            const char* a = static_cast<const char*>(A) + z * sa * static_cast<int64_t>(es);
            const char* b = static_cast<const char*>(B) + z * sb * static_cast<int64_t>(es);
            char* c = static_cast<char*>(C) + z * sc * static_cast<int64_t>(ec);
            if (!aligned16(a) || !aligned16(b))
            {
                all = false;
                break;
            }
            const int rc = tc_gemm(op, M, N, K, a, lda, b, ldb, c, ldc, dtype_c, alpha, beta, s);
            if (rc == -1)
            {
                if (z != 0)
                {
                    return fail(VEDA_ERR_CUDA, "veda_gemm: tensor-map creation failed mid-batch");
                }
                all = false;
                break;
            }
            if (rc != VEDA_OK)
            {
                return rc;
            }
        }
        if (all)
        {
            return VEDA_OK;
        }
    }
    return simt_gemm(op, batch, M, N, K, A, lda, sa, B, ldb, sb, C, ldc, sc, dtype_ab, dtype_c,
                     alpha, beta, s);
}

} // namespace
} // namespace veda::cuda

using namespace veda::cuda;

extern "C" int veda_gemm_nt(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda,
                            const void* B, int64_t ldb, void* C, int64_t ldc, int dtype_ab,
                            int dtype_c, float alpha, float beta, veda_stream_t stream)
{
    return gemm_dispatch(kNT, 1, M, N, K, A, lda, 0, B, ldb, 0, C, ldc, 0, dtype_ab, dtype_c,
                         alpha, beta, stream);
}

extern "C" int veda_gemm_nn(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda,
                            const void* B, int64_t ldb, void* C, int64_t ldc, int dtype_ab,
                            int dtype_c, float alpha, float beta, veda_stream_t stream)
{
    return gemm_dispatch(kNN, 1, M, N, K, A, lda, 0, B, ldb, 0, C, ldc, 0, dtype_ab, dtype_c,
                         alpha, beta, stream);
}

extern "C" int veda_gemm_tn(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda,
                            const void* B, int64_t ldb, void* C, int64_t ldc, int dtype_ab,
                            int dtype_c, float alpha, float beta, veda_stream_t stream)
{
    return gemm_dispatch(kTN, 1, M, N, K, A, lda, 0, B, ldb, 0, C, ldc, 0, dtype_ab, dtype_c,
                         alpha, beta, stream);
}

extern "C" int veda_gemm_swiglu_fwd(int64_t rows, int64_t F, int64_t D, const void* x, int64_t ldx,
                                    const void* w_gate_up, int64_t ldw, void* gate_up, int64_t ldgu,
                                    void* h, int64_t ldh, veda_stream_t stream)
{
    VEDA_REQUIRE(rows >= 0 && F > 0 && D > 0, "bad shape");
    VEDA_REQUIRE(ldx >= D && ldw >= D && ldgu >= 2 * F && ldh >= F, "leading dimension too small");
    if (rows == 0)
    {
        return VEDA_OK;
    }
    VEDA_REQUIRE(x && w_gate_up && gate_up && h, "null pointer");
    const int rc = gemm_swiglu_fwd_tc(rows, F, D, x, ldx, w_gate_up, ldw, gate_up, ldgu, h, ldh, stream);
    return rc == -1 ? fail(VEDA_ERR_UNSUPPORTED, "veda_gemm_swiglu_fwd: shape or alignment not supported "
                                                 "(F a multiple of 128, rows >= 256, 16-byte rows)")
                    : rc;
}

extern "C" int veda_gemm_swiglu_bwd(int64_t rows, int64_t F, int64_t D, const void* dy, int64_t lddy,
                                    const void* w_down, int64_t ldw, const void* gate_up, int64_t ldgu,
                                    void* dgate_up, int64_t lddgu, veda_stream_t stream)
{
    VEDA_REQUIRE(rows >= 0 && F > 0 && D > 0, "bad shape");
    VEDA_REQUIRE(lddy >= D && ldw >= F && ldgu >= 2 * F && lddgu >= 2 * F, "leading dimension too small");
    if (rows == 0)
    {
        return VEDA_OK;
    }
    VEDA_REQUIRE(dy && w_down && gate_up && dgate_up, "null pointer");
    const int rc =
        gemm_swiglu_bwd_tc(rows, F, D, dy, lddy, w_down, ldw, gate_up, ldgu, dgate_up, lddgu, stream);
    return rc == -1 ? fail(VEDA_ERR_UNSUPPORTED, "veda_gemm_swiglu_bwd: shape or alignment not supported "
                                                 "(F a multiple of 256, rows >= 256, 16-byte rows)")
                    : rc;
}

extern "C" int veda_gemm_batched(int op, int64_t batch, int64_t M, int64_t N, int64_t K,
                                 const void* A, int64_t lda, int64_t stride_a, const void* B,
                                 int64_t ldb, int64_t stride_b, void* C, int64_t ldc,
                                 int64_t stride_c, int dtype_ab, int dtype_c, float alpha,
                                 float beta, veda_stream_t stream)
{
    return gemm_dispatch(op, batch, M, N, K, A, lda, stride_a, B, ldb, stride_b, C, ldc, stride_c,
                         dtype_ab, dtype_c, alpha, beta, stream);
}
