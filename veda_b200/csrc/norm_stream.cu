// Streaming RMSNorm forward and backward (bf16 rows of 256..2048 elements).
//
// Same arithmetic as the row kernels of norm.cu (src/libs/ops/Normalize.cpp:50-63,
// src/libs/autograd/NonLinear.cpp:171-196; the gain through Variable.cpp:218-239): fp32 sums,
// r = sqrt(sum x^2 / n + eps), y = x / r * gamma; dx = G / r - x * sum(G x) / (n r^3) (+ the
// residual gradient), G = dy * gamma, dgamma = sum over rows of dy * x / r.
//
// Structure: one block per SM, 1 producer warp + consumer warps. The producer's lane 0 streams
// whole rows (x; for the backward also dy and the residual gradient) into a ring of shared-memory
// stages with bulk asynchronous copies (cp.async.bulk, no tensor map, no multicast) completing on
// the stage's mbarrier; a stage holds 8 rows. Consumers wait for their stage, reduce their row
// with warp shuffles, write the output row with coalesced 16-byte stores and release the stage.
// With 128-192 KB of rows in flight per SM the loads no longer wait on the arithmetic, which is
// what the register-resident kernels could not reach. Every mbarrier wait is bounded
// (tc_common.cuh).
//   forward:  8 consumer warps, one row each;
//   backward: rows of 512 or more elements are split between two warps (16 consumer warps, one
//             half-row each; the two halves' sums meet through shared memory and a named barrier
//             per row, added in the same order by both warps), with the arithmetic on packed fp32
//             pairs. Eight warps each working through a whole row left the schedulers idle on the
//             dependent sums (2.3 warps per scheduler, an instruction every 3.4 cycles, DRAM 35 %
//             busy at 8192 x 1024).
//
// The gain gradient: each consumer warp accumulates its lanes' columns over the rows it processed;
// at the end the warps' rows are summed in row-slot order into one partial row per block (the
// caller then sums the block partials in block order) — deterministic. Summing the block partials
// inside this kernel instead (the last blocks to finish, after a memory fence and a completion
// count) measured 19.9 us a call at 8192 x 1024 against 16.3 us for the two launches: the fence
// waits for the block's output rows to drain, at the end of every block.
#include "norm_stream.cuh"
#include "tc_common.cuh"

namespace veda::cuda
{
int* device_status_ptr();

namespace
{
using namespace tc;

constexpr int kRows = 8;                       // rows per stage = consumer warps
constexpr int kThreadsStream = 32 * (1 + kRows);
constexpr int kRingBytes = 192 * 1024;         // shared-memory ring per block

template <int CH, int NIN>
struct Ring
{
    static constexpr int N = CH * 256;                 // elements per row
    static constexpr int ROW = N * 2;                  // bytes per bf16 row
    static constexpr int STAGE = kRows * NIN * ROW;    // bytes per stage
    static constexpr int STAGES = kRingBytes / STAGE < 8 ? kRingBytes / STAGE : 8;
    // ring | gamma as fp32 [N] | barriers | abort flag, plus alignment slack
    static constexpr int SMEM = STAGES * STAGE + N * 4 + 2 * STAGES * 8 + 16 + 128;
    static_assert(STAGES >= 2, "ring too small");
};

__device__ __forceinline__ void unpack8(const uint4& raw, float (&o)[8])
{
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        o[2 * i] = __uint_as_float(w[i] << 16);
        o[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

// Producer: streams NIN input rows per row of each of this block's chunks of kRows rows.
template <int CH, int NIN>
__device__ __forceinline__ void produce(uint8_t* ring, uint64_t* full, uint64_t* empty,
                                        const bf16* s0, int64_t ld0, const bf16* s1, int64_t ld1,
                                        const bf16* s2, int64_t ld2, int64_t rows, int* status,
                                        volatile int* abort)
{
    using R = Ring<CH, NIN>;
    const int64_t chunks = (rows + kRows - 1) / kRows;
    int i = 0;
    for (int64_t q = blockIdx.x; q < chunks; q += gridDim.x, ++i)
    {
        const int st = i % R::STAGES;
        mbar_wait(&empty[st], ((i / R::STAGES) & 1) ^ 1, status, abort);
        const int64_t r0 = q * kRows;
        const int nr = static_cast<int>(rows - r0 < kRows ? rows - r0 : kRows);
        mbar_expect_tx(&full[st], static_cast<uint32_t>(nr * NIN * R::ROW));
        uint8_t* dst = ring + st * R::STAGE;
        for (int r = 0; r < nr; ++r)
        {
            bulk_load(dst + (r * NIN) * R::ROW, s0 + (r0 + r) * ld0, R::ROW, &full[st]);
            if constexpr (NIN >= 2)
            {
                bulk_load(dst + (r * NIN + 1) * R::ROW, s1 + (r0 + r) * ld1, R::ROW, &full[st]);
            }
            if constexpr (NIN >= 3)
            {
                bulk_load(dst + (r * NIN + 2) * R::ROW, s2 + (r0 + r) * ld2, R::ROW, &full[st]);
            }
        }
    }
}

// NIN = 2: the rows normalised are s = x + r (rounded to bf16, as the residual add stores it),
// and s is written out as well.
template <int CH, int NIN>
__global__ void __launch_bounds__(kThreadsStream, 1)
rms_fwd_stream_kernel(const bf16* __restrict__ x, int64_t ldx, const bf16* __restrict__ r, int64_t ldr,
                      const bf16* __restrict__ gamma, bf16* __restrict__ y, int64_t ldy,
                      bf16* __restrict__ sum, int64_t lds, int64_t rows, float eps, int* status)
{
    using R = Ring<CH, NIN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~static_cast<uintptr_t>(127));
    float* gsm = reinterpret_cast<float*>(ring + R::STAGES * R::STAGE);   // gamma, fp32
    uint64_t* full = reinterpret_cast<uint64_t*>(gsm + R::N);
    uint64_t* empty = full + R::STAGES;
    volatile int* abort = reinterpret_cast<volatile int*>(empty + R::STAGES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0)
    {
        *abort = 0;
        for (int s = 0; s < R::STAGES; ++s)
        {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kRows);
        }
        mbar_fence_init();
    }
    dep_wait();   // the rows (and the gain) belong to the kernels before this one
    dep_release();
    for (int c = threadIdx.x; c < R::N; c += blockDim.x)
    {
        gsm[c] = gamma != nullptr ? __bfloat162float(gamma[c]) : 1.0f;
    }
    __syncthreads();
    if (warp == 0)
    {
        if (lane == 0)
        {
            produce<CH, NIN>(ring, full, empty, x, ldx, r, ldr, nullptr, 0, rows, status, abort);
        }
        return;
    }
    const int w = warp - 1;
    const int64_t chunks = (rows + kRows - 1) / kRows;
    int i = 0;
    for (int64_t q = blockIdx.x; q < chunks; q += gridDim.x, ++i)
    {
        const int st = i % R::STAGES;
        mbar_wait(&full[st], (i / R::STAGES) & 1, status, abort);
        const int64_t row = q * kRows + w;
        if (row < rows)
        {
            const uint8_t* src = ring + st * R::STAGE + w * NIN * R::ROW;
            uint4 xr[CH];
#pragma unroll
            for (int c = 0; c < CH; ++c) xr[c] = *reinterpret_cast<const uint4*>(src + (c * 32 + lane) * 16);
            if constexpr (NIN == 2)
            {
#pragma unroll
                for (int c = 0; c < CH; ++c)
                {
                    const uint4 rr = *reinterpret_cast<const uint4*>(src + R::ROW + (c * 32 + lane) * 16);
                    float a[8], b[8];
                    unpack8(xr[c], a);
                    unpack8(rr, b);
                    uint32_t w4[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                    {
                        const __nv_bfloat162 t = __floats2bfloat162_rn(a[2 * j] + b[2 * j], a[2 * j + 1] + b[2 * j + 1]);
                        w4[j] = *reinterpret_cast<const uint32_t*>(&t);
                    }
                    xr[c] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                    *reinterpret_cast<uint4*>(sum + row * lds + (c * 32 + lane) * 8) = xr[c];
                }
            }
            float ss = 0.0f;
#pragma unroll
            for (int c = 0; c < CH; ++c)
            {
                float v[8];
                unpack8(xr[c], v);
#pragma unroll
                for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
            }
            ss = warp_sum(ss);
            const float inv = 1.0f / sqrtf(ss / static_cast<float>(R::N) + eps);
#pragma unroll
            for (int c = 0; c < CH; ++c)
            {
                float v[8];
                unpack8(xr[c], v);
                const float4 g0 = *reinterpret_cast<const float4*>(gsm + (c * 32 + lane) * 8);
                const float4 g1 = *reinterpret_cast<const float4*>(gsm + (c * 32 + lane) * 8 + 4);
                const float gm[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = (v[j] * inv) * gm[j];
                store16(y + row * ldy + (c * 32 + lane) * 8, v);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
}

// Backward layout: rows of 512 or more elements are shared by two consumer warps (one half
// each), so 16 consumer warps keep the schedulers busy where 8 could not hide the latency of
// their dependent reductions; rows of 256 keep one warp per row.
template <int CH>
struct BwdSplit
{
    static constexpr int SPLIT = CH >= 2 ? 2 : 1;     // warps per row
    static constexpr int CW = CH / SPLIT;             // 16-byte chunks per lane
    static constexpr int WARPS = kRows * SPLIT;       // consumer warps
    static constexpr int THREADS = 32 * (1 + WARPS);
};

template <int CH, int NIN>
struct BwdSmem
{
    using R = Ring<CH, NIN>;
    // ring | gain (bf16 [N]) | row-half sums [2][kRows][SPLIT] float2 | barriers | abort flag,
    // plus alignment slack
    static constexpr int SMEM = R::STAGES * R::STAGE + R::N * 2 + 2 * kRows * BwdSplit<CH>::SPLIT * 8 +
                                2 * R::STAGES * 8 + 16 + 128;
};

template <int CH, int NIN>
__global__ void __launch_bounds__(BwdSplit<CH>::THREADS, 1)
rms_bwd_stream_kernel(const bf16* __restrict__ x, int64_t ldx, const bf16* __restrict__ gamma,
                      const bf16* __restrict__ dy, int64_t lddy, const bf16* __restrict__ dresid,
                      int64_t ldr, bf16* __restrict__ dx, int64_t lddx, float* __restrict__ partials,
                      int64_t rows, float eps, int* status)
{
    using R = Ring<CH, NIN>;
    using S = BwdSplit<CH>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~static_cast<uintptr_t>(127));
    uint4* gsm = reinterpret_cast<uint4*>(ring + R::STAGES * R::STAGE);      // gain, bf16
    float2* xch = reinterpret_cast<float2*>(gsm + R::N / 8);                 // [2][kRows][SPLIT]
    uint64_t* full = reinterpret_cast<uint64_t*>(xch + 2 * kRows * S::SPLIT);
    uint64_t* empty = full + R::STAGES;
    volatile int* abort = reinterpret_cast<volatile int*>(empty + R::STAGES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0)
    {
        *abort = 0;
        for (int s = 0; s < R::STAGES; ++s)
        {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], S::WARPS);
        }
        mbar_fence_init();
    }
    dep_wait();   // the rows (and the gain) belong to the kernels before this one
    dep_release();
    for (int c = threadIdx.x; c < R::N / 8; c += blockDim.x)
    {
        // 1.0 in bf16 is 0x3F80
        gsm[c] = gamma != nullptr ? reinterpret_cast<const uint4*>(gamma)[c]
                                  : make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);
    }
    __syncthreads();
    constexpr int kPart = R::N / S::SPLIT;   // elements of a row per consumer warp
    const int w = warp - 1;
    const int r = w % kRows, hf = w / kRows;   // row of the stage, part of the row
    const int col0 = hf * kPart;
    uint64_t acc[S::CW][4];                    // gain gradient of this lane's columns
#pragma unroll
    for (int c = 0; c < S::CW; ++c)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[c][j] = 0;
    if (warp == 0)
    {
        if (lane == 0)
        {
            produce<CH, NIN>(ring, full, empty, x, ldx, dy, lddy, dresid, ldr, rows, status, abort);
        }
    }
    else
    {
        // this lane's 16-byte chunks of the gain (conflict-free: consecutive lanes, consecutive chunks)
        const uint4* gl = gsm + col0 / 8 + lane;
        const int64_t chunks = (rows + kRows - 1) / kRows;
        int i = 0;
        for (int64_t q = blockIdx.x; q < chunks; q += gridDim.x, ++i)
        {
            const int st = i % R::STAGES;
            mbar_wait(&full[st], (i / R::STAGES) & 1, status, abort);
            const int64_t row = q * kRows + r;
            if (row < rows)   // the same for both warps of a row
            {
                const uint8_t* xs = ring + st * R::STAGE + (r * NIN) * R::ROW + col0 * 2;
                const uint8_t* gs = xs + R::ROW;
                uint4 xr[S::CW], gr[S::CW];
#pragma unroll
                for (int c = 0; c < S::CW; ++c)
                {
                    xr[c] = *reinterpret_cast<const uint4*>(xs + (c * 32 + lane) * 16);
                    gr[c] = *reinterpret_cast<const uint4*>(gs + (c * 32 + lane) * 16);
                }
                // G = dy * gamma; sums of x^2 and G x over this warp's part of the row
                uint64_t ss2 = 0, ws2 = 0;
#pragma unroll
                for (int c = 0; c < S::CW; ++c)
                {
                    uint64_t xv[4], gv[4], gm[4];
                    unpack4x2(xr[c], xv);
                    unpack4x2(gr[c], gv);
                    unpack4x2(gl[c * 32], gm);
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                    {
                        ss2 = fma2(xv[j], xv[j], ss2);
                        ws2 = fma2(mul2(gv[j], gm[j]), xv[j], ws2);
                    }
                }
                float s0, s1, w0, w1;
                upk(ss2, s0, s1);
                upk(ws2, w0, w1);
                float ss = s0 + s1, wsum = w0 + w1;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1)
                {
                    ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
                    wsum += __shfl_xor_sync(0xFFFFFFFFu, wsum, o);
                }
                if constexpr (S::SPLIT == 2)
                {
                    // both warps of the row add the two halves in the same order
                    float2* slot = xch + ((i & 1) * kRows + r) * 2;
                    if (lane == 0) slot[hf] = make_float2(ss, wsum);
                    asm volatile("bar.sync %0, 64;" ::"r"(1 + r) : "memory");
                    const float2 a = slot[0], b = slot[1];
                    ss = a.x + b.x;
                    wsum = a.y + b.y;
                }
                const float inv = 1.0f / sqrtf(ss / static_cast<float>(R::N) + eps);
                const float coupling = wsum * inv * inv * inv / static_cast<float>(R::N);
                const uint64_t inv2 = pk(inv, inv), ncp2 = pk(-coupling, -coupling);
#pragma unroll
                for (int c = 0; c < S::CW; ++c)
                {
                    uint64_t xv[4], gv[4], gm[4];
                    unpack4x2(xr[c], xv);
                    unpack4x2(gr[c], gv);
                    unpack4x2(gl[c * 32], gm);
                    uint64_t res[4];
                    if constexpr (NIN == 3)
                    {
                        unpack4x2(*reinterpret_cast<const uint4*>(xs + 2 * R::ROW + (c * 32 + lane) * 16), res);
                    }
                    float out[8];
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                    {
                        // dx = G / r - x * coupling (+ the residual gradient); dgamma += dy * x / r
                        uint64_t d = fma2(mul2(gv[j], gm[j]), inv2, mul2(xv[j], ncp2));
                        if constexpr (NIN == 3)
                        {
                            d = add2(res[j], d);
                        }
                        acc[c][j] = fma2(gv[j], mul2(xv[j], inv2), acc[c][j]);
                        upk(d, out[2 * j], out[2 * j + 1]);
                    }
                    store16(dx + row * lddx + col0 + (c * 32 + lane) * 8, out);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
        }
    }
    if (partials != nullptr)
    {
        // every stage has been consumed and no copy is in flight: reuse the ring for the sums
        __syncthreads();
        float* part = reinterpret_cast<float*>(ring);   // [kRows][N]
        if (warp > 0)
        {
#pragma unroll
            for (int c = 0; c < S::CW; ++c)
            {
                float v[8];
#pragma unroll
                for (int j = 0; j < 4; ++j) upk(acc[c][j], v[2 * j], v[2 * j + 1]);
                float* dst = part + r * R::N + col0 + (c * 32 + lane) * 8;
                *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
                *reinterpret_cast<float4*>(dst + 4) = make_float4(v[4], v[5], v[6], v[7]);
            }
        }
        __syncthreads();
        for (int col = threadIdx.x; col < R::N; col += blockDim.x)
        {
            float s = 0.0f;
#pragma unroll
            for (int k = 0; k < kRows; ++k) s += part[k * R::N + col];
            partials[static_cast<size_t>(blockIdx.x) * R::N + col] = s;
        }
    }
}

bool rows_aligned(const void* p, int64_t ld) { return aligned16(p) && ld % 8 == 0; }

template <int CH, int NIN>
int launch_fwd(const bf16* x, int64_t ldx, const bf16* r, int64_t ldr, const bf16* gamma, bf16* y,
               int64_t ldy, bf16* sum, int64_t lds, int64_t rows, float eps, cudaStream_t s)
{
    using R = Ring<CH, NIN>;
    static int configured = -1;
    int device = 0;
    cudaGetDevice(&device);
    if (configured != device)
    {
        cudaFuncSetAttribute(rms_fwd_stream_kernel<CH, NIN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             R::SMEM);
        configured = device;
    }
    const int64_t chunks = (rows + kRows - 1) / kRows;
    const unsigned grid = static_cast<unsigned>(chunks < compute_sms() ? chunks : compute_sms());
    return launch("veda_rmsnorm_fwd (streaming)", rms_fwd_stream_kernel<CH, NIN>, dim3(grid),
                  dim3(kThreadsStream), R::SMEM, s, x, ldx, r, ldr, gamma, y, ldy, sum, lds, rows, eps,
                  device_status_ptr());
}

template <int CH, int NIN>
int launch_bwd(const bf16* x, int64_t ldx, const bf16* gamma, const bf16* dy, int64_t lddy,
               const bf16* dresid, int64_t ldr, bf16* dx, int64_t lddx, float* partials, int max_blocks,
               int64_t rows, float eps, cudaStream_t s, int* blocks)
{
    constexpr int kSmem = BwdSmem<CH, NIN>::SMEM;
    static int configured = -1;
    int device = 0;
    cudaGetDevice(&device);
    if (configured != device)
    {
        cudaFuncSetAttribute(rms_bwd_stream_kernel<CH, NIN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmem);
        configured = device;
    }
    const int64_t chunks = (rows + kRows - 1) / kRows;
    int64_t g = chunks < compute_sms() ? chunks : compute_sms();
    if (g > max_blocks) g = max_blocks;
    if (g < 1) g = 1;
    *blocks = static_cast<int>(g);
    return launch("veda_rmsnorm_bwd (streaming)", rms_bwd_stream_kernel<CH, NIN>,
                  dim3(static_cast<unsigned>(g)), dim3(BwdSplit<CH>::THREADS), kSmem, s, x, ldx, gamma,
                  dy, lddy, dresid, ldr, dx, lddx, partials, rows, eps, device_status_ptr());
}

} // namespace

int rms_fwd_stream(const bf16* x, int64_t ldx, const bf16* r, int64_t ldr, const bf16* gamma,
                   bf16* y, int64_t ldy, bf16* sum, int64_t lds, int64_t rows, int64_t n, float eps,
                   cudaStream_t s)
{
    if (!rows_aligned(x, ldx) || !rows_aligned(y, ldy) || (gamma != nullptr && !aligned16(gamma)))
    {
        return -1;
    }
    if (r != nullptr)
    {
        if (sum == nullptr || !rows_aligned(r, ldr) || !rows_aligned(sum, lds))
        {
            return -1;
        }
        switch (n)
        {
        case 256: return launch_fwd<1, 2>(x, ldx, r, ldr, gamma, y, ldy, sum, lds, rows, eps, s);
        case 512: return launch_fwd<2, 2>(x, ldx, r, ldr, gamma, y, ldy, sum, lds, rows, eps, s);
        case 1024: return launch_fwd<4, 2>(x, ldx, r, ldr, gamma, y, ldy, sum, lds, rows, eps, s);
        case 2048: return launch_fwd<8, 2>(x, ldx, r, ldr, gamma, y, ldy, sum, lds, rows, eps, s);
        default: return -1;
        }
    }
    switch (n)
    {
    case 256: return launch_fwd<1, 1>(x, ldx, nullptr, 0, gamma, y, ldy, nullptr, 0, rows, eps, s);
    case 512: return launch_fwd<2, 1>(x, ldx, nullptr, 0, gamma, y, ldy, nullptr, 0, rows, eps, s);
    case 1024: return launch_fwd<4, 1>(x, ldx, nullptr, 0, gamma, y, ldy, nullptr, 0, rows, eps, s);
    case 2048: return launch_fwd<8, 1>(x, ldx, nullptr, 0, gamma, y, ldy, nullptr, 0, rows, eps, s);
    default: return -1;
    }
}

int rms_bwd_stream(const bf16* x, int64_t ldx, const bf16* gamma, const bf16* dy, int64_t lddy,
                   const bf16* dresid, int64_t ldr, bf16* dx, int64_t lddx, float* partials,
                   int max_blocks, int64_t rows, int64_t n, float eps, cudaStream_t s, int* blocks)
{
    if (!rows_aligned(x, ldx) || !rows_aligned(dy, lddy) || !rows_aligned(dx, lddx) ||
        (dresid != nullptr && !rows_aligned(dresid, ldr)) || (gamma != nullptr && !aligned16(gamma)))
    {
        return -1;
    }
#define VEDA_BWD(CH)                                                                              \
    return dresid != nullptr                                                                      \
               ? launch_bwd<CH, 3>(x, ldx, gamma, dy, lddy, dresid, ldr, dx, lddx, partials,       \
                                   max_blocks, rows, eps, s, blocks)                              \
               : launch_bwd<CH, 2>(x, ldx, gamma, dy, lddy, dresid, ldr, dx, lddx, partials,       \
                                   max_blocks, rows, eps, s, blocks)
    switch (n)
    {
    case 256: VEDA_BWD(1);
    case 512: VEDA_BWD(2);
    case 1024: VEDA_BWD(4);
    default: return -1;   // 2048: the per-lane gain sums would not fit in registers
    }
#undef VEDA_BWD
}

} // namespace veda::cuda
