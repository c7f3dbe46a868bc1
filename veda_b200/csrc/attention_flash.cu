// Tiled causal GQA attention on the tensor cores: bf16 operands, fp32 accumulation, head_dim 128.
//
// Forward (one CTA = 64 queries of one (batch, head); 4 warps x 16 query rows):
//   for each 64-key tile up to the diagonal: S = Q K^T (mma m16n8k16), causal mask on the diagonal
//   tile, online softmax in registers (running max and sum in the log2 domain), P (bf16, straight
//   from the accumulators) times V accumulated into O. K/V tiles are double-buffered with cp.async.
//   Writes O (bf16) and LSE = max + log(sum) (fp32), the statistics the backward recomputes P from.
// Backward (one CTA = 64 keys of one (batch, KV head); 4 warps x 16 keys):
//   for each query head of the GQA group and each 64-query tile at or after the diagonal:
//     S^T = K Q^T, P^T = exp(scale S^T - LSE), dP^T = V dO^T, dS^T = P^T (dP^T - D),
//     dV += P^T dO, dK += dS^T Q (registers, summed over the group's heads — deterministic),
//     dQ += dS K (fp32 atomics into a workspace accumulator; scaled and rounded to bf16 after).
//   D = rowsum(dO * O) is computed first by a small kernel.
// This is the composition of src/libs/train/Model.cpp:182-189 (scale after QK^T, -inf causal
// mask, softmax over keys, P V) with kv head h / (H / Hkv) (src/libs/model/Attention.cpp:191);
// the softmax backward P (dP - D) equals NonLinear.cpp:123-133 since sum_j dP_ij P_ij = dO_i . O_i.
#include "attention.cuh"

namespace veda::cuda
{

const bool kFlashReady = true;

namespace
{

constexpr int kDh = 128;
constexpr int kTile = 64;          // queries per forward CTA, keys per backward CTA, key/query tile
constexpr int kLds = kDh + 8;      // padded shared row (272 bytes): conflict-free ldmatrix
constexpr int kTileElems = kTile * kLds;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi)
{
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait()
{
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Stages rows [row0, row0 + 64) of one head (head_dim 128) of a token-major [B*T, ld] operand into
// a padded shared tile; rows at or past T are zero-filled.
__device__ __forceinline__ void load_tile(bf16* dst, const bf16* base, int64_t ld, int64_t b,
                                          int64_t T, int64_t row0, int64_t col0)
{
#pragma unroll
    for (int k = 0; k < 8; ++k)
    {
        const int c = threadIdx.x + 128 * k;
        const int r = c >> 4;
        const int c16 = c & 15;
        const int64_t row = row0 + r;
        const bool valid = row < T;
        const bf16* src = valid ? base + (b * T + row) * ld + col0 + c16 * 8 : base;
        cp_async16(dst + r * kLds + c16 * 8, src, valid);
    }
}

// A fragments (16 rows x 16 cols) of a row-major shared tile at (r0, c0).
__device__ __forceinline__ void frag_a(const bf16* tile, int r0, int c0, uint32_t (&a)[4])
{
    const int i = threadIdx.x & 31;
    const bf16* p = tile + (r0 + (i & 7) + ((i >> 3) & 1) * 8) * kLds + c0 + (i >> 4) * 8;
    ldsm_x4(smem_u32(p), a[0], a[1], a[2], a[3]);
}

// B fragments for two n-tiles (n0..n0+15) and one k-slice (k0..k0+15) when B[k][n] = M[n][k]
// (M row-major by n): {b0, b1} of n-tile 0, then of n-tile 1.
__device__ __forceinline__ void frag_b_nrows(const bf16* tile, int n0, int k0, uint32_t& b00,
                                             uint32_t& b01, uint32_t& b10, uint32_t& b11)
{
    const int i = threadIdx.x & 31;
    const bf16* p = tile + (n0 + (i & 7) + (i >> 4) * 8) * kLds + k0 + ((i >> 3) & 1) * 8;
    ldsm_x4(smem_u32(p), b00, b01, b10, b11);
}

// Same when B[k][n] = M[k][n] (M row-major by k): transposing ldmatrix.
__device__ __forceinline__ void frag_b_krows(const bf16* tile, int ld, int k0, int n0,
                                             uint32_t& b00, uint32_t& b01, uint32_t& b10,
                                             uint32_t& b11)
{
    const int i = threadIdx.x & 31;
    const bf16* p = tile + (k0 + (i & 7) + ((i >> 3) & 1) * 8) * ld + n0 + (i >> 4) * 8;
    ldsm_x4_t(smem_u32(p), b00, b01, b10, b11);
}

// ---------------------------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------------------------
struct FwdArgs
{
    const bf16 *q, *k, *v;
    bf16* o;
    float* lse;
    int64_t ldq, ldk, ldv, ldo;
    int64_t T, H, Hkv;
    float scale_log2;   // scale * log2(e)
    int causal;
};

__global__ void __launch_bounds__(128)
flash_fwd_kernel(const FwdArgs a)
{
    extern __shared__ __align__(16) uint8_t smem_raw[];
    bf16* sq = reinterpret_cast<bf16*>(smem_raw);
    bf16* sk = sq + kTileElems;          // [2][tile]
    bf16* sv = sk + 2 * kTileElems;      // [2][tile]

    const int ntiles = static_cast<int>((a.T + kTile - 1) / kTile);
    const int qt = ntiles - 1 - static_cast<int>(blockIdx.x);   // longest rows first
    const int64_t bh = blockIdx.y;
    const int64_t b = bh / a.H, h = bh % a.H;
    const int64_t kvh = h / (a.H / a.Hkv);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t4 = lane & 3;

    load_tile(sq, a.q, a.ldq, b, a.T, static_cast<int64_t>(qt) * kTile, h * kDh);
    load_tile(sk, a.k, a.ldk, b, a.T, 0, kvh * kDh);
    load_tile(sv, a.v, a.ldv, b, a.T, 0, kvh * kDh);
    cp_async_commit();

    const int last = a.causal ? qt : ntiles - 1;
    uint32_t qf[8][4];
    float o[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
    const int row0 = qt * kTile + warp * 16 + g;   // this thread's rows: row0 and row0 + 8

    for (int kt = 0; kt <= last; ++kt)
    {
        const int buf = kt & 1;
        if (kt + 1 <= last)
        {
            load_tile(sk + (buf ^ 1) * kTileElems, a.k, a.ldk, b, a.T,
                      static_cast<int64_t>(kt + 1) * kTile, kvh * kDh);
            load_tile(sv + (buf ^ 1) * kTileElems, a.v, a.ldv, b, a.T,
                      static_cast<int64_t>(kt + 1) * kTile, kvh * kDh);
            cp_async_commit();
            cp_async_wait<1>();
        }
        else
        {
            cp_async_wait<0>();
        }
        __syncthreads();
        if (kt == 0)
        {
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) frag_a(sq, warp * 16, ks * 16, qf[ks]);
        }
        const bf16* kb = sk + buf * kTileElems;
        const bf16* vb = sv + buf * kTileElems;

        float s[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.0f;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
        {
#pragma unroll
            for (int np = 0; np < 4; ++np)
            {
                uint32_t b00, b01, b10, b11;
                frag_b_nrows(kb, np * 16, ks * 16, b00, b01, b10, b11);
                mma(s[2 * np], qf[ks], b00, b01);
                mma(s[2 * np + 1], qf[ks], b10, b11);
            }
        }
        // scale into the log2 domain and mask
        const bool diag = a.causal && kt == qt;
        const bool tail = static_cast<int64_t>(kt + 1) * kTile > a.T;
        float mx0 = m0, mx1 = m1;
#pragma unroll
        for (int n = 0; n < 8; ++n)
        {
#pragma unroll
            for (int e = 0; e < 4; ++e)
            {
                const int col = kt * kTile + n * 8 + 2 * t4 + (e & 1);
                const int row = row0 + (e >> 1) * 8;
                float v = s[n][e] * a.scale_log2;
                if ((diag && col > row) || (tail && col >= a.T))
                {
                    v = -INFINITY;
                }
                s[n][e] = v;
            }
            mx0 = fmaxf(mx0, fmaxf(s[n][0], s[n][1]));
            mx1 = fmaxf(mx1, fmaxf(s[n][2], s[n][3]));
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xFFFFFFFFu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xFFFFFFFFu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xFFFFFFFFu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xFFFFFFFFu, mx1, 2));
        const float c0 = m0 == -INFINITY ? 0.0f : exp2f(m0 - mx0);
        const float c1 = m1 == -INFINITY ? 0.0f : exp2f(m1 - mx1);
        m0 = mx0;
        m1 = mx1;
        float rs0 = 0.0f, rs1 = 0.0f;
#pragma unroll
        for (int n = 0; n < 8; ++n)
        {
            s[n][0] = mx0 == -INFINITY ? 0.0f : exp2f(s[n][0] - mx0);
            s[n][1] = mx0 == -INFINITY ? 0.0f : exp2f(s[n][1] - mx0);
            s[n][2] = mx1 == -INFINITY ? 0.0f : exp2f(s[n][2] - mx1);
            s[n][3] = mx1 == -INFINITY ? 0.0f : exp2f(s[n][3] - mx1);
            rs0 += s[n][0] + s[n][1];
            rs1 += s[n][2] + s[n][3];
        }
        l0 = l0 * c0 + rs0;
        l1 = l1 * c1 + rs1;
#pragma unroll
        for (int n = 0; n < 16; ++n)
        {
            o[n][0] *= c0;
            o[n][1] *= c0;
            o[n][2] *= c1;
            o[n][3] *= c1;
        }
        // O += P V
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
        {
            uint32_t pa[4];
            pa[0] = pack_bf16(s[2 * ks][0], s[2 * ks][1]);
            pa[1] = pack_bf16(s[2 * ks][2], s[2 * ks][3]);
            pa[2] = pack_bf16(s[2 * ks + 1][0], s[2 * ks + 1][1]);
            pa[3] = pack_bf16(s[2 * ks + 1][2], s[2 * ks + 1][3]);
#pragma unroll
            for (int np = 0; np < 8; ++np)
            {
                uint32_t b00, b01, b10, b11;
                frag_b_krows(vb, kLds, ks * 16, np * 16, b00, b01, b10, b11);
                mma(o[2 * np], pa, b00, b01);
                mma(o[2 * np + 1], pa, b10, b11);
            }
        }
        __syncthreads();   // the buffer is refilled by the next iteration's prefetch
    }
    // finalize: the row sums live across the 4 threads of a quad
    l0 += __shfl_xor_sync(0xFFFFFFFFu, l0, 1);
    l0 += __shfl_xor_sync(0xFFFFFFFFu, l0, 2);
    l1 += __shfl_xor_sync(0xFFFFFFFFu, l1, 1);
    l1 += __shfl_xor_sync(0xFFFFFFFFu, l1, 2);
    const float inv0 = l0 > 0.0f ? 1.0f / l0 : 0.0f;
    const float inv1 = l1 > 0.0f ? 1.0f / l1 : 0.0f;
    const int64_t r0 = row0, r1 = row0 + 8;
#pragma unroll
    for (int n = 0; n < 16; ++n)
    {
        const int col = n * 8 + 2 * t4;
        if (r0 < a.T)
        {
            *reinterpret_cast<uint32_t*>(a.o + (b * a.T + r0) * a.ldo + h * kDh + col) =
                pack_bf16(o[n][0] * inv0, o[n][1] * inv0);
        }
        if (r1 < a.T)
        {
            *reinterpret_cast<uint32_t*>(a.o + (b * a.T + r1) * a.ldo + h * kDh + col) =
                pack_bf16(o[n][2] * inv1, o[n][3] * inv1);
        }
    }
    if (t4 == 0)
    {
        if (r0 < a.T) a.lse[(b * a.H + h) * a.T + r0] = (m0 + log2f(l0)) * kLn2;
        if (r1 < a.T) a.lse[(b * a.H + h) * a.T + r1] = (m1 + log2f(l1)) * kLn2;
    }
}

// ---------------------------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------------------------
// D[b,h,i] = sum_d dO * O (fp32); one warp per row, 16-byte loads.
__global__ void flash_rowdot_kernel(const bf16* __restrict__ o, int64_t ldo,
                                    const bf16* __restrict__ dout, int64_t lddo,
                                    float* __restrict__ dvec, int64_t B, int64_t T, int64_t H)
{
    const int lane = threadIdx.x & 31;
    const int64_t rows = B * H * T;
    for (int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < rows;
         r += (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5)
    {
        const int64_t i = r % T, h = (r / T) % H, b = r / (T * H);
        float x[8], y[8];
        if (lane < 16)
        {
            load16(o + (b * T + i) * ldo + h * kDh + lane * 8, x);
            load16(dout + (b * T + i) * lddo + h * kDh + lane * 8, y);
        }
        float s = 0.0f;
        if (lane < 16)
        {
#pragma unroll
            for (int e = 0; e < 8; ++e) s += x[e] * y[e];
        }
        s = warp_sum(s);
        if (lane == 0) dvec[(b * H + h) * T + i] = s;
    }
}

// dq = bf16(scale * acc)
__global__ void flash_dq_convert_kernel(const float* __restrict__ acc, bf16* __restrict__ dq,
                                        int64_t lddq, int64_t rows, int64_t width, float scale)
{
    const int64_t total = rows * width / 4;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        const int64_t r = (idx * 4) / width, c = (idx * 4) % width;
        const float4 v = reinterpret_cast<const float4*>(acc)[idx];
        uint2 packed;
        packed.x = pack_bf16(v.x * scale, v.y * scale);
        packed.y = pack_bf16(v.z * scale, v.w * scale);
        *reinterpret_cast<uint2*>(dq + r * lddq + c) = packed;
    }
}

struct BwdArgs
{
    const bf16 *q, *k, *v, *dout;
    const float *lse, *dvec;
    float* dq_acc;       // [B*T, H*128] fp32
    bf16 *dk, *dv;
    int64_t ldq, ldk, ldv, lddo, lddk, lddv;
    int64_t T, H, Hkv;
    float scale, scale_log2;
    int causal;
};

__global__ void __launch_bounds__(128, 1)
flash_bwd_kernel(const BwdArgs a)
{
    extern __shared__ __align__(16) uint8_t smem_raw[];
    bf16* sk = reinterpret_cast<bf16*>(smem_raw);
    bf16* sv = sk + kTileElems;
    bf16* sq = sv + kTileElems;         // [2][tile]
    bf16* sdo = sq + 2 * kTileElems;    // [2][tile]
    constexpr int kLdsS = kTile + 8;
    bf16* sds = sdo + 2 * kTileElems;   // dS^T [64 keys][64 + 8 queries]
    float* slse = reinterpret_cast<float*>(sds + kTile * kLdsS);   // [2][64] (log2 units)
    float* sd = slse + 2 * kTile;                                  // [2][64]

    const int kt = static_cast<int>(blockIdx.x);
    const int64_t bk = blockIdx.y;
    const int64_t b = bk / a.Hkv, kvh = bk % a.Hkv;
    const int64_t rep = a.H / a.Hkv;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const int ntiles = static_cast<int>((a.T + kTile - 1) / kTile);
    const int first_qt = a.causal ? kt : 0;

    load_tile(sk, a.k, a.ldk, b, a.T, static_cast<int64_t>(kt) * kTile, kvh * kDh);
    load_tile(sv, a.v, a.ldv, b, a.T, static_cast<int64_t>(kt) * kTile, kvh * kDh);
    cp_async_commit();

    float dk[16][4], dv[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n)
    {
        dk[n][0] = dk[n][1] = dk[n][2] = dk[n][3] = 0.0f;
        dv[n][0] = dv[n][1] = dv[n][2] = dv[n][3] = 0.0f;
    }
    const int key0 = kt * kTile + warp * 16 + g;   // this thread's keys: key0 and key0 + 8

    const int per_head = ntiles - first_qt;
    const int iters = static_cast<int>(rep) * per_head;
    auto issue = [&](int it, int buf) {
        const int64_t h = kvh * rep + it / per_head;
        const int qt = first_qt + it % per_head;
        load_tile(sq + buf * kTileElems, a.q, a.ldq, b, a.T, static_cast<int64_t>(qt) * kTile, h * kDh);
        load_tile(sdo + buf * kTileElems, a.dout, a.lddo, b, a.T, static_cast<int64_t>(qt) * kTile,
                  h * kDh);
        if (threadIdx.x < kTile)
        {
            const int64_t row = static_cast<int64_t>(qt) * kTile + threadIdx.x;
            const bool valid = row < a.T;
            slse[buf * kTile + threadIdx.x] =
                valid ? a.lse[(b * a.H + h) * a.T + row] * kLog2e : INFINITY;
            sd[buf * kTile + threadIdx.x] = valid ? a.dvec[(b * a.H + h) * a.T + row] : 0.0f;
        }
    };
    if (iters > 0)
    {
        issue(0, 0);
    }
    cp_async_commit();

    for (int it = 0; it < iters; ++it)
    {
        const int buf = it & 1;
        const int64_t h = kvh * rep + it / per_head;
        const int qt = first_qt + it % per_head;
        if (it + 1 < iters)
        {
            issue(it + 1, buf ^ 1);
            cp_async_commit();
            cp_async_wait<1>();
        }
        else
        {
            cp_async_wait<0>();
        }
        __syncthreads();
        const bf16* qb = sq + buf * kTileElems;
        const bf16* dob = sdo + buf * kTileElems;
        const float* lb = slse + buf * kTile;
        const float* db = sd + buf * kTile;

        // S^T = K_w Q^T and dP^T = V_w dO^T  (16 keys x 64 queries each)
        float st[8][4], dpt[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n)
        {
            st[n][0] = st[n][1] = st[n][2] = st[n][3] = 0.0f;
            dpt[n][0] = dpt[n][1] = dpt[n][2] = dpt[n][3] = 0.0f;
        }
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
        {
            uint32_t ka[4], va[4];
            frag_a(sk, warp * 16, ks * 16, ka);
            frag_a(sv, warp * 16, ks * 16, va);
#pragma unroll
            for (int np = 0; np < 4; ++np)
            {
                uint32_t b00, b01, b10, b11;
                frag_b_nrows(qb, np * 16, ks * 16, b00, b01, b10, b11);
                mma(st[2 * np], ka, b00, b01);
                mma(st[2 * np + 1], ka, b10, b11);
                frag_b_nrows(dob, np * 16, ks * 16, b00, b01, b10, b11);
                mma(dpt[2 * np], va, b00, b01);
                mma(dpt[2 * np + 1], va, b10, b11);
            }
        }
        // P^T and dS^T; queries are the columns here
        const bool diag = a.causal && qt == kt;
#pragma unroll
        for (int n = 0; n < 8; ++n)
        {
#pragma unroll
            for (int e = 0; e < 4; ++e)
            {
                const int qcol = n * 8 + 2 * t4 + (e & 1);
                const int key = key0 + (e >> 1) * 8;
                const int query = qt * kTile + qcol;
                float p = exp2f(st[n][e] * a.scale_log2 - lb[qcol]);
                if (diag && key > query)
                {
                    p = 0.0f;
                }
                st[n][e] = p;
                dpt[n][e] = p * (dpt[n][e] - db[qcol]);
            }
        }
        // dV += P^T dO ; dK += dS^T Q   (k = queries)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
        {
            uint32_t pa[4], sa[4];
            pa[0] = pack_bf16(st[2 * ks][0], st[2 * ks][1]);
            pa[1] = pack_bf16(st[2 * ks][2], st[2 * ks][3]);
            pa[2] = pack_bf16(st[2 * ks + 1][0], st[2 * ks + 1][1]);
            pa[3] = pack_bf16(st[2 * ks + 1][2], st[2 * ks + 1][3]);
            sa[0] = pack_bf16(dpt[2 * ks][0], dpt[2 * ks][1]);
            sa[1] = pack_bf16(dpt[2 * ks][2], dpt[2 * ks][3]);
            sa[2] = pack_bf16(dpt[2 * ks + 1][0], dpt[2 * ks + 1][1]);
            sa[3] = pack_bf16(dpt[2 * ks + 1][2], dpt[2 * ks + 1][3]);
            // dS^T to shared memory for the dQ product: rows = keys, cols = queries
            bf16* srow0 = sds + (warp * 16 + g) * kLdsS + ks * 16 + 2 * t4;
            bf16* srow1 = srow0 + 8 * kLdsS;
            *reinterpret_cast<uint32_t*>(srow0) = sa[0];
            *reinterpret_cast<uint32_t*>(srow1) = sa[1];
            *reinterpret_cast<uint32_t*>(srow0 + 8) = sa[2];
            *reinterpret_cast<uint32_t*>(srow1 + 8) = sa[3];
#pragma unroll
            for (int np = 0; np < 8; ++np)
            {
                uint32_t b00, b01, b10, b11;
                frag_b_krows(dob, kLds, ks * 16, np * 16, b00, b01, b10, b11);
                mma(dv[2 * np], pa, b00, b01);
                mma(dv[2 * np + 1], pa, b10, b11);
                frag_b_krows(qb, kLds, ks * 16, np * 16, b00, b01, b10, b11);
                mma(dk[2 * np], sa, b00, b01);
                mma(dk[2 * np + 1], sa, b10, b11);
            }
        }
        __syncthreads();
        // dQ (queries 16w..16w+15 of this tile) += dS K : A = dS from the transposed shared copy
        {
            float dq[16][4];
#pragma unroll
            for (int n = 0; n < 16; ++n) dq[n][0] = dq[n][1] = dq[n][2] = dq[n][3] = 0.0f;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)   // keys 16ks..16ks+15
            {
                uint32_t da[4];
                {
                    const int i = lane;
                    const bf16* p = sds + (ks * 16 + (i & 7) + (i >> 4) * 8) * kLdsS + warp * 16 +
                                    ((i >> 3) & 1) * 8;
                    ldsm_x4_t(smem_u32(p), da[0], da[1], da[2], da[3]);
                }
#pragma unroll
                for (int np = 0; np < 8; ++np)
                {
                    uint32_t b00, b01, b10, b11;
                    frag_b_krows(sk, kLds, ks * 16, np * 16, b00, b01, b10, b11);
                    mma(dq[2 * np], da, b00, b01);
                    mma(dq[2 * np + 1], da, b10, b11);
                }
            }
            const int64_t q0 = static_cast<int64_t>(qt) * kTile + warp * 16 + g;
            const int64_t width = a.H * kDh;
#pragma unroll
            for (int n = 0; n < 16; ++n)
            {
                const int64_t col = h * kDh + n * 8 + 2 * t4;
                if (q0 < a.T)
                {
                    atomicAdd(reinterpret_cast<float2*>(a.dq_acc + (b * a.T + q0) * width + col),
                              make_float2(dq[n][0], dq[n][1]));
                }
                if (q0 + 8 < a.T)
                {
                    atomicAdd(reinterpret_cast<float2*>(a.dq_acc + (b * a.T + q0 + 8) * width + col),
                              make_float2(dq[n][2], dq[n][3]));
                }
            }
        }
        __syncthreads();   // sds and this buffer are rewritten next iteration
    }
    // write dK (scaled) and dV
    const int64_t k0 = key0, k1 = key0 + 8;
#pragma unroll
    for (int n = 0; n < 16; ++n)
    {
        const int col = n * 8 + 2 * t4;
        if (k0 < a.T)
        {
            *reinterpret_cast<uint32_t*>(a.dk + (b * a.T + k0) * a.lddk + kvh * kDh + col) =
                pack_bf16(dk[n][0] * a.scale, dk[n][1] * a.scale);
            *reinterpret_cast<uint32_t*>(a.dv + (b * a.T + k0) * a.lddv + kvh * kDh + col) =
                pack_bf16(dv[n][0], dv[n][1]);
        }
        if (k1 < a.T)
        {
            *reinterpret_cast<uint32_t*>(a.dk + (b * a.T + k1) * a.lddk + kvh * kDh + col) =
                pack_bf16(dk[n][2] * a.scale, dk[n][3] * a.scale);
            *reinterpret_cast<uint32_t*>(a.dv + (b * a.T + k1) * a.lddv + kvh * kDh + col) =
                pack_bf16(dv[n][2], dv[n][3]);
        }
    }
}

constexpr size_t kFwdSmem = 5 * kTileElems * sizeof(bf16);
constexpr size_t kBwdSmem = 6 * kTileElems * sizeof(bf16) + kTile * (kTile + 8) * sizeof(bf16) +
                            4 * kTile * sizeof(float);

} // namespace

size_t flash_bwd_extra_workspace(int64_t B, int64_t T, int64_t H, int64_t, int64_t)
{
    return static_cast<size_t>(B * T * H * kDh) * sizeof(float);
}

int flash_fwd(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
              void* o, int64_t ldo, float* lse, int64_t B, int64_t T, int64_t H, int64_t Hkv,
              float scale, int causal, cudaStream_t s)
{
    VEDA_REQUIRE(B * H <= 65535 * 64, "too many (batch, head) pairs");
    static int configured = -1;
    int device = 0;
    cudaGetDevice(&device);
    if (configured != device)
    {
        cudaFuncSetAttribute(flash_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kFwdSmem));
        configured = device;
    }
    FwdArgs a{static_cast<const bf16*>(q), static_cast<const bf16*>(k), static_cast<const bf16*>(v),
              static_cast<bf16*>(o), lse, ldq, ldk, ldv, ldo, T, H, Hkv, scale * kLog2e, causal};
    const dim3 grid(static_cast<unsigned>((T + kTile - 1) / kTile), static_cast<unsigned>(B * H));
    flash_fwd_kernel<<<grid, 128, kFwdSmem, s>>>(a);
    count_launch();
    return check_launch("veda_attention_fwd (tiled)");
}

int flash_bwd(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
              const void* o, int64_t ldo, const void* dout, int64_t lddo, const float* lse,
              void* dq, int64_t lddq, void* dk, int64_t lddk, void* dv, int64_t lddv, float* dvec,
              void* extra, int64_t B, int64_t T, int64_t H, int64_t Hkv, float scale, int causal,
              cudaStream_t s)
{
    static int configured = -1;
    int device = 0;
    cudaGetDevice(&device);
    if (configured != device)
    {
        cudaFuncSetAttribute(flash_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kBwdSmem));
        configured = device;
    }
    float* acc = static_cast<float*>(extra);
    const int64_t width = H * kDh;
    if (cudaMemsetAsync(acc, 0, static_cast<size_t>(B * T * width) * sizeof(float), s) != cudaSuccess)
    {
        return fail(VEDA_ERR_CUDA, "veda_attention_bwd: clearing the dQ accumulator failed");
    }
    flash_rowdot_kernel<<<grid_for(B * H * T * 32, 256), 256, 0, s>>>(
        static_cast<const bf16*>(o), ldo, static_cast<const bf16*>(dout), lddo, dvec, B, T, H);
    BwdArgs a{static_cast<const bf16*>(q), static_cast<const bf16*>(k), static_cast<const bf16*>(v),
              static_cast<const bf16*>(dout), lse, dvec, acc, static_cast<bf16*>(dk),
              static_cast<bf16*>(dv), ldq, ldk, ldv, lddo, lddk, lddv, T, H, Hkv, scale,
              scale * kLog2e, causal};
    const dim3 grid(static_cast<unsigned>((T + kTile - 1) / kTile), static_cast<unsigned>(B * Hkv));
    flash_bwd_kernel<<<grid, 128, kBwdSmem, s>>>(a);
    flash_dq_convert_kernel<<<grid_for(B * T * width / 4, 256), 256, 0, s>>>(
        acc, static_cast<bf16*>(dq), lddq, B * T, width, scale);
    count_launch(3);
    return check_launch("veda_attention_bwd (tiled)");
}

} // namespace veda::cuda
