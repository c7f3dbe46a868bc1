// Causal GQA attention on the 5th-generation tensor cores (tcgen05.mma, TMEM), bf16, head_dim 128.
//
// Same semantics as the warp-per-row kernels of attention.cu (the composition of
// src/libs/train/Model.cpp:182-189 with kv head h / (H/Hkv), src/libs/model/Attention.cpp:191);
// this file is the bf16, head_dim-128 tensor-core form the entry points dispatch to.
//
// Forward — persistent, one CTA per SM; a work item is one (batch, head, pair of 128-query tiles
// A and B), pairs with the longest causal rows first, handed out in rounds of one item per CTA
// whose direction over the CTAs alternates (round r gives CTA c item r G + c for even r and
// r G + G - 1 - c for odd r, G CTAs), so the long items of one round and the shorter ones of the
// next even out per CTA. Against one CTA per item this took B4 T2048 from 0.099 to 0.094 ms and
// B8 T2048 from 0.178 to 0.170 ms (plain round robin, r G + c for every r, was slower than one
// CTA per item: 0.108 ms). The rings and barrier phases run on across a CTA's items, and the next
// item's Q tiles load once the last S products of the current one have read them. 10 warps:
//   warp 0     TMA (lane 0: both Q tiles, then 128-key K tiles; lane 1: the V tiles), each into
//              its own 2-stage ring shared by the two query tiles (3-D tensor maps [B, T, columns],
//              so rows past T read as zeros; no multicast);
//   warp 1     MMA issuer, ping-pong between the query tiles: per key tile j it issues
//              O_A += P_A V_j, S_A = Q_A K_{j+1}^T, O_B += P_B V_j, S_B = Q_B K_{j+1}^T
//              (M128 N128 K128 each; S, P and O all in TMEM, P read by the MMA straight from
//              tensor memory), so the tensor core computes one tile's products while the softmax
//              warps of the other work;
//   warps 2-5  softmax of tile A, warps 6-9 of tile B: thread i owns query row i (TMEM lane i):
//              loads its S row, masks, keeps a running max in the log2 domain and rescales O in
//              TMEM only when the max grows by more than 2^8 (otherwise the stale max is kept;
//              every exponent stays below 2^8), writes P (bf16 pairs) over the first half of its
//              S columns, and at the end writes O / l and LSE = (m + log2 l) ln 2.
// Every mbarrier wait is bounded (see tc_common.cuh).
#include "attention.cuh"
#include "tc_common.cuh"

#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <mutex>

namespace veda::cuda
{
int* device_status_ptr();

namespace
{
using namespace tc;

constexpr int kTq = 128;                 // queries per CTA
constexpr int kTk = 128;                 // keys per tile
constexpr int kTileBytes = 128 * 128 * 2;   // a [128 rows x 128 dims] bf16 tile (two 16 KB halves)
constexpr int kHalf = kTileBytes / 2;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;   // log2 units

struct FwdParams
{
    bf16* o;
    float* lse;
    int64_t ldo;
    int B, T, H, Hkv;
    float scale_log2;
    int causal;
    int* status;
};

__device__ __forceinline__ void load_tile_3d(uint8_t* dst, const CUtensorMap* map, uint64_t* bar,
                                             int col, int row, int batch)
{
    tma_load_3d(dst, map, bar, col, row, batch);
    tma_load_3d(dst + kHalf, map, bar, col + 64, row, batch);
}

// K-major [128 x 128] operand, k-step ks (16 elements) of the 128-wide K dimension.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int ks)
{
    return smem_desc(base + (ks >> 2) * kHalf + (ks & 3) * 32, 16, 1024);
}

// MN-major operand whose rows are the K dimension (16 rows per k-step) and whose 128 MN columns
// are two 64-column halves kHalf bytes apart.
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int ks, uint32_t lbo)
{
    return smem_desc(base + ks * 2048, lbo, 1024);
}

// smem: Q[2] | K[2] | V[2] | barriers
constexpr int kFwdThreads = 320;
constexpr int kFwdSmem = 1024 + kTileBytes * 6 + 256;

__device__ __forceinline__ uint64_t f2_pack(float a, float b)
{
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b)
{
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c)
{
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b)
{
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// 2^x with the hardware approximation (relative error far below bf16 rounding; -inf -> 0)
__device__ __forceinline__ float ex2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float max3(float a, float b, float c)
{
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

__global__ void __launch_bounds__(kFwdThreads, 1)
attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, const FwdParams p)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* sq = smem;                      // [2]: the pair's two query tiles
    uint8_t* sk = sq + 2 * kTileBytes;       // [2]
    uint8_t* sv = sk + 2 * kTileBytes;       // [2]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sv + 2 * kTileBytes);
    uint64_t* q_full = bars + 0;
    uint64_t* k_full = bars + 1;     // [2] ring stages
    uint64_t* k_empty = bars + 3;    // [2]
    uint64_t* v_full = bars + 5;     // [2]
    uint64_t* v_empty = bars + 7;    // [2]
    uint64_t* s_full = bars + 9;     // [2] per query tile
    uint64_t* p_full = bars + 11;    // [2] per query tile
    uint64_t* o_done = bars + 13;    // [2] per query tile
    uint64_t* q_empty = bars + 15;   // the item's last S products have read its Q tiles
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nq = (p.T + kTq - 1) / kTq;
    const int nkt = (p.T + kTk - 1) / kTk;
    const int npairs = (nq + 1) / 2;
    const int bh_count = p.B * p.H;
    const int items = bh_count * npairs;
    // Work item w: (batch, head) w % (B H) and the pair of query tiles of index w / (B H), pairs
    // with the longest rows first; this CTA takes one item a round, in snake order (item_at)
    struct Item
    {
        int b, h, kvh, qt0, n_a, n_b, nmax;
        bool has_b;
    };
    // round rr of the CTA's items: rounds alternate direction over the CTAs (a snake), so the
    // long items of one round and the short ones of the next even out per CTA
    auto item_at = [&](int rr) {
        const int c = (rr & 1) ? static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x)
                               : static_cast<int>(blockIdx.x);
        const int w = rr * static_cast<int>(gridDim.x) + c;
        return w < items ? w : -1;
    };
    auto item = [&](int w) {
        Item it;
        const int y = w / bh_count, bh = w - y * bh_count;
        it.qt0 = 2 * (npairs - 1 - y);
        it.has_b = it.qt0 + 1 < nq;
        it.b = bh / p.H;
        it.h = bh - it.b * p.H;
        it.kvh = it.h / (p.H / p.Hkv);
        it.n_a = p.causal ? it.qt0 + 1 : nkt;
        it.n_b = it.has_b ? (p.causal ? it.qt0 + 2 : nkt) : 0;
        it.nmax = it.n_a > it.n_b ? it.n_a : it.n_b;
        return it;
    };

    if (threadIdx.x == 0)
    {
        *abort = 0;
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        for (int i = 0; i < 2; ++i)
        {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 4);
            mbar_init(&o_done[i], 1);
        }
        mbar_fence_init();
    }
    if (warp == 1)
    {
        tmem_alloc(tmem_slot, 512);
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    dep_wait();   // Q, K, V (and O, LSE) belong to the kernels before this one
    dep_release();
    // TMEM columns: S_A | S_B | O_A | O_B (128 each); P_x (bf16 pairs) overwrites S_x's first 64
    // Every ring and barrier phase runs on across the CTA's items (counters kept per role).

    if (warp == 0 && lane == 0)
    {
        tma_prefetch(&tq);
        tma_prefetch(&tk);
        int kc = 0, n_item = 0;
        for (int rr = 0, w = item_at(0); w >= 0; w = item_at(++rr), ++n_item)
        {
            const Item it = item(w);
            // the Q tiles of this item replace the last item's once its final S products (issued
            // one key tile before its end) have completed
            if (n_item > 0)
            {
                mbar_wait(q_empty, (n_item - 1) & 1, p.status, abort);
            }
            mbar_expect_tx(q_full, (it.has_b ? 2 : 1) * kTileBytes);
            load_tile_3d(sq, &tq, q_full, it.h * 128, it.qt0 * kTq, it.b);
            if (it.has_b)
            {
                load_tile_3d(sq + kTileBytes, &tq, q_full, it.h * 128, (it.qt0 + 1) * kTq, it.b);
            }
            for (int j = 0; j < it.nmax; ++j, ++kc)
            {
                const int st = kc & 1;
                mbar_wait(&k_empty[st], ((kc >> 1) & 1) ^ 1, p.status, abort);
                mbar_expect_tx(&k_full[st], kTileBytes);
                load_tile_3d(sk + st * kTileBytes, &tk, &k_full[st], it.kvh * 128, j * kTk, it.b);
            }
        }
    }
    else if (warp == 0 && lane == 1)
    {
        tma_prefetch(&tv);
        int vc = 0;
        for (int rr = 0, w = item_at(0); w >= 0; w = item_at(++rr))
        {
            const Item it = item(w);
            for (int j = 0; j < it.nmax; ++j, ++vc)
            {
                const int st = vc & 1;
                mbar_wait(&v_empty[st], ((vc >> 1) & 1) ^ 1, p.status, abort);
                mbar_expect_tx(&v_full[st], kTileBytes);
                load_tile_3d(sv + st * kTileBytes, &tv, &v_full[st], it.kvh * 128, j * kTk, it.b);
            }
        }
    }
    else if (warp == 1 && lane == 0)
    {
        // Order per key tile j: P_A V_j, S_A(j+1), P_B V_j, S_B(j+1) — so the tensor core works
        // on one query tile while the softmax warps of the other compute its probabilities.
        // An S_x(j+1) issued after P_x V_j overwrites P_x only once that product has read it
        // (the MMAs of one thread execute in issue order); the same holds for the next item's
        // S_x(0). The next item's first P_x V_0 overwrites O_x only after p_full, which the
        // softmax warps of tile x arrive on after they have read O_x out for the last item.
        constexpr uint32_t idesc_s = instr_desc(128, 128, false, false);
        constexpr uint32_t idesc_o = instr_desc(128, 128, false, true);
        const uint32_t q_base = smem_u32(sq);
        int kc = 0, vc = 0, n_item = 0;
        int pc[2] = {0, 0};   // P tiles consumed per query tile
        auto issue_s = [&](int x, int kslot) {
            const uint32_t k_base = smem_u32(sk + kslot * kTileBytes);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
            {
                mma(tmem + x * 128, kmajor_desc(q_base + x * kTileBytes, ks), kmajor_desc(k_base, ks),
                    idesc_s, ks > 0 ? 1u : 0u);
            }
            commit(&s_full[x]);
        };
        auto issue_pv = [&](int x, int j, int n, int vslot) {
            mbar_wait(&p_full[x], pc[x] & 1, p.status, abort);
            ++pc[x];
            fence_after();
            const uint32_t v_base = smem_u32(sv + vslot * kTileBytes);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
            {
                mma_ts(tmem + 256 + x * 128, tmem + x * 128 + ks * 8, mnmajor_desc(v_base, ks, kHalf),
                       idesc_o, (j > 0 || ks > 0) ? 1u : 0u);
            }
            if (j == n - 1)
            {
                commit(&o_done[x]);
            }
        };
        for (int rr = 0, w = item_at(0); w >= 0; w = item_at(++rr), ++n_item)
        {
            const Item it = item(w);
            mbar_wait(q_full, n_item & 1, p.status, abort);
            mbar_wait(&k_full[kc & 1], (kc >> 1) & 1, p.status, abort);
            fence_after();
            issue_s(0, kc & 1);
            if (it.n_b > 0)
            {
                issue_s(1, kc & 1);
            }
            commit(&k_empty[kc & 1]);
            ++kc;
            if (it.nmax == 1)
            {
                commit(q_empty);   // every S product of the item has been issued
            }
            for (int j = 0; j < it.nmax; ++j, ++vc)
            {
                const int st = vc & 1, jn = j + 1;
                mbar_wait(&v_full[st], (vc >> 1) & 1, p.status, abort);
                fence_after();
                if (j < it.n_a)
                {
                    issue_pv(0, j, it.n_a, st);
                }
                if (jn < it.nmax)
                {
                    mbar_wait(&k_full[kc & 1], (kc >> 1) & 1, p.status, abort);
                    fence_after();
                    if (jn < it.n_a)
                    {
                        issue_s(0, kc & 1);
                    }
                }
                if (j < it.n_b)
                {
                    issue_pv(1, j, it.n_b, st);
                }
                commit(&v_empty[st]);
                if (jn < it.nmax)
                {
                    if (jn < it.n_b)
                    {
                        issue_s(1, kc & 1);
                    }
                    commit(&k_empty[kc & 1]);
                    ++kc;
                    if (jn + 1 == it.nmax)
                    {
                        commit(q_empty);   // the item's last S products have been issued
                    }
                }
            }
        }
    }
    else if (warp >= 2)
    {
        const int x = warp >= 6 ? 1 : 0;                  // query tile of this warpgroup
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;                // row within the tile (TMEM lane)
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        const uint32_t s_addr = tmem + lane_base + x * 128;
        const uint32_t o_addr = tmem + lane_base + 256 + x * 128;
        const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2);
        int sc = 0, oc = 0;                               // S tiles and items taken by this tile
        for (int rr = 0, w = item_at(0); w >= 0; w = item_at(++rr))
        {
            const Item it = item(w);
            const int n = x ? it.n_b : it.n_a;
            const int b = it.b, h = it.h;
            const int qtile = it.qt0 + x;
            const int query = qtile * kTq + r;
            float m = -INFINITY, l = 0.0f;   // running max (scaled, log2 units) and row sum
            for (int j = 0; j < n; ++j)
            {
                mbar_wait(&s_full[x], sc & 1, p.status, abort);
                ++sc;
                fence_after();
                uint32_t s[4][32];
#pragma unroll
                for (int c = 0; c < 4; ++c) tmem_ld32_async(s_addr + c * 32, s[c]);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 4; ++c) reg_fence(s[c]);
                const int key0 = j * kTk;
                if ((p.causal && j == qtile) || key0 + kTk > p.T)
                {
                    int limit = p.T - key0 - 1;               // last visible column of this row
                    if (p.causal && j == qtile && r < limit) limit = r;
#pragma unroll
                    for (int e = 0; e < 128; ++e)
                    {
                        if (e > limit) s[e >> 5][e & 31] = 0xFF800000u;   // -inf
                    }
                }
                float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
#pragma unroll
                for (int e = 0; e < 128; e += 8)
                {
                    const uint32_t* v = &s[e >> 5][e & 31];
                    m0 = max3(m0, __uint_as_float(v[0]), __uint_as_float(v[1]));
                    m1 = max3(m1, __uint_as_float(v[2]), __uint_as_float(v[3]));
                    m2 = max3(m2, __uint_as_float(v[4]), __uint_as_float(v[5]));
                    m3 = max3(m3, __uint_as_float(v[6]), __uint_as_float(v[7]));
                }
                const float mx = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3)) * p.scale_log2;
                const bool first = m == -INFINITY;
                const bool grow = mx > m + kRescaleThreshold;
                // O_x is rescaled after P is written (fewer live registers); corr = 1 for rows whose
                // max is kept
                const bool rescale = __any_sync(0xFFFFFFFFu, grow && !first);
                const float corr = (grow && !first) ? ex2(m - mx) : 1.0f;
                if (grow || first)
                {
                    m = mx;
                }
                const float mu = m == -INFINITY ? 0.0f : m;
                const uint64_t neg = f2_pack(-mu, -mu);
                uint64_t acc0 = 0, acc1 = 0;   // two packed partial sums (+0.0f pairs)
#pragma unroll
                for (int g = 0; g < 4; ++g)
                {
                    uint32_t pk[16];   // 32 probabilities as bf16 pairs, stored as soon as computed
#pragma unroll
                    for (int c = 0; c < 16; ++c)
                    {
                        const uint32_t* v = &s[g][c * 2];
                        float a, bb;
                        f2_unpack(f2_fma(f2_pack(__uint_as_float(v[0]), __uint_as_float(v[1])), sc2, neg), a, bb);
                        a = ex2(a);
                        bb = ex2(bb);
                        if (c & 1)
                            acc1 = f2_add(acc1, f2_pack(a, bb));
                        else
                            acc0 = f2_add(acc0, f2_pack(a, bb));
                        const __nv_bfloat162 t = __floats2bfloat162_rn(a, bb);
                        pk[c] = *reinterpret_cast<const uint32_t*>(&t);
                    }
                    tmem_st16_async(s_addr + g * 16, pk);
                }
                float a0, a1, b0, b1;
                f2_unpack(acc0, a0, a1);
                f2_unpack(acc1, b0, b1);
                if (rescale)
                {
                    // the products of tiles < j have completed (S_x(j), issued after them, has), and
                    // P_x V_j is not issued before this warp arrives on p_full
#pragma unroll 1
                    for (int c = 0; c < 4; ++c)
                    {
                        uint32_t raw[32];
                        tmem_ld32(o_addr + c * 32, raw);
#pragma unroll
                        for (int e = 0; e < 32; ++e) raw[e] = __float_as_uint(__uint_as_float(raw[e]) * corr);
                        tmem_st32(o_addr + c * 32, raw);
                    }
                }
                l = l * corr + ((a0 + a1) + (b0 + b1));
                tmem_wait_st();
                fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[x]);
            }
            if (n > 0)
            {
                // epilogue: O / l and the log-sum-exp
                mbar_wait(&o_done[x], oc & 1, p.status, abort);
                ++oc;
                fence_after();
                const float inv = l > 0.0f ? 1.0f / l : 0.0f;
                const bool valid = query < p.T;
                bf16* orow = p.o + (static_cast<int64_t>(b) * p.T + query) * p.ldo + static_cast<int64_t>(h) * 128;
#pragma unroll 1
                for (int c = 0; c < 4; ++c)
                {
                    uint32_t raw[32];
                    tmem_ld32(o_addr + c * 32, raw);
                    if (valid)
                    {
#pragma unroll
                        for (int e = 0; e < 32; e += 8)
                        {
                            float v8[8];
#pragma unroll
                            for (int q = 0; q < 8; ++q) v8[q] = __uint_as_float(raw[e + q]) * inv;
                            store16(orow + c * 32 + e, v8);
                        }
                    }
                }
                if (valid)
                {
                    p.lse[(static_cast<int64_t>(b) * p.H + h) * p.T + query] = (m + log2f(l)) * kLn2;
                }
            }
        }
    }
    fence_before();
    __syncthreads();
    if (warp == 1)
    {
        fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------------------------------------
// Backward, in three launches.
// (0) attn_rowdot_kernel — D = rowsum(dO * O) and -LSE log2(e) per (batch, head, query).
// (1) attn_bwd_tc_kernel — one CTA per (batch, KV head, 128-key tile); 10 warps. For every query
//     head of the GQA group and every 64-query tile at or after the diagonal:
//       TMA    Q, dO (64 x 128 each) and that tile's -LSE log2(e) and D into a 4-stage ring;
//       MMA    S^T = K Q^T and dP^T = V dO^T (M128 keys, N64 queries, K128 dims) into one of two
//              TMEM buffer pairs, so the products of tile i+1 run while tile i is elementwise;
//       warps  (8, two per TMEM lane quarter, 32 query columns each)
//              P^T = exp2(S^T scale log2e - LSE log2e), causal mask, dS^T = P^T (dP^T - D);
//              P^T and dS^T (bf16 pairs) overwrite their S^T and dP^T columns in TMEM, and dS^T
//              also goes straight to HBM for the dQ kernel;
//       MMA    dV += P^T dO, dK += dS^T Q (M128 keys, N128 dims, K64 queries; P^T and dS^T read
//              by the MMA from tensor memory, accumulators in TMEM).
//     dK and dV are summed over the group's heads in TMEM: written once, deterministically.
// (2) attn_dq_tc_kernel — one CTA per (batch, head, 128-query tile): dQ = sum over key tiles of
//     dS K (M128 queries, N128 dims, K128 keys) from the stored dS^T, accumulated in TMEM — no
//     atomics, so dQ is deterministic too.
// The Q/dO tiles are staged once per tile and serve both as K-major operands (rows = queries = N)
// and as MN-major operands (rows = queries = K); likewise K for S^T and the dQ product.
// ---------------------------------------------------------------------------------------------
constexpr int kBq = 64;                      // queries per backward iteration
constexpr int kQTileBytes = kBq * 128 * 2;   // [64 rows x 128 dims] = two 8 KB halves
constexpr int kQHalf = kQTileBytes / 2;
constexpr int kQStages = 3;
constexpr int kComputeWarps = 16;            // four per TMEM lane quarter, 16 query columns each
constexpr int kBwdThreads = 64 + 32 * kComputeWarps;
constexpr int kDsTileBytes = 128 * kBq * 2;  // dS^T [128 keys x 64 queries] staging for the store
// alignment slack | K, V | (Q, dO)[3] | dS^T staging [2] | (-LSE log2e, D)[3] | barriers
constexpr int kBwdSmem = 1024 + 2 * kTileBytes + 2 * kQStages * kQTileBytes + 2 * kDsTileBytes +
                         kQStages * 2 * kBq * 4 + 256;

struct BwdParams
{
    const float* nlse2;   // -LSE log2(e) [B, H, T]
    const float* dvec;    // D [B, H, T]
    bf16 *dk, *dv, *ds;   // ds: dS^T [B*H][T keys][T queries]
    int64_t lddk, lddv;
    int T, H, Hkv;
    float scale, scale_log2;
    int causal;
    int* status;
};

__device__ __forceinline__ void load_qtile_3d(uint8_t* dst, const CUtensorMap* map, uint64_t* bar,
                                              int col, int row, int batch)
{
    tma_load_3d(dst, map, bar, col, row, batch);
    tma_load_3d(dst + kQHalf, map, bar, col + 64, row, batch);
}

__device__ __forceinline__ void named_sync(int id, int count)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ uint32_t pack2(float a, float b)
{
    const __nv_bfloat162 t = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&t);
}

__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b)
{
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

__global__ void __launch_bounds__(kBwdThreads, 1)
attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                   const __grid_constant__ CUtensorMap tds, const BwdParams p)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* sk = smem;
    uint8_t* sv = sk + kTileBytes;
    uint8_t* sq = sv + kTileBytes;                          // [stages]
    uint8_t* sdo = sq + kQStages * kQTileBytes;             // [stages]
    uint8_t* sdst = sdo + kQStages * kQTileBytes;            // [2] dS^T staging
    float* srow = reinterpret_cast<float*>(sdst + 2 * kDsTileBytes);   // [stages][2][64]
    uint64_t* bars = reinterpret_cast<uint64_t*>(srow + kQStages * 2 * kBq);
    uint64_t* kv_full = bars + 0;
    uint64_t* qd_full = bars + 1;                  // [stages]
    uint64_t* qd_empty = bars + 1 + kQStages;      // [stages]
    uint64_t* sp_full = bars + 1 + 2 * kQStages;   // [2]
    uint64_t* ds_full = bars + 3 + 2 * kQStages;   // [2]
    uint64_t* done = bars + 5 + 2 * kQStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 6 + 2 * kQStages);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kt = static_cast<int>(blockIdx.y);   // launch order: all heads' key tile 0 (the
    const int bk = blockIdx.x;                      // longest under the causal mask) first
    const int b = bk / p.Hkv, kvh = bk % p.Hkv;
    const int rep = p.H / p.Hkv;
    const int nq = (p.T + kBq - 1) / kBq;
    const int qi0 = p.causal ? (kt * 128) / kBq : 0;
    const int per_head = nq - qi0;
    const int iters = rep * per_head;

    if (threadIdx.x == 0)
    {
        *abort = 0;
        mbar_init(kv_full, 1);
        for (int i = 0; i < kQStages; ++i)
        {
            mbar_init(&qd_full[i], 1);
            mbar_init(&qd_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i)
        {
            mbar_init(&sp_full[i], 1);
            mbar_init(&ds_full[i], kComputeWarps);
        }
        mbar_init(done, 1);
        mbar_fence_init();
    }
    if (warp == 1)
    {
        tmem_alloc(tmem_slot, 512);
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    // TMEM columns: S^T[2] (64 each) | dP^T[2] (64 each) | dV (128) | dK (128). P^T and dS^T
    // (bf16 pairs) overwrite columns [16 g, 16 g + 8) of their buffer, g = the 16-query group.
    constexpr uint32_t kST = 0, kDPT = 128, kDV = 256, kDK = 384;

    if (warp == 0 && lane == 0)
    {
        tma_prefetch(&tq);
        tma_prefetch(&tk);
        tma_prefetch(&tv);
        tma_prefetch(&tdo);
        mbar_expect_tx(kv_full, 2 * kTileBytes);
        load_tile_3d(sk, &tk, kv_full, kvh * 128, kt * 128, b);
        load_tile_3d(sv, &tv, kv_full, kvh * 128, kt * 128, b);
        for (int it = 0; it < iters; ++it)
        {
            const int sq_i = it % kQStages;
            const int h = kvh * rep + it / per_head;
            const int q0 = (qi0 + it % per_head) * kBq;
            const int nrow = p.T - q0 < kBq ? p.T - q0 : kBq;   // a multiple of 8 (T % 8 == 0)
            const uint32_t rbytes = static_cast<uint32_t>(nrow) * 4;
            const int64_t at = (static_cast<int64_t>(b) * p.H + h) * p.T + q0;
            mbar_wait(&qd_empty[sq_i], ((it / kQStages) & 1) ^ 1, p.status, abort);
            mbar_expect_tx(&qd_full[sq_i], 2 * kQTileBytes + 2 * rbytes);
            load_qtile_3d(sq + sq_i * kQTileBytes, &tq, &qd_full[sq_i], h * 128, q0, b);
            load_qtile_3d(sdo + sq_i * kQTileBytes, &tdo, &qd_full[sq_i], h * 128, q0, b);
            bulk_load(srow + sq_i * 2 * kBq, p.nlse2 + at, rbytes, &qd_full[sq_i]);
            bulk_load(srow + sq_i * 2 * kBq + kBq, p.dvec + at, rbytes, &qd_full[sq_i]);
        }
    }
    else if (warp == 1 && lane == 0)
    {
        constexpr uint32_t idesc_s = instr_desc(128, kBq, false, false);
        constexpr uint32_t idesc_kv = instr_desc(128, 128, false, true);
        const uint32_t k_base = smem_u32(sk), v_base = smem_u32(sv);
        mbar_wait(kv_full, 0, p.status, abort);
        auto issue_dvdk = [&](int i) {
            const int s = i & 1, sq_i = i % kQStages;
            mbar_wait(&ds_full[s], (i >> 1) & 1, p.status, abort);
            fence_after();
            const uint32_t q_base = smem_u32(sq + sq_i * kQTileBytes);
            const uint32_t do_base = smem_u32(sdo + sq_i * kQTileBytes);
#pragma unroll
            for (int ks = 0; ks < kBq / 16; ++ks)
            {
                const uint32_t acc = (i > 0 || ks > 0) ? 1u : 0u;
                const uint32_t col = s * 64 + ks * 16;   // queries [16 ks, 16 ks + 16), packed
                mma_ts(tmem + kDV, tmem + kST + col, mnmajor_desc(do_base, ks, kQHalf), idesc_kv, acc);
                mma_ts(tmem + kDK, tmem + kDPT + col, mnmajor_desc(q_base, ks, kQHalf), idesc_kv, acc);
            }
            commit(&qd_empty[sq_i]);
        };
        for (int it = 0; it < iters; ++it)
        {
            const int st = it & 1, sq_i = it % kQStages;
            const uint32_t q_base = smem_u32(sq + sq_i * kQTileBytes);
            const uint32_t do_base = smem_u32(sdo + sq_i * kQTileBytes);
            mbar_wait(&qd_full[sq_i], (it / kQStages) & 1, p.status, abort);
            fence_after();
            // S^T / dP^T of buffer st were last read (as P^T / dS^T) by the dV/dK products of
            // tile it-2, issued before these: the MMAs of one thread execute in issue order.
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
            {
                const uint32_t off = (ks >> 2) * kQHalf + (ks & 3) * 32;
                mma(tmem + kST + st * 64, kmajor_desc(k_base, ks), smem_desc(q_base + off, 16, 1024),
                    idesc_s, ks > 0 ? 1u : 0u);
                mma(tmem + kDPT + st * 64, kmajor_desc(v_base, ks),
                    smem_desc(do_base + off, 16, 1024), idesc_s, ks > 0 ? 1u : 0u);
            }
            commit(&sp_full[st]);
            if (it > 0)
            {
                issue_dvdk(it - 1);
            }
        }
        if (iters > 0)
        {
            issue_dvdk(iters - 1);
        }
        commit(done);
    }
    else if (warp >= 2)
    {
        const int quarter = warp & 3;
        const int grp = (warp - 2) >> 2;        // query columns [16 grp, 16 grp + 16)
        const int r = quarter * 32 + lane;      // key row
        const int key = kt * 128 + r;
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2);
        const uint64_t neg1 = f2_pack(-1.0f, -1.0f);
        const bool issuer = warp == 2 && lane == 0;   // issues the dS^T tile stores
        for (int it = 0; it < iters; ++it)
        {
            const int st = it & 1, sq_i = it % kQStages;
            const int h = kvh * rep + it / per_head;
            const int q0 = (qi0 + it % per_head) * kBq;
            const int qc = q0 + grp * 16;       // first query of this thread's columns
            mbar_wait(&sp_full[st], (it >> 1) & 1, p.status, abort);
            // the stage's -LSE log2e / D rows arrived with its Q / dO (phase already complete)
            mbar_wait(&qd_full[sq_i], (it / kQStages) & 1, p.status, abort);
            fence_after();
            uint32_t sraw[16], draw[16];
            const uint32_t col = st * 64 + grp * 16;
            tmem_ld16_async(tmem + lane_base + kST + col, sraw);
            tmem_ld16_async(tmem + lane_base + kDPT + col, draw);
            tmem_wait_ld();
            reg_fence(sraw);
            reg_fence(draw);
            const float* nl = srow + sq_i * 2 * kBq + grp * 16;
            const float* dd = nl + kBq;
            // visible columns c: lo <= c < hi (queries before T and, causal, not before this key)
            const int hi = qc + 16 > p.T ? (p.T - qc > 0 ? p.T - qc : 0) : 16;
            const bool causal_tile = p.causal && qc < kt * 128 + 127;   // some key > query here
            const int lo = causal_tile ? (key - qc > 0 ? key - qc : 0) : 0;
            uint32_t pk[8], dk[8];
            if (!causal_tile && hi == 16)
            {
#pragma unroll
                for (int c = 0; c < 16; c += 4)
                {
                    const float4 nl4 = *reinterpret_cast<const float4*>(nl + c);
                    const float4 d4 = *reinterpret_cast<const float4*>(dd + c);
#pragma unroll
                    for (int u = 0; u < 4; u += 2)
                    {
                        const int e = c + u;
                        float p0, p1;
                        f2_unpack(f2_fma(f2_pack(__uint_as_float(sraw[e]), __uint_as_float(sraw[e + 1])), sc2,
                                         u == 0 ? f2_pack(nl4.x, nl4.y) : f2_pack(nl4.z, nl4.w)),
                                  p0, p1);
                        p0 = ex2(p0);
                        p1 = ex2(p1);
                        const uint64_t t = f2_fma(u == 0 ? f2_pack(d4.x, d4.y) : f2_pack(d4.z, d4.w), neg1,
                                                  f2_pack(__uint_as_float(draw[e]), __uint_as_float(draw[e + 1])));
                        float d0, d1;
                        f2_unpack(f2_mul(f2_pack(p0, p1), t), d0, d1);
                        pk[e >> 1] = pack2(p0, p1);
                        dk[e >> 1] = pack2(d0, d1);
                    }
                }
            }
            else
            {
#pragma unroll
                for (int c = 0; c < 16; c += 2)
                {
                    const float2 nl2 = *reinterpret_cast<const float2*>(nl + c);
                    const float2 d2 = *reinterpret_cast<const float2*>(dd + c);
                    float p0, p1;
                    f2_unpack(f2_fma(f2_pack(__uint_as_float(sraw[c]), __uint_as_float(sraw[c + 1])), sc2,
                                     f2_pack(nl2.x, nl2.y)),
                              p0, p1);
                    const bool v0 = c >= lo && c < hi;
                    const bool v1 = c + 1 >= lo && c + 1 < hi;
                    p0 = v0 ? ex2(p0) : 0.0f;
                    p1 = v1 ? ex2(p1) : 0.0f;
                    const uint64_t t = f2_fma(f2_pack(d2.x, d2.y), neg1,
                                              f2_pack(__uint_as_float(draw[c]), __uint_as_float(draw[c + 1])));
                    float d0, d1;
                    f2_unpack(f2_mul(f2_pack(p0, p1), t), d0, d1);
                    d0 = v0 ? d0 : 0.0f;   // masked columns may hold stale -LSE / D values
                    d1 = v1 ? d1 : 0.0f;
                    pk[c >> 1] = pack2(p0, p1);
                    dk[c >> 1] = pack2(d0, d1);
                }
            }
            tmem_st8_async(tmem + lane_base + kST + col, pk);
            tmem_st8_async(tmem + lane_base + kDPT + col, dk);
            // dS^T row piece into the swizzled staging tile (two 16-byte chunks of the 128-byte row)
            uint8_t* stile = sdst + st * kDsTileBytes;
            *reinterpret_cast<uint4*>(stile + sw128_offset(r, grp * 2)) = make_uint4(dk[0], dk[1], dk[2], dk[3]);
            *reinterpret_cast<uint4*>(stile + sw128_offset(r, grp * 2 + 1)) = make_uint4(dk[4], dk[5], dk[6], dk[7]);
            fence_proxy_async();
            tmem_wait_st();
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ds_full[st]);
            if (issuer)
            {
                // the previous tile's store has read its staging buffer, which the next
                // iteration rewrites (every thread passes the barrier below before that)
                bulk_wait_group_read<0>();
            }
            named_sync(1, 32 * kComputeWarps);   // every row of this dS^T tile is staged
            if (issuer)
            {
                tma_store_3d(&tds, stile, q0, kt * 128, b * p.H + h);
                bulk_commit_group();
            }
        }
        if (issuer)
        {
            bulk_wait_group<0>();
        }
        // dV and dK rows of this key (summed over the group's heads in TMEM): 32 dims per warp
        mbar_wait(done, 0, p.status, abort);
        fence_after();
        const bool valid = key < p.T;
        bf16* vrow = p.dv + (static_cast<int64_t>(b) * p.T + key) * p.lddv + static_cast<int64_t>(kvh) * 128;
        bf16* krow = p.dk + (static_cast<int64_t>(b) * p.T + key) * p.lddk + static_cast<int64_t>(kvh) * 128;
        {
            const int c = grp;
            uint32_t rv[32], rk[32];
            tmem_ld32(tmem + lane_base + kDV + c * 32, rv);
            tmem_ld32(tmem + lane_base + kDK + c * 32, rk);
            if (valid)
            {
#pragma unroll
                for (int e = 0; e < 32; e += 8)
                {
                    float a8[8], k8[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                    {
                        a8[q] = __uint_as_float(rv[e + q]);
                        k8[q] = __uint_as_float(rk[e + q]) * p.scale;
                    }
                    store16(vrow + c * 32 + e, a8);
                    store16(krow + c * 32 + e, k8);
                }
            }
        }
    }
    fence_before();
    __syncthreads();
    if (warp == 1)
    {
        fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------------------------------------
// Fused backward (the default): the five products of the backward in one kernel on 128 x 128
// tiles, so dS^T never leaves the SM and the workspace is O(B H T). One CTA per (batch, KV head,
// 128-key tile), looping over the GQA group's query heads x 128-query tiles; 16 warps in four
// warpgroups, with registers moved between them by setmaxnreg:
//   warps 0-3    dQ drain (144 registers), one per TMEM lane quarter (32 queries x 128 dims): the
//                whole tile out of TMEM at once (the next dP^T reuses the columns), then 32-dim
//                slices through a swizzled shared ring into TMA bulk reduce-adds on the fp32
//                accumulator [B, T, H*128] (zeroed by attn_rowdot_kernel; attn_dq_cast_kernel
//                scales and rounds it into dQ);
//   warps 4-11   elementwise, thread = key row, 64 query columns each. Phase 1: P^T = exp2(S^T
//                scale log2e - LSE log2e) (causal mask on the diagonal tile only), written as bf16
//                pairs over the first half of the warp's own S^T columns. Phase 2: dS^T = P^T (dP^T
//                - D), bf16, into the swizzled shared tile both the dQ and the dK products read;
//   warp 12      TMA (112 registers): K and V once; per query tile Q with its -LSE log2(e) and D
//                rows (2 stages) and dO (1 stage);
//   warp 13      MMA (112 registers), every product M128 x N128 x K128: per tile i the order is
//                  S^T(i+1) = K Q^T,  dQ(i) = dS(i) K,  dK += dS^T(i) Q,  dP^T(i+1) = V dO^T,
//                  dV += P^T(i+1) dO
//                so the elementwise work of each phase overlaps other products: P(i+1) is formed
//                while dQ(i) and dK(i) run, dS(i+1) while dV(i+1) and S^T(i+2) run; dQ(i) comes
//                before dK(i) so that its drain overlaps dK(i) (dP^T(i+1) reuses its columns);
//   warps 14-15  idle (they complete the warpgroup that gives up registers).
// dK and dV are summed over the group's query heads in TMEM and written once. The order in which
// the key tiles of a query add into its accumulator varies between runs, so dQ is not
// bit-reproducible; the two-kernel path is (veda_attention_set_deterministic).
// TMEM columns: S^T -> P^T [0, 128) | dP^T, then dQ [128, 256) | dV | dK.
// ---------------------------------------------------------------------------------------------
constexpr int kFq = 128;                            // queries per tile
constexpr int kSoftWarps = 8;                       // two per TMEM lane quarter, 64 columns each
constexpr int kDrainWarps = 4;                      // one per lane quarter
// warpgroup 0: drain; 1-2: elementwise; 3: TMA, MMA and two idle warps (whole warpgroups, so
// setmaxnreg can move registers: launched at 128 a thread = 65536, then 144 + 128 + 128 + 112)
constexpr int kFusedThreads = 512;
constexpr int kTmaWarp = 12, kMmaWarp = 13;
constexpr int kDrainRegs = 144, kIssueRegs = 112;
static_assert(kDrainRegs + 2 * 128 + kIssueRegs == 4 * 128, "register split must add up");
constexpr int kDqSlice = 32 * 32 * 4;               // [32 queries][32 dims] fp32, 128-byte rows
// K, V | Q[2] | dO | dS^T | dQ staging [4 warps][2] | -LSE log2e [2][128] | D [2][128] | barriers,
// from a 1024-byte aligned base; the request is the largest an SM allows, and the kernel checks
// that the aligned layout fits in it.
constexpr int kFusedBytes = 2 * kTileBytes + 2 * kTileBytes + kTileBytes + kTileBytes +
                            kDrainWarps * 2 * kDqSlice + 2 * kFq * 4 + 2 * kFq * 4 + 256;
constexpr int kFusedSmem = 232448;
static_assert(kFusedBytes <= kFusedSmem, "fused attention backward exceeds the shared memory of an SM");

struct FusedParams
{
    const float* nlse2;   // -LSE log2(e) [B, H, T]
    const float* dvec;    // D [B, H, T]
    bf16 *dk, *dv;
    int64_t lddk, lddv;
    int T, H, Hkv;
    float scale, scale_log2;
    int causal;
    int* status;
    int chunk;   // (batch, KV head) pairs per launch-order chunk (see attn_bwd_fused_kernel)
};

__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* map, const void* src, int x,
                                                  int y, int z)
{
    asm volatile(
        "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group"
        " [%0, {%2, %3, %4}], [%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
        "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// The descriptor of the operand `bytes` further on in shared memory: only the start-address field
// (address >> 4, the low 14 bits) changes, and it cannot carry for addresses below 256 KB.
__device__ __forceinline__ uint64_t desc_at(uint64_t d, uint32_t bytes)
{
    return d + (bytes >> 4);
}

// Column (inside the 128-column S^T or dP^T region) of the bf16 P^T / dS^T pairs of the k-th
// 16-query step: each elementwise warp packs its 64 queries into the first 32 of its own columns.
__device__ __forceinline__ uint32_t pt_col(int ks)
{
    return static_cast<uint32_t>(64 * (ks >> 2) + 8 * (ks & 3));
}

template <int N>
__device__ __forceinline__ void regs_inc()
{
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_dec()
{
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// P^T = exp2(S^T scale log2e - LSE log2e) for 16 query columns (c visible iff lo <= c < hi).
__device__ __forceinline__ void p_block(const uint32_t* sr, const float* nl, float* pv, bool full,
                                        int lo, int hi, uint64_t sc2)
{
    if (full)
    {
#pragma unroll
        for (int c = 0; c < 16; c += 4)
        {
            const float4 nl4 = *reinterpret_cast<const float4*>(nl + c);
#pragma unroll
            for (int u = 0; u < 4; u += 2)
            {
                float p0, p1;
                f2_unpack(f2_fma(f2_pack(__uint_as_float(sr[c + u]), __uint_as_float(sr[c + u + 1])), sc2,
                                 u == 0 ? f2_pack(nl4.x, nl4.y) : f2_pack(nl4.z, nl4.w)),
                          p0, p1);
                pv[c + u] = ex2(p0);
                pv[c + u + 1] = ex2(p1);
            }
        }
    }
    else
    {
#pragma unroll
        for (int c = 0; c < 16; c += 2)
        {
            const float2 nl2 = *reinterpret_cast<const float2*>(nl + c);
            float p0, p1;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), sc2,
                             f2_pack(nl2.x, nl2.y)),
                      p0, p1);
            pv[c] = (c >= lo && c < hi) ? ex2(p0) : 0.0f;
            pv[c + 1] = (c + 1 >= lo && c + 1 < hi) ? ex2(p1) : 0.0f;
        }
    }
}

__global__ void __launch_bounds__(kFusedThreads, 1)
attn_bwd_fused_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                      const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                      const __grid_constant__ CUtensorMap tdq, const FusedParams p)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* sk = smem;
    uint8_t* sv = sk + kTileBytes;
    uint8_t* sq = sv + kTileBytes;                 // [2]
    uint8_t* sdo = sq + 2 * kTileBytes;
    uint8_t* sds = sdo + kTileBytes;               // dS^T [128 keys][128 queries], two halves
    uint8_t* sdq = sds + kTileBytes;               // [4 warps][2][32 x 32 fp32]
    float* snl = reinterpret_cast<float*>(sdq + kDrainWarps * 2 * kDqSlice);   // [2][128]
    float* sdv = snl + 2 * kFq;                                               // [2][128]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sdv + 2 * kFq);
    uint64_t* kv_full = bars + 0;
    uint64_t* q_full = bars + 1;      // [2] Q (+ -LSE log2e, D) staged
    uint64_t* q_empty = bars + 3;     // [2] S^T and dK of that Q done
    uint64_t* do_full = bars + 5;     // dO staged
    uint64_t* do_empty = bars + 6;    // dP^T and dV of that dO done
    uint64_t* s_full = bars + 7;      // S^T in TMEM
    uint64_t* p_full = bars + 8;      // P^T in TMEM
    uint64_t* dp_full = bars + 9;     // dP^T in TMEM
    uint64_t* ds_full = bars + 10;    // dS^T in TMEM and in shared memory
    uint64_t* dq_full = bars + 11;    // dQ in TMEM
    uint64_t* dq_empty = bars + 12;   // dQ read out of TMEM
    uint64_t* done = bars + 13;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    if (static_cast<int>(smem - smem_raw) + kFusedBytes > kFusedSmem)
    {
        // the dynamic shared memory base is not aligned as this layout assumes (uniform exit)
        if (threadIdx.x == 0 && p.status != nullptr) atomicExch(p.status, VEDA_ERR_UNSUPPORTED);
        return;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Launch order: the (batch, KV head) pairs in chunks of p.chunk, and inside a chunk every
    // pair's key tile 0 (the longest under the causal mask) first, then tile 1, ... So the CTAs
    // running at any time share the Q / dO tiles and dQ accumulator rows of one chunk, which stay
    // in L2 (all pairs at once thrashed it: 45 % L2 hits, 1.59 GB of DRAM traffic at B 8 T 2048),
    // while the longest-first order inside the chunk keeps the tail short.
    const int npair = static_cast<int>(gridDim.x), ntile = static_cast<int>(gridDim.y);
    const int order = static_cast<int>(blockIdx.y) * npair + static_cast<int>(blockIdx.x);
    const int chunk = order / (p.chunk * ntile), within = order % (p.chunk * ntile);
    const int in_chunk = npair - chunk * p.chunk < p.chunk ? npair - chunk * p.chunk : p.chunk;
    const int kt = within / in_chunk;
    const int bk = chunk * p.chunk + within % in_chunk;
    const int b = bk / p.Hkv, kvh = bk % p.Hkv;
    const int rep = p.H / p.Hkv;
    const int nq = (p.T + kFq - 1) / kFq;
    const int qi0 = p.causal ? kt : 0;
    const int per_head = nq - qi0;
    const int iters = rep * per_head;

    if (threadIdx.x == 0)
    {
        *abort = 0;
        mbar_init(kv_full, 1);
        for (int i = 0; i < 2; ++i)
        {
            mbar_init(&q_full[i], 1);
            mbar_init(&q_empty[i], 1);
        }
        mbar_init(do_full, 1);
        mbar_init(do_empty, 1);
        mbar_init(s_full, 1);
        mbar_init(p_full, kSoftWarps);
        mbar_init(dp_full, 1);
        mbar_init(ds_full, kSoftWarps);
        mbar_init(dq_full, 1);
        mbar_init(dq_empty, kDrainWarps);
        mbar_init(done, 1);
        mbar_fence_init();
    }
    // rows of -LSE log2e / D past T are never loaded: keep them finite (0 * NaN would be NaN)
    for (int i = threadIdx.x; i < 4 * kFq; i += blockDim.x)
    {
        snl[i] = 0.0f;   // snl [2][128] and sdv [2][128] are contiguous
    }
    if (warp == kMmaWarp)
    {
        tmem_alloc(tmem_slot, 512);
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    dep_wait();   // D, -LSE log2 e and the zeroed dQ accumulator come from attn_rowdot_kernel
    dep_release();
    constexpr uint32_t kS = 0, kDP = 128, kDV = 256, kDK = 384;

    if (warp == kTmaWarp)
    {
        regs_dec<kIssueRegs>();
        if (lane == 0)
        {
            tma_prefetch(&tq);
            tma_prefetch(&tk);
            tma_prefetch(&tv);
            tma_prefetch(&tdo);
            tma_prefetch(&tdq);
            mbar_expect_tx(kv_full, 2 * kTileBytes);
            load_tile_3d(sk, &tk, kv_full, kvh * 128, kt * 128, b);
            load_tile_3d(sv, &tv, kv_full, kvh * 128, kt * 128, b);
            for (int it = 0; it < iters; ++it)
            {
                const int s = it & 1;
                const int h = kvh * rep + it / per_head;
                const int q0 = (qi0 + it % per_head) * kFq;
                const int nrow = p.T - q0 < kFq ? p.T - q0 : kFq;   // a multiple of 8 (T % 8 == 0)
                const uint32_t rbytes = static_cast<uint32_t>(nrow) * 4;
                const int64_t at = (static_cast<int64_t>(b) * p.H + h) * p.T + q0;
                // Q stage s (and its -LSE log2e, D rows) is free once dK(it-2) is done, which
                // follows dS^T(it-2), the last elementwise read of those rows
                mbar_wait(&q_empty[s], ((it >> 1) & 1) ^ 1, p.status, abort);
                mbar_expect_tx(&q_full[s], kTileBytes + 2 * rbytes);
                load_tile_3d(sq + s * kTileBytes, &tq, &q_full[s], h * 128, q0, b);
                bulk_load(snl + s * kFq, p.nlse2 + at, rbytes, &q_full[s]);
                bulk_load(sdv + s * kFq, p.dvec + at, rbytes, &q_full[s]);
                mbar_wait(do_empty, (it & 1) ^ 1, p.status, abort);   // dV(it-1) done
                mbar_expect_tx(do_full, kTileBytes);
                load_tile_3d(sdo, &tdo, do_full, h * 128, q0, b);
            }
        }
    }
    else if (warp == kMmaWarp)
    {
        regs_dec<kIssueRegs>();
        if (lane == 0)
        {
            constexpr uint32_t idesc_s = instr_desc(128, kFq, false, false);
            constexpr uint32_t idesc_kv = instr_desc(128, 128, false, true);
            constexpr uint32_t idesc_dq = instr_desc(kFq, 128, true, true);
            // Every operand descriptor is a base descriptor plus a constant offset (desc_at), so
            // the issuing thread spends almost nothing between MMAs.
            const uint64_t k_kmaj = smem_desc(smem_u32(sk), 16, 1024);     // K for S^T
            const uint64_t v_kmaj = smem_desc(smem_u32(sv), 16, 1024);     // V for dP^T
            const uint64_t k_mnmaj = smem_desc(smem_u32(sk), kHalf, 1024); // K for dQ
            const uint64_t q_kmaj = smem_desc(smem_u32(sq), 16, 1024);     // Q (stage 0) for S^T
            const uint64_t q_mnmaj = smem_desc(smem_u32(sq), kHalf, 1024); // Q (stage 0) for dK
            const uint64_t do_kmaj = smem_desc(smem_u32(sdo), 16, 1024);   // dO for dP^T
            const uint64_t do_mnmaj = smem_desc(smem_u32(sdo), kHalf, 1024); // dO for dV
            const uint64_t ds_mnmaj = smem_desc(smem_u32(sds), kHalf, 1024); // dS for dQ
            const uint64_t ds_kmaj = smem_desc(smem_u32(sds), 16, 1024);     // dS^T for dK
            auto kmaj_step = [](int ks) {   // k-step of a K-major [128 x 128] tile
                return static_cast<uint32_t>((ks >> 2) * kHalf + (ks & 3) * 32);
            };
            auto issue_s = [&](int i) {
                const int s = i & 1;
                mbar_wait(&q_full[s], (i >> 1) & 1, p.status, abort);
                fence_after();
                const uint64_t dq = desc_at(q_kmaj, static_cast<uint32_t>(s) * kTileBytes);
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)
                {
                    mma(tmem + kS, desc_at(k_kmaj, kmaj_step(ks)), desc_at(dq, kmaj_step(ks)), idesc_s,
                        ks > 0 ? 1u : 0u);
                }
                commit(s_full);
            };
            auto issue_dp_dv = [&](int i) {
                mbar_wait(do_full, i & 1, p.status, abort);
                fence_after();
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)
                {
                    mma(tmem + kDP, desc_at(v_kmaj, kmaj_step(ks)), desc_at(do_kmaj, kmaj_step(ks)),
                        idesc_s, ks > 0 ? 1u : 0u);
                }
                commit(dp_full);
                mbar_wait(p_full, i & 1, p.status, abort);   // P^T(i) written over S^T(i)
                fence_after();
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)
                {
                    mma_ts(tmem + kDV, tmem + kS + pt_col(ks), desc_at(do_mnmaj, ks * 2048), idesc_kv,
                           (i > 0 || ks > 0) ? 1u : 0u);
                }
                commit(do_empty);
            };
            mbar_wait(kv_full, 0, p.status, abort);
            if (iters > 0)
            {
                issue_s(0);
                issue_dp_dv(0);
            }
            for (int it = 0; it < iters; ++it)
            {
                const int s = it & 1;
                // S^T(it+1): its columns held P^T(it), read by dV(it), issued before this
                if (it + 1 < iters)
                {
                    issue_s(it + 1);
                }
                mbar_wait(ds_full, it & 1, p.status, abort);   // dS^T(it) in shared memory
                fence_after();
                // dQ(it) over the dP^T(it) columns (the elementwise warps have read them), first, so
                // the drain empties it while dK(it) runs; both read the shared dS^T tile
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)
                {
                    mma(tmem + kDP, desc_at(ds_mnmaj, ks * 2048), desc_at(k_mnmaj, ks * 2048), idesc_dq,
                        ks > 0 ? 1u : 0u);
                }
                commit(dq_full);
                const uint64_t dq = desc_at(q_mnmaj, static_cast<uint32_t>(s) * kTileBytes);
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)
                {
                    mma(tmem + kDK, desc_at(ds_kmaj, kmaj_step(ks)), desc_at(dq, ks * 2048), idesc_kv,
                        (it > 0 || ks > 0) ? 1u : 0u);
                }
                commit(&q_empty[s]);
                if (it + 1 < iters)
                {
                    mbar_wait(dq_empty, it & 1, p.status, abort);   // dQ(it) read out of TMEM
                    fence_after();
                    issue_dp_dv(it + 1);
                }
            }
            commit(done);
        }
    }
    else if (warp < kDrainWarps)
    {
        regs_inc<kDrainRegs>();
        // dQ (lane = query, column = dim) of each tile into the fp32 accumulator: the whole
        // tile leaves TMEM at once (the next dP^T reuses its columns), then 32-dim slices go
        // through a swizzled shared ring into TMA bulk reduce-adds
        const int quarter = warp & 3;
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        uint8_t* ring = sdq + quarter * 2 * kDqSlice;
        int g = 0;   // slices issued by this warp
        for (int i = 0; i < iters; ++i)
        {
            const int h = kvh * rep + i / per_head;
            const int q0 = (qi0 + i % per_head) * kFq;
            mbar_wait(dq_full, i & 1, p.status, abort);
            fence_after();
            uint32_t v[4][32];
#pragma unroll
            for (int c = 0; c < 4; ++c)
            {
                tmem_ld32_async(tmem + lane_base + kDP + c * 32, v[c]);
            }
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 4; ++c)
            {
                reg_fence(v[c]);
            }
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(dq_empty);
#pragma unroll
            for (int c = 0; c < 4; ++c, ++g)
            {
                uint8_t* slice = ring + (g & 1) * kDqSlice;
                if (lane == 0)
                {
                    bulk_wait_group_read<1>();   // the reduce that last read this slice is done
                }
                __syncwarp();
                // row = this lane's query, 16-byte chunks XOR-swizzled by the row (128-byte rows)
#pragma unroll
                for (int j = 0; j < 8; ++j)
                {
                    *reinterpret_cast<uint4*>(slice + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                        make_uint4(v[c][4 * j], v[c][4 * j + 1], v[c][4 * j + 2], v[c][4 * j + 3]);
                }
                fence_proxy_async();
                __syncwarp();
                if (lane == 0)
                {
                    // rows past T fall outside the tensor map and are not written
                    tma_reduce_add_3d(&tdq, slice, h * 128 + c * 32, q0 + quarter * 32, b);
                    bulk_commit_group();
                }
            }
        }
        if (lane == 0)
        {
            bulk_wait_group<0>();
        }
    }
    else if (warp < kDrainWarps + kSoftWarps)
    {
        const int quarter = warp & 3;
        const int grp = (warp - kDrainWarps) >> 2;   // query columns [64 grp, 64 grp + 64)
        const int r = quarter * 32 + lane;                 // key row
        const int key = kt * 128 + r;
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2);
        const uint64_t neg1 = f2_pack(-1.0f, -1.0f);
        for (int it = 0; it < iters; ++it)
        {
            const int s = it & 1;
            const int q0 = (qi0 + it % per_head) * kFq;
            const int qg = q0 + grp * 64;   // first query of this warp's columns
            // Phase 1: P^T. The -LSE log2e rows arrived with Q, before S^T.
            mbar_wait(&q_full[s], (it >> 1) & 1, p.status, abort);
            mbar_wait(s_full, it & 1, p.status, abort);
            fence_after();
            // 32 columns at a time; P^T of a half goes to the first 16 of the 32 columns that half
            // loaded itself, so nothing is overwritten before it is read
            uint32_t pk[32];   // P^T of the 64 columns as bf16 pairs, kept for phase 2
            const float* nl = snl + s * kFq + grp * 64;
#pragma unroll
            for (int half = 0; half < 2; ++half)
            {
                uint32_t sraw[32];
                tmem_ld32_async(tmem + lane_base + kS + grp * 64 + half * 32, sraw);
                tmem_wait_ld();
                reg_fence(sraw);
#pragma unroll
                for (int j = 0; j < 2; ++j)
                {
                    const int qc = qg + 32 * half + 16 * j;
                    const int hi = qc + 16 > p.T ? (p.T - qc > 0 ? p.T - qc : 0) : 16;
                    const bool causal_tile = p.causal && qc < kt * 128 + 127;   // a key > a query
                    const int lo = causal_tile ? (key - qc > 0 ? key - qc : 0) : 0;
                    float pv[16];
                    p_block(sraw + 16 * j, nl + 32 * half + 16 * j, pv, !causal_tile && hi == 16, lo,
                            hi, sc2);
#pragma unroll
                    for (int e = 0; e < 8; ++e) pk[16 * half + 8 * j + e] = pack2(pv[2 * e], pv[2 * e + 1]);
                }
                tmem_st16_async(tmem + lane_base + kS + grp * 64 + half * 16,
                                *reinterpret_cast<uint32_t(*)[16]>(pk + 16 * half));
            }
            tmem_wait_st();
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
            // Phase 2: dS^T. D arrived with Q; the dS^T tile's readers dQ(it-1) and dK(it-1) were
            // issued before dP^T(it), so they are complete once dP^T(it) is (the commit tracks
            // every earlier product of the issuing thread).
            mbar_wait(dp_full, it & 1, p.status, abort);
            fence_after();
            // this warp's 64 queries are the 128-byte row r of half grp of the dS^T tile
            uint8_t* row = sds + grp * kHalf;
#pragma unroll
            for (int half = 0; half < 2; ++half)
            {
                uint32_t draw[32];
                tmem_ld32_async(tmem + lane_base + kDP + grp * 64 + half * 32, draw);
                tmem_wait_ld();
                reg_fence(draw);
                uint32_t dk[16];
#pragma unroll
                for (int c = 0; c < 32; c += 4)
                {
                    const float4 d4 = *reinterpret_cast<const float4*>(sdv + s * kFq + grp * 64 + half * 32 + c);
#pragma unroll
                    for (int u = 0; u < 4; u += 2)
                    {
                        // masked columns have P = 0, so dS = 0 (D and dP^T are finite there)
                        const uint64_t t = f2_fma(u == 0 ? f2_pack(d4.x, d4.y) : f2_pack(d4.z, d4.w), neg1,
                                                  f2_pack(__uint_as_float(draw[c + u]),
                                                          __uint_as_float(draw[c + u + 1])));
                        // dS from the bf16 P the dV product uses (the pair's low half is the even column)
                        const uint32_t pp = pk[16 * half + ((c + u) >> 1)];
                        float d0, d1;
                        f2_unpack(f2_mul(f2_pack(__uint_as_float(pp << 16), __uint_as_float(pp & 0xFFFF0000u)), t),
                                  d0, d1);
                        dk[(c + u) >> 1] = pack2(d0, d1);
                    }
                }
#pragma unroll
                for (int c = 0; c < 4; ++c)
                {
                    *reinterpret_cast<uint4*>(row + sw128_offset(r, 4 * half + c)) =
                        make_uint4(dk[4 * c], dk[4 * c + 1], dk[4 * c + 2], dk[4 * c + 3]);
                }
            }
            fence_proxy_async();
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(ds_full);
        }
        // dV and dK rows of this key (summed over the group's heads in TMEM): 64 dims per warp
        mbar_wait(done, 0, p.status, abort);
        fence_after();
        const bool valid = key < p.T;
        bf16* vrow = p.dv + (static_cast<int64_t>(b) * p.T + key) * p.lddv + static_cast<int64_t>(kvh) * 128;
        bf16* krow = p.dk + (static_cast<int64_t>(b) * p.T + key) * p.lddk + static_cast<int64_t>(kvh) * 128;
#pragma unroll 1
        for (int c = grp * 2; c < grp * 2 + 2; ++c)
        {
            uint32_t rv[32], rk[32];
            tmem_ld32(tmem + lane_base + kDV + c * 32, rv);
            tmem_ld32(tmem + lane_base + kDK + c * 32, rk);
            if (valid)
            {
#pragma unroll
                for (int e = 0; e < 32; e += 8)
                {
                    float a8[8], k8[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                    {
                        a8[q] = __uint_as_float(rv[e + q]);
                        k8[q] = __uint_as_float(rk[e + q]) * p.scale;
                    }
                    store16(vrow + c * 32 + e, a8);
                    store16(krow + c * 32 + e, k8);
                }
            }
        }
    }
    else if (warp > kMmaWarp)
    {
        regs_dec<kIssueRegs>();   // the idle warps of the TMA / MMA warpgroup
    }
    fence_before();
    __syncthreads();
    if (warp == kMmaWarp)
    {
        fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// dQ = scale * the fp32 accumulator [B*T][H*128], rounded to bf16 into the caller's layout; eight
// dims per thread.
__global__ void attn_dq_cast_kernel(const float* __restrict__ acc, bf16* __restrict__ dq,
                                    int64_t lddq, int64_t rows, int64_t width, float scale)
{
    dep_wait();
    dep_release();
    const int64_t per_row = width >> 3;
    const int64_t n = rows * per_row;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        const int64_t row = i / per_row, c = (i - row * per_row) << 3;
        const float4 a = *reinterpret_cast<const float4*>(acc + row * width + c);
        const float4 b = *reinterpret_cast<const float4*>(acc + row * width + c + 4);
        const float v8[8] = {a.x * scale, a.y * scale, a.z * scale, a.w * scale,
                             b.x * scale, b.y * scale, b.z * scale, b.w * scale};
        store16(dq + row * lddq + c, v8);
    }
}

// dQ[q-tile] = sum over key tiles of dS K, from dS^T stored as [B*H][keys][queries].
// Persistent: one CTA per SM walks the (batch, head, 128-query tile) items, longest first, with
// the TMA ring (a dS^T tile and a K tile per stage) streaming across item boundaries and two TMEM
// accumulators, so one item's epilogue overlaps the next item's products (a CTA per item paid the
// ring's fill and the epilogue on every short item). Warp 0 TMA, warp 1 MMA (M128 queries, N128
// dims, K128 keys; both operands MN-major), warps 2-5 epilogue.
constexpr int kDqStages = 3;
constexpr int kDqSmem = 1024 + kDqStages * 2 * kTileBytes + 256;

struct DqParams
{
    bf16* dq;
    int64_t lddq;
    int T, H, Hkv, B;
    float scale;
    int causal;
    int* status;
};

// item k -> (query tile, batch*head), heaviest (latest) query tiles first
__device__ __forceinline__ void dq_item(int k, int bhs, int nq, int& qt, int& bh)
{
    qt = nq - 1 - k / bhs;
    bh = k % bhs;
}

__global__ void __launch_bounds__(192, 1)
attn_dq_tc_kernel(const __grid_constant__ CUtensorMap tds, const __grid_constant__ CUtensorMap tk,
                  const DqParams p)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* sds = smem;                                   // [stages]
    uint8_t* sk = sds + kDqStages * kTileBytes;            // [stages]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sk + kDqStages * kTileBytes);
    uint64_t* full = bars;                     // [stages]
    uint64_t* empty = bars + kDqStages;        // [stages]
    uint64_t* acc_full = bars + 2 * kDqStages;       // [2]
    uint64_t* acc_empty = bars + 2 * kDqStages + 2;  // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kDqStages + 4);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nq = (p.T + 127) / 128;
    const int bhs = p.B * p.H;
    const int items = bhs * nq;
    const int rep = p.H / p.Hkv;

    if (threadIdx.x == 0)
    {
        *abort = 0;
        for (int s = 0; s < kDqStages; ++s)
        {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; ++i)
        {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 4);   // one arrival per epilogue warp
        }
        mbar_fence_init();
    }
    if (warp == 1)
    {
        tmem_alloc(tmem_slot, 256);
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0)
    {
        tma_prefetch(&tds);
        tma_prefetch(&tk);
        int g = 0;   // stages issued so far
        for (int k = blockIdx.x; k < items; k += gridDim.x)
        {
            int qt, bh;
            dq_item(k, bhs, nq, qt, bh);
            const int b = bh / p.H, kvh = (bh % p.H) / rep;
            const int nk = p.causal ? qt + 1 : nq;
            for (int j = 0; j < nk; ++j, ++g)
            {
                const int s = g % kDqStages;
                mbar_wait(&empty[s], ((g / kDqStages) & 1) ^ 1, p.status, abort);
                mbar_expect_tx(&full[s], 2 * kTileBytes);
                // dS^T tile: rows = keys j*128.., columns = this item's 128 queries
                load_tile_3d(sds + s * kTileBytes, &tds, &full[s], qt * 128, j * 128, bh);
                load_tile_3d(sk + s * kTileBytes, &tk, &full[s], kvh * 128, j * 128, b);
            }
        }
    }
    else if (warp == 1 && lane == 0)
    {
        constexpr uint32_t idesc = instr_desc(128, 128, true, true);
        int g = 0, i = 0;
        for (int k = blockIdx.x; k < items; k += gridDim.x, ++i)
        {
            int qt, bh;
            dq_item(k, bhs, nq, qt, bh);
            const int nk = p.causal ? qt + 1 : nq;
            const int buf = i & 1;
            // the epilogue has drained this accumulator (item i - 2)
            mbar_wait(&acc_empty[buf], ((i >> 1) & 1) ^ 1, p.status, abort);
            fence_after();
            for (int j = 0; j < nk; ++j, ++g)
            {
                const int s = g % kDqStages;
                mbar_wait(&full[s], (g / kDqStages) & 1, p.status, abort);
                fence_after();
                const uint32_t a_base = smem_u32(sds + s * kTileBytes);
                const uint32_t b_base = smem_u32(sk + s * kTileBytes);
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)
                {
                    mma(tmem + buf * 128, mnmajor_desc(a_base, ks, kHalf), mnmajor_desc(b_base, ks, kHalf),
                        idesc, (j > 0 || ks > 0) ? 1u : 0u);
                }
                commit(&empty[s]);
            }
            commit(&acc_full[buf]);
        }
    }
    else if (warp >= 2)
    {
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        int i = 0;
        for (int k = blockIdx.x; k < items; k += gridDim.x, ++i)
        {
            int qt, bh;
            dq_item(k, bhs, nq, qt, bh);
            const int b = bh / p.H, h = bh % p.H;
            const int query = qt * 128 + r;
            const int buf = i & 1;
            mbar_wait(&acc_full[buf], (i >> 1) & 1, p.status, abort);
            fence_after();
            bf16* row = p.dq + (static_cast<int64_t>(b) * p.T + query) * p.lddq + static_cast<int64_t>(h) * 128;
#pragma unroll 1
            for (int c = 0; c < 4; ++c)
            {
                uint32_t raw[32];
                tmem_ld32(tmem + lane_base + buf * 128 + c * 32, raw);
                if (query < p.T)
                {
#pragma unroll
                    for (int e = 0; e < 32; e += 8)
                    {
                        float v8[8];
#pragma unroll
                        for (int q = 0; q < 8; ++q) v8[q] = __uint_as_float(raw[e + q]) * p.scale;
                        store16(row + c * 32 + e, v8);
                    }
                }
            }
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
    }
    fence_before();
    __syncthreads();
    if (warp == 1)
    {
        fence_after();
        tmem_dealloc(tmem, 256);
    }
}

// D = rowsum(dO * O) and -LSE log2(e) per (batch, head, query), and (fused path) the zeroed dQ
// accumulator rows. One block per (batch, head) and 64 consecutive queries: 16 groups of 16
// lanes, each group four consecutive queries with all eight of a lane's 16-byte loads in flight
// together; the per-query LSE read and D / -LSE log2(e) writes are contiguous in the query, and
// no index needs a division (a grid-stride loop over (token, head) rows with 64-bit divisions and
// LSE accesses strided by T took 34 us a launch at B 4, H 16, T 2048).
constexpr int kRowdotRows = 4;
constexpr int kRowdotBlockRows = 16 * kRowdotRows;

__global__ void __launch_bounds__(256)
attn_rowdot_kernel(const bf16* __restrict__ o, int64_t ldo, const bf16* __restrict__ dout,
                   int64_t lddo, const float* __restrict__ lse, float* __restrict__ dvec,
                   float* __restrict__ nlse2, float* __restrict__ dqacc, int T, int H)
{
    dep_wait();
    dep_release();
    const int sub = threadIdx.x & 15, grp = threadIdx.x >> 4;
    const unsigned half = (threadIdx.x & 16) ? 0xFFFF0000u : 0x0000FFFFu;
    const int bh = static_cast<int>(blockIdx.x);   // b * H + h
    const int b = bh / H, h = bh - b * H;
    const int t0 = static_cast<int>(blockIdx.y) * kRowdotBlockRows + grp * kRowdotRows;
    float x[kRowdotRows][8], y[kRowdotRows][8];
#pragma unroll
    for (int u = 0; u < kRowdotRows; ++u)
    {
        const int t = t0 + u < T ? t0 + u : T - 1;   // rows past T: a valid row, result unused
        const int64_t bt = static_cast<int64_t>(b) * T + t;
        load16(o + bt * ldo + h * 128 + sub * 8, x[u]);
        load16(dout + bt * lddo + h * 128 + sub * 8, y[u]);
    }
    if (dqacc != nullptr)
    {
        // row (token b T + t, head h) of the fused path's dQ accumulator [B*T][H*128]
#pragma unroll
        for (int u = 0; u < kRowdotRows; ++u)
        {
            if (t0 + u < T)
            {
                float4* z = reinterpret_cast<float4*>(
                    dqacc + ((static_cast<int64_t>(b) * T + t0 + u) * H + h) * 128 + sub * 8);
                z[0] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                z[1] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
        }
    }
#pragma unroll
    for (int u = 0; u < kRowdotRows; ++u)
    {
        float s = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) s += x[u][e] * y[u][e];
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) s += __shfl_xor_sync(half, s, off);
        if (sub == 0 && t0 + u < T)
        {
            const int64_t at = static_cast<int64_t>(bh) * T + t0 + u;
            dvec[at] = s;
            nlse2[at] = -lse[at] * kLog2e;
        }
    }
}

dim3 rowdot_grid(int64_t B, int64_t T, int64_t H)
{
    return dim3(static_cast<unsigned>(B * H), static_cast<unsigned>((T + kRowdotBlockRows - 1) / kRowdotBlockRows));
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                             cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
        {
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
        }
    });
    return fn;
}

// [B, T, width] bf16 view of a token-major operand with row stride ld; box 64 columns x `rows`.
bool make_map3(CUtensorMap* map, const void* base, int64_t width, int64_t T, int64_t B, int64_t ld,
               uint32_t rows)
{
    auto fn = encode_fn();
    if (fn == nullptr)
    {
        return false;
    }
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(T),
                                static_cast<cuuint64_t>(B)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * 2,
                                   static_cast<cuuint64_t>(ld) * 2 * static_cast<cuuint64_t>(T)};
    const cuuint32_t box[3] = {64, rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [B, T, width] fp32 (row stride width) with a box of 32 columns (128-byte rows, 128-byte swizzle
// in shared memory) x box_rows rows, for bulk reduce-adds from shared memory.
bool make_map3_f32(CUtensorMap* map, void* base, int64_t width, int64_t T, int64_t B,
                   uint32_t box_w, uint32_t box_rows)
{
    auto fn = encode_fn();
    if (fn == nullptr)
    {
        return false;
    }
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(T),
                                static_cast<cuuint64_t>(B)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(width) * 4,
                                   static_cast<cuuint64_t>(width) * 4 * static_cast<cuuint64_t>(T)};
    const cuuint32_t box[3] = {box_w, box_rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

} // namespace

// Which backward serves bf16 / head_dim 128: 0 the fused kernel (the default), 1 the two-kernel
// path whose dQ is bit-reproducible. Process-wide; VEDA_ATTENTION_DETERMINISTIC=1 sets 1 at load.
std::atomic<int> g_attn_deterministic{[] {
    const char* v = std::getenv("VEDA_ATTENTION_DETERMINISTIC");
    return (v != nullptr && v[0] == '1') ? 1 : 0;
}()};

int attention_deterministic() { return g_attn_deterministic.load(std::memory_order_relaxed); }

int attn_tc_fwd(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                void* o, int64_t ldo, float* lse, int64_t B, int64_t T, int64_t H, int64_t Hkv,
                float scale, int causal, cudaStream_t s)
{
    CUtensorMap mq, mk, mv;
    if (!make_map3(&mq, q, H * 128, T, B, ldq, kTq) || !make_map3(&mk, k, Hkv * 128, T, B, ldk, kTk) ||
        !make_map3(&mv, v, Hkv * 128, T, B, ldv, kTk))
    {
        return -1;   // caller falls back
    }
    static int configured = -1;
    int device = 0;
    cudaGetDevice(&device);
    if (configured != device)
    {
        cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kFwdSmem);
        configured = device;
    }
    FwdParams p{static_cast<bf16*>(o), lse, ldo, static_cast<int>(B), static_cast<int>(T),
                static_cast<int>(H), static_cast<int>(Hkv), scale * kLog2e, causal, device_status_ptr()};
    // persistent: one CTA per SM working through the (batch, head, query-tile pair) items
    const int64_t pairs = ((T + kTq - 1) / kTq + 1) / 2;
    const int64_t items = B * H * pairs;
    const unsigned grid = static_cast<unsigned>(items < compute_sms() ? items : compute_sms());
    return launch("veda_attention_fwd (tcgen05)", attn_fwd_tc_kernel, dim3(grid), dim3(kFwdThreads),
                  kFwdSmem, s, mq, mk, mv, p);
}

// Workspace of the tcgen05 backward after D: the fused path's fp32 dQ accumulator
// [B*T][H*128] (O(B H T)), or the deterministic path's dS^T [B*H][T][T] bf16 (O(B H T^2)); then
// -LSE log2(e) [B, H, T] fp32.
size_t tc_bwd_ds_bytes(int64_t B, int64_t T, int64_t H)
{
    const size_t bytes =
        attention_deterministic()
            ? static_cast<size_t>(B * H) * static_cast<size_t>(T) * static_cast<size_t>(T) * sizeof(bf16)
            : static_cast<size_t>(B * T * H) * 128 * sizeof(float);
    return (bytes + 255) & ~static_cast<size_t>(255);
}

size_t tc_bwd_extra_workspace(int64_t B, int64_t T, int64_t H)
{
    return tc_bwd_ds_bytes(B, T, H) + static_cast<size_t>(B * H * T) * sizeof(float);
}

int attn_tc_bwd(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                const void* o, int64_t ldo, const void* dout, int64_t lddo, const float* lse,
                void* dq, int64_t lddq, void* dk, int64_t lddk, void* dv, int64_t lddv, float* dvec,
                void* extra, int64_t B, int64_t T, int64_t H, int64_t Hkv, float scale, int causal,
                cudaStream_t s)
{
    // dS^T rows are T bf16 wide: the tensor map needs their byte stride to be a multiple of 16,
    // and the per-tile -LSE / D bulk copies whole 32-byte pieces.
    if (T % 8 != 0 || B * H > 65535)
    {
        return -1;
    }
    // Q and dO tiles: 128 query rows for the fused kernel, 64 for the two-kernel path
    const bool det = attention_deterministic() != 0;
    if (det && dq == nullptr)
    {
        return -1;   // only the fused kernel leaves dQ in an fp32 accumulator
    }
    const uint32_t qrows = det ? kBq : kFq;
    CUtensorMap mq, mk, mv, mdo, mds;
    if (!make_map3(&mq, q, H * 128, T, B, ldq, qrows) || !make_map3(&mk, k, Hkv * 128, T, B, ldk, 128) ||
        !make_map3(&mv, v, Hkv * 128, T, B, ldv, 128) ||
        !make_map3(&mdo, dout, H * 128, T, B, lddo, qrows) || !aligned16(dvec) || !aligned16(extra) ||
        (det && !make_map3(&mds, extra, T, T, B * H, T, 128)))
    {
        return -1;   // caller falls back
    }
    static int configured = -1;
    int device = 0;
    cudaGetDevice(&device);
    if (configured != device)
    {
        cudaFuncSetAttribute(attn_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBwdSmem);
        cudaFuncSetAttribute(attn_bwd_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kFusedSmem);
        cudaFuncSetAttribute(attn_dq_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDqSmem);
        configured = device;
    }
    float* nlse2 = reinterpret_cast<float*>(static_cast<char*>(extra) + tc_bwd_ds_bytes(B, T, H));
    const dim3 grid(static_cast<unsigned>(B * Hkv), static_cast<unsigned>((T + 127) / 128));
    if (!det)
    {
        float* dqacc = static_cast<float*>(extra);
        CUtensorMap mdq;
        if (!make_map3_f32(&mdq, dqacc, H * 128, T, B, 32, 32))
        {
            return -1;
        }
        int rc = launch("veda_attention_bwd (D)", attn_rowdot_kernel, rowdot_grid(B, T, H), dim3(256), 0,
                        s, static_cast<const bf16*>(o), ldo, static_cast<const bf16*>(dout), lddo,
                        lse, dvec, nlse2, dqacc, static_cast<int>(T), static_cast<int>(H));
        if (rc != VEDA_OK)
        {
            return rc;
        }
        // pairs per chunk: as many as keep a chunk's Q, dO (2 x 256 B) and dQ accumulator rows
        // (512 B) per query and head within ~48 MB of L2, a power of two from 8 (fewer leaves a
        // long tail of key-tile-0 CTAs) up to all pairs
        const int64_t per_pair = 1024 * (H / Hkv) * T;
        int chunk = 8;
        while (chunk < B * Hkv && static_cast<int64_t>(chunk) * 2 * per_pair <= (48ll << 20)) chunk *= 2;
        FusedParams p{nlse2, dvec, static_cast<bf16*>(dk), static_cast<bf16*>(dv), lddk, lddv,
                      static_cast<int>(T), static_cast<int>(H), static_cast<int>(Hkv), scale,
                      scale * kLog2e, causal, device_status_ptr(),
                      static_cast<int>(std::min<int64_t>(chunk, B * Hkv))};
        rc = launch("veda_attention_bwd (tcgen05, fused)", attn_bwd_fused_kernel, grid,
                    dim3(kFusedThreads), kFusedSmem, s, mq, mk, mv, mdo, mdq, p);
        if (rc != VEDA_OK || dq == nullptr)
        {
            return rc;   // dq == nullptr: the caller reads dQ / scale from the fp32 accumulator
        }
        return launch("veda_attention_bwd (dQ cast)", attn_dq_cast_kernel,
                      dim3(grid_for(B * T * H * 16, 256)), dim3(256), 0, s,
                      static_cast<const float*>(dqacc), static_cast<bf16*>(dq), lddq, B * T, H * 128,
                      scale);
    }
    bf16* ds = static_cast<bf16*>(extra);
    const int rc = launch("veda_attention_bwd (D)", attn_rowdot_kernel, rowdot_grid(B, T, H), dim3(256),
                          0, s, static_cast<const bf16*>(o), ldo, static_cast<const bf16*>(dout), lddo,
                          lse, dvec, nlse2, static_cast<float*>(nullptr), static_cast<int>(T),
                          static_cast<int>(H));
    if (rc != VEDA_OK)
    {
        return rc;
    }
    BwdParams p{nlse2, dvec, static_cast<bf16*>(dk), static_cast<bf16*>(dv), ds, lddk, lddv,
                static_cast<int>(T), static_cast<int>(H), static_cast<int>(Hkv), scale,
                scale * kLog2e, causal, device_status_ptr()};
    attn_bwd_tc_kernel<<<grid, kBwdThreads, kBwdSmem, s>>>(mq, mk, mv, mdo, mds, p);
    DqParams pq{static_cast<bf16*>(dq), lddq, static_cast<int>(T), static_cast<int>(H),
                static_cast<int>(Hkv), static_cast<int>(B), scale, causal, device_status_ptr()};
    const int64_t dq_items = B * H * ((T + 127) / 128);
    const unsigned gq = static_cast<unsigned>(dq_items < compute_sms() ? dq_items : compute_sms());
    attn_dq_tc_kernel<<<gq, 192, kDqSmem, s>>>(mds, mk, pq);
    count_launch(2);
    return check_launch("veda_attention_bwd (tcgen05)");
}

} // namespace veda::cuda
