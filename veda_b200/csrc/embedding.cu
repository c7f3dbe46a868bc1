// Embedding gather and scatter-add (src/libs/autograd/NonLinear.cpp:203-254).
//
// Forward: out[p] = table[ids[p]], a bit-exact copy, one warp per position with 16-byte moves.
// Backward, two modes:
//   deterministic  positions are sorted by (id, position) in shared memory (bitonic sort of
//                  (id << 32 | position) keys, up to kChunk positions per pass; longer inputs are
//                  processed chunk after chunk in position order), then one warp per distinct id
//                  adds that id's rows onto dtable[id] one position after another in ascending
//                  order — the order of the reference's loop (NonLinear.cpp:245-252), so given
//                  equal inputs the result is equal bit for bit;
//   atomic         fp32 atomicAdd per element (order unspecified, fastest).
#include "common.cuh"

namespace veda::cuda
{
namespace
{

constexpr int kChunk = 16384;          // positions sorted per pass (128 KB of keys in smem)
constexpr int kSortThreads = 1024;

template <typename T>
__global__ void gather_kernel(const int64_t* __restrict__ ids, int64_t count,
                              const T* __restrict__ table, int64_t vocab, int64_t dim,
                              T* __restrict__ out, int64_t ldo, int* status, bool vec)
{
    const int lane = threadIdx.x & 31;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    constexpr int V = Vec16<T>::N;
    for (int64_t p = warp; p < count; p += warps)
    {
        const int64_t id = ids[p];
        T* dst = out + p * ldo;
        if (id < 0 || id >= vocab)
        {
            if (lane == 0 && status != nullptr)
            {
                *status = VEDA_ERR_OUT_OF_RANGE;
            }
            for (int64_t d = lane; d < dim; d += 32)
            {
                dst[d] = from_f32<T>(0.0f);
            }
            continue;
        }
        const T* src = table + id * dim;
        if (vec)
        {
            for (int64_t d = static_cast<int64_t>(lane) * V; d < dim; d += 32 * V)
            {
                *reinterpret_cast<uint4*>(dst + d) = *reinterpret_cast<const uint4*>(src + d);
            }
        }
        else
        {
            for (int64_t d = lane; d < dim; d += 32)
            {
                dst[d] = src[d];
            }
        }
    }
}

template <typename T>
__global__ void scatter_atomic_kernel(const int64_t* __restrict__ ids, int64_t count,
                                      const T* __restrict__ dout, int64_t ldd, int64_t vocab,
                                      int64_t dim, float* __restrict__ dtable)
{
    const int64_t total = count * dim;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        const int64_t p = idx / dim;
        const int64_t d = idx - p * dim;
        const int64_t id = ids[p];
        if (id >= 0 && id < vocab)
        {
            atomicAdd(dtable + id * dim + d, to_f32(dout[p * ldd + d]));
        }
    }
}

// Sorts the keys (id << 32 | position-in-chunk) of one chunk in shared memory; padding keys are
// all-ones so they sort last. Writes the sorted keys to `sorted`.
__global__ void __launch_bounds__(kSortThreads)
sort_chunk_kernel(const int64_t* __restrict__ ids, int64_t first, int n, int64_t vocab,
                  uint64_t* __restrict__ sorted)
{
    extern __shared__ uint64_t keys[];
    int size = 1;
    while (size < n)
    {
        size <<= 1;
    }
    for (int i = threadIdx.x; i < size; i += blockDim.x)
    {
        uint64_t k = ~0ull;
        if (i < n)
        {
            const int64_t id = ids[first + i];
            // out-of-range ids sort last and are ignored by the apply kernel
            const uint64_t idk = (id >= 0 && id < vocab) ? static_cast<uint64_t>(id) : 0xFFFFFFFFull;
            k = (idk << 32) | static_cast<uint32_t>(i);
        }
        keys[i] = k;
    }
    __syncthreads();
    for (int k = 2; k <= size; k <<= 1)
    {
        for (int j = k >> 1; j > 0; j >>= 1)
        {
            for (int i = threadIdx.x; i < size; i += blockDim.x)
            {
                const int partner = i ^ j;
                if (partner > i)
                {
                    const bool ascending = (i & k) == 0;
                    const uint64_t a = keys[i], b = keys[partner];
                    if ((a > b) == ascending)
                    {
                        keys[i] = b;
                        keys[partner] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x)
    {
        sorted[i] = keys[i];
    }
}

// One warp per segment start: adds the segment's rows in position order onto
// dtable[id - id_lo] for ids in [id_lo, id_hi) (the others are skipped).
template <typename T>
__global__ void apply_segments_kernel(const uint64_t* __restrict__ sorted, int n, int64_t first,
                                      const T* __restrict__ dout, int64_t ldd, int64_t dim,
                                      float* __restrict__ dtable, int64_t id_lo, int64_t id_hi)
{
    const int lane = threadIdx.x & 31;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    for (int64_t e = warp; e < n; e += warps)
    {
        const uint64_t key = sorted[e];
        const uint32_t id = static_cast<uint32_t>(key >> 32);
        if (id == 0xFFFFFFFFu || static_cast<int64_t>(id) < id_lo || static_cast<int64_t>(id) >= id_hi)
        {
            continue;
        }
        if (e > 0 && static_cast<uint32_t>(sorted[e - 1] >> 32) == id)
        {
            continue;   // not the first position of its id
        }
        int64_t end = e + 1;
        while (end < n && static_cast<uint32_t>(sorted[end] >> 32) == id)
        {
            ++end;
        }
        float* row = dtable + (static_cast<int64_t>(id) - id_lo) * dim;
        for (int64_t d = lane; d < dim; d += 32)
        {
            float acc = row[d];
            for (int64_t q = e; q < end; ++q)
            {
                const int64_t p = first + static_cast<int64_t>(static_cast<uint32_t>(sorted[q]));
                acc = __fadd_rn(acc, to_f32(dout[p * ldd + d]));
            }
            row[d] = acc;
        }
    }
}

} // namespace
} // namespace veda::cuda

using namespace veda::cuda;

extern "C" int veda_embedding_fwd(const int64_t* ids, int64_t count, const void* table,
                                  int64_t vocab, int64_t dim, void* out, int64_t ldo, int* status,
                                  int dtype, veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype), "unknown dtype");
    VEDA_REQUIRE(count >= 0 && vocab > 0 && dim > 0 && ldo >= dim, "bad shape");
    if (count == 0)
    {
        return VEDA_OK;
    }
    VEDA_REQUIRE(ids && table && out, "null pointer");
    const size_t es = dtype_size(dtype);
    const int64_t v = 16 / static_cast<int64_t>(es);
    const bool vec = aligned16(table) && aligned16(out) && dim % v == 0 && ldo % v == 0;
    const unsigned grid = grid_for(count * 32, 256);
    if (dtype == VEDA_BF16)
    {
        gather_kernel<bf16><<<grid, 256, 0, stream>>>(ids, count, static_cast<const bf16*>(table),
                                                      vocab, dim, static_cast<bf16*>(out), ldo,
                                                      status, vec);
    }
    else
    {
        gather_kernel<float><<<grid, 256, 0, stream>>>(ids, count,
                                                       static_cast<const float*>(table), vocab,
                                                       dim, static_cast<float*>(out), ldo, status,
                                                       vec);
    }
    count_launch();
    return check_launch("veda_embedding_fwd");
}

extern "C" size_t veda_embedding_bwd_workspace(int64_t count)
{
    const int64_t n = count < kChunk ? count : kChunk;
    return static_cast<size_t>(n > 0 ? n : 1) * sizeof(uint64_t);
}

extern "C" int veda_embedding_bwd(const int64_t* ids, int64_t count, const void* dout, int64_t ldd,
                                  int64_t vocab, int64_t dim, float* dtable, int deterministic,
                                  void* workspace, size_t workspace_bytes, int dtype,
                                  veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype), "unknown dtype");
    VEDA_REQUIRE(count >= 0 && vocab > 0 && dim > 0 && ldd >= dim, "bad shape");
    VEDA_REQUIRE(vocab < 0xFFFFFFFFll, "vocabulary too large");
    if (count == 0)
    {
        return VEDA_OK;
    }
    VEDA_REQUIRE(ids && dout && dtable, "null pointer");
    if (!deterministic)
    {
        const unsigned grid = grid_for(count * dim, 256);
        if (dtype == VEDA_BF16)
        {
            scatter_atomic_kernel<bf16><<<grid, 256, 0, stream>>>(
                ids, count, static_cast<const bf16*>(dout), ldd, vocab, dim, dtable);
        }
        else
        {
            scatter_atomic_kernel<float><<<grid, 256, 0, stream>>>(
                ids, count, static_cast<const float*>(dout), ldd, vocab, dim, dtable);
        }
        count_launch();
        return check_launch("veda_embedding_bwd");
    }
    VEDA_REQUIRE(workspace != nullptr && workspace_bytes >= veda_embedding_bwd_workspace(count),
                 "workspace too small (see veda_embedding_bwd_workspace)");
    uint64_t* sorted = static_cast<uint64_t*>(workspace);
    static bool configured = false;
    if (!configured)
    {
        cudaFuncSetAttribute(sort_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kChunk * static_cast<int>(sizeof(uint64_t)));
        configured = true;
    }
    for (int64_t first = 0; first < count; first += kChunk)
    {
        const int n = static_cast<int>(count - first < kChunk ? count - first : kChunk);
        int size = 1;
        while (size < n)
        {
            size <<= 1;
        }
        sort_chunk_kernel<<<1, kSortThreads, size * sizeof(uint64_t), stream>>>(ids, first, n,
                                                                                vocab, sorted);
        const unsigned grid = grid_for(static_cast<int64_t>(n) * 32, 256);
        if (dtype == VEDA_BF16)
        {
            apply_segments_kernel<bf16><<<grid, 256, 0, stream>>>(
                sorted, n, first, static_cast<const bf16*>(dout), ldd, dim, dtable, 0, vocab);
        }
        else
        {
            apply_segments_kernel<float><<<grid, 256, 0, stream>>>(
                sorted, n, first, static_cast<const float*>(dout), ldd, dim, dtable, 0, vocab);
        }
        count_launch(2);
    }
    return check_launch("veda_embedding_bwd");
}

extern "C" int veda_embedding_sort(const int64_t* ids, int64_t count, int64_t vocab,
                                   uint64_t* keys, veda_stream_t stream)
{
    VEDA_REQUIRE(count >= 0 && count <= kChunk, "count must lie in [0, 16384]");
    VEDA_REQUIRE(vocab > 0 && vocab < 0xFFFFFFFFll, "bad vocabulary");
    if (count == 0)
    {
        return VEDA_OK;
    }
    VEDA_REQUIRE(ids != nullptr && keys != nullptr, "null pointer");
    static bool configured = false;
    if (!configured)
    {
        cudaFuncSetAttribute(sort_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kChunk * static_cast<int>(sizeof(uint64_t)));
        configured = true;
    }
    const int n = static_cast<int>(count);
    int size = 1;
    while (size < n)
    {
        size <<= 1;
    }
    sort_chunk_kernel<<<1, kSortThreads, size * sizeof(uint64_t), stream>>>(ids, 0, n, vocab, keys);
    count_launch();
    return check_launch("veda_embedding_sort");
}

extern "C" int veda_embedding_apply_sorted(const uint64_t* keys, int64_t count, const void* dout,
                                           int64_t ldd, int64_t dim, int64_t id_lo, int64_t id_hi,
                                           float* dtable, int dtype, veda_stream_t stream)
{
    VEDA_REQUIRE(valid_dtype(dtype), "unknown dtype");
    VEDA_REQUIRE(count >= 0 && count <= kChunk, "count must lie in [0, 16384]");
    VEDA_REQUIRE(dim > 0 && ldd >= dim && id_lo >= 0 && id_hi >= id_lo, "bad shape");
    if (count == 0 || id_hi == id_lo)
    {
        return VEDA_OK;
    }
    VEDA_REQUIRE(keys != nullptr && dout != nullptr && dtable != nullptr, "null pointer");
    const int n = static_cast<int>(count);
    const unsigned grid = grid_for(static_cast<int64_t>(n) * 32, 256);
    if (dtype == VEDA_BF16)
    {
        apply_segments_kernel<bf16><<<grid, 256, 0, stream>>>(
            keys, n, 0, static_cast<const bf16*>(dout), ldd, dim, dtable, id_lo, id_hi);
    }
    else
    {
        apply_segments_kernel<float><<<grid, 256, 0, stream>>>(
            keys, n, 0, static_cast<const float*>(dout), ldd, dim, dtable, id_lo, id_hi);
    }
    count_launch();
    return check_launch("veda_embedding_apply_sorted");
}
