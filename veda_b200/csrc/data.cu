// Device side of the corpus batcher: the [B, T] input and target windows of one batch gathered
// from the device-resident corpus, the window starts drawn on the device.
//
// The reference (src/libs/data/Corpus.cpp:64-107) draws one start per row from a splitmix64
// stream: state += 0x9E3779B97F4A7C15, output = mix(state), start = begin + output % offsets.
// The k-th draw of a batch depends only on the state before the batch plus (k + 1) increments,
// so every row's start is computed independently here; the host advances the state by B
// increments per batch. Integer arithmetic only: the windows are bit-identical to the reference's.
#include "common.cuh"

namespace veda::cuda
{
namespace
{

constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

// splitmix64's output function (the published generator's finaliser)
__device__ __forceinline__ uint64_t splitmix_mix(uint64_t z)
{
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void corpus_gather_kernel(const int64_t* __restrict__ ids, uint64_t state, int64_t begin,
                                     uint64_t offsets, int64_t batch, int64_t length,
                                     int64_t* __restrict__ inputs, int64_t* __restrict__ targets)
{
    const int64_t total = batch * length;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    {
        const int64_t row = i / length, t = i % length;
        const uint64_t draw = splitmix_mix(state + static_cast<uint64_t>(row + 1) * kGolden);
        const int64_t start = begin + static_cast<int64_t>(draw % offsets);
        inputs[i] = ids[start + t];
        targets[i] = ids[start + t + 1];
    }
}

} // namespace
} // namespace veda::cuda

using namespace veda::cuda;

extern "C" int veda_corpus_gather(const int64_t* ids, int64_t begin, int64_t end, uint64_t state,
                                  int64_t batch, int64_t length, int64_t* inputs, int64_t* targets,
                                  veda_stream_t stream)
{
    VEDA_REQUIRE(batch > 0 && length > 0, "batch size and length must be positive");
    VEDA_REQUIRE(begin >= 0 && end >= begin, "bad split range");
    VEDA_REQUIRE(end - begin >= length + 1, "the split holds fewer ids than one window");
    VEDA_REQUIRE(ids != nullptr && inputs != nullptr && targets != nullptr, "null pointer");
    const uint64_t offsets = static_cast<uint64_t>(end - begin - (length + 1) + 1);
    corpus_gather_kernel<<<grid_for(batch * length, 256), 256, 0, stream>>>(
        ids, state, begin, offsets, batch, length, inputs, targets);
    count_launch();
    return check_launch("veda_corpus_gather");
}
