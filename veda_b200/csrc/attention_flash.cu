// Tiled tensor-core attention kernels (bf16, head_dim 128). Not yet enabled.
#include "attention.cuh"

namespace veda::cuda
{
const bool kFlashReady = false;

size_t flash_bwd_extra_workspace(int64_t, int64_t, int64_t, int64_t, int64_t) { return 0; }

int flash_fwd(const void*, int64_t, const void*, int64_t, const void*, int64_t, void*, int64_t,
              float*, int64_t, int64_t, int64_t, int64_t, float, int, cudaStream_t)
{
    return fail(VEDA_ERR_UNSUPPORTED, "flash_fwd: not built");
}

int flash_bwd(const void*, int64_t, const void*, int64_t, const void*, int64_t, const void*,
              int64_t, const void*, int64_t, const float*, void*, int64_t, void*, int64_t, void*,
              int64_t, float*, void*, int64_t, int64_t, int64_t, int64_t, float, int, cudaStream_t)
{
    return fail(VEDA_ERR_UNSUPPORTED, "flash_bwd: not built");
}
} // namespace veda::cuda
