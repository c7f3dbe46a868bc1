// Shared device and host helpers of libveda_cuda.so (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <string>
#include <utility>

#include "veda_cuda.h"

namespace veda::cuda
{

using bf16 = __nv_bfloat16;

// ---- host: status and error reporting ------------------------------------------------------
void set_error(const std::string& message);
int fail(int code, const std::string& message);
int check_launch(const char* what);
void count_launch(uint64_t n = 1);
int sm_count();
// SMs a persistent kernel may use: sm_count() less those reserved by veda_set_reserved_sms.
int compute_sms();
uint64_t g_launches_value();
const char* last_error_cstr();

#define VEDA_REQUIRE(cond, msg)                                                                   \
    do                                                                                            \
    {                                                                                             \
        if (!(cond))                                                                              \
        {                                                                                         \
            return ::veda::cuda::fail(VEDA_ERR_INVALID_ARGUMENT, std::string(__func__) + ": " +   \
                                                                     (msg));                      \
        }                                                                                         \
    } while (0)

inline bool valid_dtype(int d) { return d == VEDA_F32 || d == VEDA_BF16; }
inline size_t dtype_size(int d) { return d == VEDA_BF16 ? 2 : 4; }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---- overlapped (programmatic dependent) launches -------------------------------------------
// A kernel started by launch() may begin while the kernel before it on the stream is still
// running, so that its launch and its set-up (shared memory, mbarriers, TMEM allocation) hide
// under the tail of its predecessor. Such a kernel must touch no global memory before
// dep_wait(), which returns once the predecessor has completed and its writes are visible; after
// it, dep_release() lets the kernel's own successor start early. A kernel launched without the
// attribute (or one whose predecessor never releases) sees both as no-ops. VEDA_PDL=0 launches
// without the attribute.
__device__ __forceinline__ void dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void dep_release()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

bool overlapped_launches();

template <typename... Params, typename... Args>
int launch(const char* what, void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
           cudaStream_t s, Args&&... args)
{
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = overlapped_launches() ? 1 : 0;
    count_launch();
    const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
    if (err != cudaSuccess)
    {
        cudaGetLastError();
        return fail(VEDA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
    }
    return check_launch(what);
}

inline unsigned grid_for(int64_t work, int threads, int per_sm = 8)
{
    int64_t blocks = (work + threads - 1) / threads;
    const int64_t cap = static_cast<int64_t>(sm_count()) * per_sm;
    if (blocks > cap)
    {
        blocks = cap;
    }
    return static_cast<unsigned>(blocks < 1 ? 1 : blocks);
}

// ---- device: element conversion -----------------------------------------------------------
__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(bf16 x) { return __bfloat162float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x)
{
    return x;
}
template <>
__device__ __forceinline__ bf16 from_f32<bf16>(float x)
{
    return __float2bfloat16_rn(x);
}

// 16-byte vectors: 4 floats or 8 bf16.
template <typename T>
struct Vec16
{
    static constexpr int N = 16 / sizeof(T);
};

template <typename T>
__device__ __forceinline__ void load16(const T* p, float (&out)[16 / sizeof(T)])
{
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    if constexpr (sizeof(T) == 4)
    {
        out[0] = __uint_as_float(raw.x);
        out[1] = __uint_as_float(raw.y);
        out[2] = __uint_as_float(raw.z);
        out[3] = __uint_as_float(raw.w);
    }
    else
    {
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
        {
            out[2 * i] = __uint_as_float(w[i] << 16);
            out[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        }
    }
}

template <typename T>
__device__ __forceinline__ void store16(T* p, const float (&in)[16 / sizeof(T)])
{
    uint4 raw;
    if constexpr (sizeof(T) == 4)
    {
        raw.x = __float_as_uint(in[0]);
        raw.y = __float_as_uint(in[1]);
        raw.z = __float_as_uint(in[2]);
        raw.w = __float_as_uint(in[3]);
    }
    else
    {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
        {
            const __nv_bfloat162 pair = __floats2bfloat162_rn(in[2 * i], in[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t*>(&pair);
        }
        raw = make_uint4(w[0], w[1], w[2], w[3]);
    }
    *reinterpret_cast<uint4*>(p) = raw;
}

// ---- device: packed fp32 pairs (sm_100: one f32x2 instruction does the work of two) ---------
__device__ __forceinline__ uint64_t pk(float a, float b)
{
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void upk(uint64_t v, float& a, float& b)
{
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c)
{
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b)
{
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b)
{
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// the 8 bf16 of a 16-byte chunk as four fp32 pairs
__device__ __forceinline__ void unpack4x2(const uint4& raw, uint64_t (&o)[4])
{
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = pk(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xFFFF0000u));
}

// ---- device: reductions --------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
    {
        v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    }
    return v;
}

__device__ __forceinline__ double warp_sum(double v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
    {
        v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    }
    return v;
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
    {
        v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    }
    return v;
}

} // namespace veda::cuda
