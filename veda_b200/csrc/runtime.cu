// Library-wide state of libveda_cuda.so: the per-thread error message, the launch counter and
// the cached device properties.
#include "common.cuh"
#include "tc_common.cuh"

#include <cstdlib>
#include <mutex>



namespace veda::cuda
{

namespace
{
thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};
int g_sm_count[64] = {0};
} // namespace

void set_error(const std::string& message) { g_last_error = message; }

int fail(int code, const std::string& message)
{
    g_last_error = message;
    return code;
}

int check_launch(const char* what)
{
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess)
    {
        return fail(VEDA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
    }
    return VEDA_OK;
}

void count_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

bool overlapped_launches()
{
    static const bool on = [] {
        const char* v = std::getenv("VEDA_PDL");
        return !(v != nullptr && v[0] == '0');
    }();
    return on;
}

uint64_t g_launches_value() { return g_launches.load(std::memory_order_relaxed); }

int sm_count()
{
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64)
    {
        return 148;
    }
    if (g_sm_count[device] == 0)
    {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
        g_sm_count[device] = n > 0 ? n : 148;
    }
    return g_sm_count[device];
}

// SMs the persistent kernels leave free (veda_set_reserved_sms).
std::atomic<int> g_reserved_sms{0};

int compute_sms()
{
    const int n = sm_count() - g_reserved_sms.load(std::memory_order_relaxed);
    return n < 2 ? 2 : n;
}

const char* last_error_cstr() { return g_last_error.c_str(); }

namespace
{
// The status word itself: a file-scope device variable, so every GPU that loads the library has
// its own copy, zero when the module loads, and no call ever allocates it.
__device__ int g_device_status;
} // namespace

// Device address of the current device's status word: kernels whose bounded waits give up write
// VEDA_ERR_TIMEOUT there instead of spinning forever. The address is looked up with
// cudaGetSymbolAddress while the device is current (host code cannot use the variable's name as
// a device pointer) and cached per device for the life of the process; a context destroyed by
// cudaDeviceReset leaves the cached address stale, so a reset needs a fresh process.
int* device_status_ptr()
{
    static int* ptrs[64] = {nullptr};
    static std::mutex mu;
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64)
    {
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (ptrs[device] == nullptr)
    {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_status) == cudaSuccess)
        {
            ptrs[device] = static_cast<int*>(p);
        }
    }
    return ptrs[device];
}

} // namespace veda::cuda

extern "C" int veda_kernel_status(int reset)
{
    int* p = veda::cuda::device_status_ptr();
    if (p == nullptr)
    {
        return veda::cuda::fail(VEDA_ERR_CUDA, "veda_kernel_status: no device status word");
    }
    int value = 0;
    if (cudaMemcpy(&value, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    {
        return veda::cuda::fail(VEDA_ERR_CUDA, "veda_kernel_status: read failed");
    }
    if (reset)
    {
        cudaMemset(p, 0, sizeof(int));
    }
    if (value != 0)
    {
        veda::cuda::set_error("a kernel's bounded wait gave up (device status word)");
    }
    return value;
}

namespace veda::cuda
{
namespace
{
// One CTA waits, through the same bounded mbarrier wait as the tensor-core and streaming kernels,
// on a barrier nothing arrives on; nothing else is in flight, so the timeout path can be taken
// safely. Every thread of the CTA waits (as the consumer warps of those kernels do).
__global__ void wait_timeout_check_kernel(long long budget, int* status)
{
    __shared__ uint64_t bar;
    __shared__ int abort;
    if (threadIdx.x == 0)
    {
        abort = 0;
        tc::mbar_init(&bar, 1);
        tc::mbar_fence_init();
    }
    __syncthreads();
    tc::mbar_wait(&bar, 0, status, &abort, budget);
}
} // namespace
} // namespace veda::cuda

extern "C" int veda_wait_timeout_check(long long budget_cycles, veda_stream_t stream)
{
    VEDA_REQUIRE(budget_cycles > 0 && budget_cycles <= veda::cuda::tc::kWaitBudget,
                 "budget must lie in (0, 2^32] cycles");
    int* status = veda::cuda::device_status_ptr();
    VEDA_REQUIRE(status != nullptr, "no device status word");
    veda::cuda::wait_timeout_check_kernel<<<1, 128, 0, stream>>>(budget_cycles, status);
    veda::cuda::count_launch();
    return veda::cuda::check_launch("veda_wait_timeout_check");
}

extern "C" const char* veda_last_error(void) { return veda::cuda::last_error_cstr(); }

extern "C" uint64_t veda_launch_count(void)
{
    return veda::cuda::g_launches_value();
}

extern "C" int veda_device_info(int* sm, int* major, int* minor)
{
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess)
    {
        return veda::cuda::fail(VEDA_ERR_CUDA, "veda_device_info: no CUDA device");
    }
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess)
    {
        return veda::cuda::fail(VEDA_ERR_CUDA, "veda_device_info: cudaGetDeviceProperties failed");
    }
    if (sm) *sm = prop.multiProcessorCount;
    if (major) *major = prop.major;
    if (minor) *minor = prop.minor;
    return VEDA_OK;
}

extern "C" int veda_set_reserved_sms(int n)
{
    return veda::cuda::g_reserved_sms.exchange(n < 0 ? 0 : n);
}
