// Host-side helpers shared by the kernels' launchers: CUDA error checks that throw, tensor-map encoding through the
// driver entry point (no link-time dependency on libcuda), and the launch-parameter structs of every kernel.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <atomic>
#include <cstdint>
#include <stdexcept>
#include <string>

namespace h3 {

struct CudaError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

inline void cuda_check(cudaError_t e, const char* what)
{
    if (e != cudaSuccess)
        throw CudaError(std::string(what) + ": " + cudaGetErrorString(e));
}
#define H3_CUDA(x) ::h3::cuda_check((x), #x)

// A 2-D or 3-D row-major tensor described for TMA: dims[0] is the contiguous extent, strides in bytes for dims 1..
// `box` gives the tile copied per load (box[0] * element size must be 128 bytes for the 128-byte swizzle).
CUtensorMap make_tmap(CUtensorMapDataType type, int rank, const void* base, const uint64_t* dims, const uint64_t* strides_bytes,
                      const uint32_t* box, bool swizzle128 = true);

// Reads and clears the device error word (nonzero: a kernel's bounded wait ran out or a shape check failed).
uint32_t take_device_error(cudaStream_t s);

int num_sms();

// One bit for the current device (devices 0-63), for per-device one-time set-up.
uint64_t device_bit();

// Raises a kernel's dynamic shared-memory limit to `bytes` once per device: the opt-in belongs to the kernel in each
// device's context, so a process that drives several GPUs needs it on every one. Setting it twice is harmless, so
// the flag is only marked after the call.
template <class Kernel>
void smem_opt_in(Kernel* kernel, int bytes, std::atomic<uint64_t>& done)
{
    const uint64_t bit = device_bit();
    if (done.load(std::memory_order_acquire) & bit)
        return;
    cuda_check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes), "cudaFuncSetAttribute");
    done.fetch_or(bit, std::memory_order_release);
}

// True when a kernel may dereference p: device or managed memory, or pinned host memory mapped into the device's
// address space (null counts as accessible; callers check their own required arguments).
bool device_accessible(const void* p);

// Queues the bounded-wait self-test (a wait on an mbarrier nothing arrives on, given up after budget_cycles).
void wait_selftest(long long budget_cycles, cudaStream_t s);

} // namespace h3
