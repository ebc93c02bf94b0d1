// Failure-detection self-test: a kernel whose mbarrier wait can never complete (nothing arrives on the barrier) must
// give up after its cycle budget, record kErrWaitTimeout in the device error word and end, leaving the context
// usable. It exercises the same bounded wait (mbar_wait) that every pipeline wait in the library uses.
#include "common.hpp"
#include "ptx.cuh"

namespace h3 {
namespace {

__global__ void wait_selftest_kernel(long long budget)
{
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    // Phase 0 never completes: no thread arrives.
    if (threadIdx.x == 0)
        mbar_wait(&bar, 0, budget);
    __syncthreads();
}

} // namespace

void wait_selftest(long long budget_cycles, cudaStream_t s)
{
    if (budget_cycles <= 0 || budget_cycles > 4000000000ll)
        throw CudaError("wait_selftest: the budget must be within (0, 4e9] cycles");
    wait_selftest_kernel<<<1, 32, 0, s>>>(budget_cycles);
    H3_CUDA(cudaGetLastError());
}

} // namespace h3
