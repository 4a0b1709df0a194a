// Self-test of the bounded waits every pipelined kernel relies on: a CTA
// waits on an mbarrier that nothing ever arrives on. The wait gives up after
// its poll / time limit (about 1 s), records `code` in the device error word
// and the kernel returns normally, so the context stays usable. This is the
// failure path of a lost producer, exercised without a GPU fault.
#include <cstdint>

#include "aic_common.cuh"
#include "aic_kernels.h"
#include "tc_ptx.cuh"

namespace aic {
namespace {

__global__ void selftest_wait_kernel(int* err, int code, int* returned)
{
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        tc::mbar_init(tc::smem_addr(&bar), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const bool done = tc::mbar_wait(tc::smem_addr(&bar), 0u, err, code);  // never completes
        *returned = done ? 2 : 1;
    }
}

}  // namespace

cudaError_t launch_selftest_wait(int code, int* returned, cudaStream_t stream)
{
    int* err = device_error_word();
    if (!err) return cudaErrorInvalidValue;
    selftest_wait_kernel<<<1, 32, 0, stream>>>(err, code, returned);
    return cudaGetLastError();
}

}  // namespace aic
