// Failure detection without a GPU fault: every spin in the library's kernels
// is an mbarrier wait bounded by a globaltimer limit, after which the kernel
// records a code in the device status word and returns.  This self-test runs
// that path on purpose: one thread waits, with a short limit, on an mbarrier
// that nothing arrives at.  The wait must give up, the status word must carry
// kErrTimeoutProbe, and the context must stay usable.
#include "kernels.h"
#include "ptx.cuh"

namespace s3t {

namespace {

__global__ void wait_timeout_probe(int* status, uint64_t limit_ns, int* gave_up) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);   // expects one arrival; none comes
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) *gave_up = mbar_wait_limit(&bar, 0, status, kErrTimeoutProbe, nullptr, limit_ns) ? 0 : 1;
}

}  // namespace

cudaError_t launch_wait_timeout_probe(int* status, uint64_t limit_ns, int* gave_up, cudaStream_t stream) {
    wait_timeout_probe<<<1, 32, 0, stream>>>(status, limit_ns, gave_up);
    return cudaGetLastError();
}

}  // namespace s3t
