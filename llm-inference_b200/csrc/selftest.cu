// Self-test of the kernels' bounded waits: a wait that nothing will ever complete must give up
// after its time limit, record DEV_ERR_WAIT_TIMEOUT in the device error word and return, leaving
// the context usable. The kernel here runs the same wait primitive the pipelined kernels use
// (mbar_wait, common.cuh) on an mbarrier whose phase never completes: one thread arrives with an
// expected transaction count that no copy will ever deliver. Nothing faults, traps or hangs:
// the wait ends at WAIT_LIMIT_NS.
#include "common.cuh"

namespace q3 {
namespace {

__device__ unsigned g_dev_error;

__global__ void wait_timeout_kernel(int *done) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    fence_barrier_init();
    mbar_arrive_expect_tx(&bar, 16);  // 16 bytes that no copy brings: phase 0 never completes
    const bool ok = mbar_wait(&bar, 0, &g_dev_error);
    *done = ok ? 1 : 2;
}

}  // namespace

unsigned take_error_selftest() {
    unsigned v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(v)) != cudaSuccess) return 0;
    if (v) cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(zero));
    return v;
}

}  // namespace q3

// Runs one wait that must time out (about WAIT_LIMIT_NS, two seconds) on `stream`; *done (device
// memory) becomes 2 when the wait gave up, 1 if it had completed. q3_device_error then reports
// Q3_DEV_ERR_WAIT_TIMEOUT.
extern "C" int q3_selftest_wait_timeout(int *done, void *stream) {
    if (!done) return Q3_ERR_ARG;
    q3::wait_timeout_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(done);
    return q3::record_cuda_error(cudaGetLastError());
}
