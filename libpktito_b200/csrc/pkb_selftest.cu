// A self-test of the failure path every kernel of this library shares: a
// wait on an mbarrier that nothing will ever complete runs out after its
// bounded time, the kernel sets the device-side error word's timeout bit and
// returns, and the context stays usable. No copy, tensor-memory allocation
// or trap is involved, so the test cannot fault or hang the GPU.

#include <stdio.h>

#include "pkb_device.cuh"
#include "pkb_internal.h"
#include "pktito_b200.h"

namespace pkb {
namespace {

__device__ uint32_t g_selftest_gave_up;  // 1 once the wait gave up

__global__ void __launch_bounds__(32) wait_selftest_kernel(uint32_t* err, long long limit) {
    __shared__ uint64_t bar;
    __shared__ int abort;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);  // one arrival completes phase 0; none comes
        abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    const bool ok = mbar_wait(&bar, 0, &abort, limit);
    if (!ok && threadIdx.x == 0) {
        atomicOr(err, PKB_DEVERR_TIMEOUT);
        g_selftest_gave_up = 1;
    }
}

}  // namespace
}  // namespace pkb

using namespace pkb;

extern "C" int pkb_wait_selftest(uint64_t limit_cycles, int* gave_up) {
    if (limit_cycles < 1000 || limit_cycles > (1ull << 31))
        return set_error(PKB_EINVAL, "wait self-test: limit %llu cycles outside [1000, 2^31]",
                         static_cast<unsigned long long>(limit_cycles));
    int sms = 0;
    uint32_t* err = nullptr;
    int rc = current_device_info(&sms, &err);
    if (rc) return rc;
    const uint32_t zero = 0;
    cudaError_t e = cudaMemcpyToSymbol(g_selftest_gave_up, &zero, sizeof zero);
    if (e == cudaSuccess) {
        wait_selftest_kernel<<<1, 32, 0, cudaStreamPerThread>>>(err, static_cast<long long>(limit_cycles));
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(cudaStreamPerThread);
    uint32_t flag = 0;
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&flag, g_selftest_gave_up, sizeof flag);
    if (e != cudaSuccess) return set_error(PKB_ECUDA, "wait self-test: %s", cudaGetErrorString(e));
    count_launch();
    if (gave_up) *gave_up = flag ? 1 : 0;
    return PKB_OK;
}
