// A self-test of the failure path every kernel of this library shares: a
// wait on an mbarrier that nothing will ever complete runs out after its
// bounded time, the kernel sets the device-side error word's timeout bit and
// returns, and the context stays usable. No copy, tensor-memory allocation
// or trap is involved, so the test cannot fault or hang the GPU.

#include <stdio.h>

#include "pkb_device.cuh"
#include "pkb_internal.h"
#include "pkb_vmath.cuh"
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

// Every float with bits in [lo, hi): the sigmoids' reciprocal (rcp_batch, on
// a thread's pair of neighbouring floats, as the producers call it) against
// the correctly rounded one (rcp_r: CUDA's __frcp_r*), counting the floats
// whose bits differ and keeping the smallest such. Every thread of a warp
// runs the same number of passes, so the pair's vote sees the whole warp.
template <int RM>
__global__ void __launch_bounds__(256) rcp_selftest_kernel(uint32_t lo, uint32_t hi,
                                                           unsigned long long* mismatches, uint32_t* first_bad) {
    unsigned long long bad = 0;
    uint32_t first = 0xFFFFFFFFu;
    const uint64_t step = 2ull * gridDim.x * blockDim.x;
    const uint64_t passes = (hi - lo + step - 1) / step;
    for (uint64_t p = 0; p < passes; p++) {
        const uint64_t b0 = lo + p * step + 2ull * (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x);
        const uint32_t ba = static_cast<uint32_t>(b0 < hi ? b0 : lo);
        const uint32_t bb = static_cast<uint32_t>(b0 + 1 < hi ? b0 + 1 : lo);
        const float ya = __uint_as_float(ba), yb = __uint_as_float(bb);
        const float den[2] = {ya, yb};
        float rec[2];
        rcp_batch<RM, 2>(den, rec);
        const float ra = rec[0], rb = rec[1];
        if (b0 < hi && __float_as_uint(ra) != __float_as_uint(rcp_r<RM>(ya))) {
            bad++;
            first = min(first, ba);
        }
        if (b0 + 1 < hi && __float_as_uint(rb) != __float_as_uint(rcp_r<RM>(yb))) {
            bad++;
            first = min(first, bb);
        }
    }
    if (bad) {
        atomicAdd(mismatches, bad);
        atomicMin(first_bad, first);
    }
}

__device__ unsigned long long g_rcp_mismatches;
__device__ uint32_t g_rcp_first_bad;

}  // namespace
}  // namespace pkb

using namespace pkb;

extern "C" int pkb_rcp_selftest(int rmode, uint32_t lo_bits, uint32_t hi_bits, uint64_t* mismatches,
                                uint32_t* first_bad) {
    if (rmode < PKB_RN || rmode > PKB_RZ) return set_error(PKB_EINVAL, "rcp self-test: rounding mode %d", rmode);
    if (lo_bits < 0x3F800000u || hi_bits > 0x7F800000u || lo_bits >= hi_bits)
        return set_error(PKB_EINVAL, "rcp self-test: [0x%08x, 0x%08x) outside [1, 2^128)", lo_bits, hi_bits);
    int sms = 0;
    uint32_t* err = nullptr;
    int rc = current_device_info(&sms, &err);
    if (rc) return rc;
    const unsigned long long zero = 0;
    const uint32_t none = 0xFFFFFFFFu;
    cudaError_t e = cudaMemcpyToSymbol(g_rcp_mismatches, &zero, sizeof zero);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_rcp_first_bad, &none, sizeof none);
    unsigned long long* dm = nullptr;
    uint32_t* df = nullptr;
    if (e == cudaSuccess) e = cudaGetSymbolAddress(reinterpret_cast<void**>(&dm), g_rcp_mismatches);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(reinterpret_cast<void**>(&df), g_rcp_first_bad);
    if (e == cudaSuccess) {
        const dim3 grid(static_cast<unsigned>(sms * 8)), block(256);
        switch (rmode) {
        case 1: rcp_selftest_kernel<1><<<grid, block, 0, cudaStreamPerThread>>>(lo_bits, hi_bits, dm, df); break;
        case 2: rcp_selftest_kernel<2><<<grid, block, 0, cudaStreamPerThread>>>(lo_bits, hi_bits, dm, df); break;
        case 3: rcp_selftest_kernel<3><<<grid, block, 0, cudaStreamPerThread>>>(lo_bits, hi_bits, dm, df); break;
        default: rcp_selftest_kernel<0><<<grid, block, 0, cudaStreamPerThread>>>(lo_bits, hi_bits, dm, df); break;
        }
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(cudaStreamPerThread);
    unsigned long long m = 0;
    uint32_t f = 0;
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&m, g_rcp_mismatches, sizeof m);
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&f, g_rcp_first_bad, sizeof f);
    if (e != cudaSuccess) return set_error(PKB_ECUDA, "rcp self-test: %s", cudaGetErrorString(e));
    count_launch();
    if (mismatches) *mismatches = m;
    if (first_bad) *first_bad = f;
    return PKB_OK;
}

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
