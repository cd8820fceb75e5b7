// pkb_quantize_host_noalloc: pkb_quantize_host for callers that cannot
// allocate memory.
//
// Some callers cannot call cudaMalloc or cudaMallocHost at the time they
// quantize: an application that hands all of a GPU's memory to its own pool
// at start-up, or an audio callback that runs under a real-time deadline,
// where an allocation (which can synchronize the whole device and take
// milliseconds) is not allowed. This entry point uses no memory it allocates:
// its device staging is a fixed array, compiled into the library, that every
// GPU which loads the library holds until the process exits.
//
// The array holds one call's data: the float32 columns, the int8 bytes and
// the block scales, each region on a 256-byte boundary, PKB_NOALLOC_BYTES in
// all; a call that needs more is refused (PKB_EINVAL) before any work. Every
// call shares the array and finds the previous call's bytes in it; every byte
// a call reads it has written first, so nothing needs clearing. Two calls
// whose GPU work overlapped would race on the array: calls in this process
// take a lock and wait for their GPU work before returning, so they do not
// overlap.
//
// The array's device address is asked of the runtime once per device, with
// that device current, by the first call on the device; that first call
// should come before any stream capture the caller starts.

#include <cuda_runtime.h>

#include <mutex>

#include "../../include/pktito_b200.h"
#include "pkb_internal.h"

namespace {

// The fixed staging, on every device that loads the library.
static __device__ __align__(256) unsigned char g_noalloc_scratch[PKB_NOALLOC_BYTES];

constexpr int MAX_DEV = 16;

std::mutex g_noalloc_mu;
unsigned char* g_noalloc_ptr[MAX_DEV];  // the array's device address, per device
bool g_noalloc_ready[MAX_DEV];

int refuse(int code, const char* msg) { return pkb::set_error(code, "quantize (no allocation): %s", msg); }

size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

extern "C" int pkb_quantize_host_noalloc(int8_t* q, float* d, uint32_t n, uint32_t qb, uint32_t T, const float* x,
                                         size_t xs, int rmode) {
    if (n == 0 || n % 32 || n > PKB_MAX_N) return refuse(PKB_EINVAL, "n: a multiple of 32 up to PKB_MAX_N");
    if (qb == 0 || qb % 32 || n % qb) return refuse(PKB_EINVAL, "qb: a multiple of 32 dividing n");
    if (rmode < PKB_RN || rmode > PKB_RZ) return refuse(PKB_EINVAL, "rounding mode");
    if (!T) return PKB_OK;
    if (!q || !d || !x) return refuse(PKB_EINVAL, "null pointer");
    if (T > 1 && xs < n) return refuse(PKB_EINVAL, "column stride below n");
    if (T == 1) xs = n;  // one column reads no stride
    const size_t xbytes = static_cast<size_t>(T) * n * 4;
    const size_t qbytes = static_cast<size_t>(T) * n, dbytes = static_cast<size_t>(T) * (n / qb) * 4;
    const size_t off_q = up256(xbytes), off_d = off_q + up256(qbytes), need = off_d + dbytes;
    if (need > PKB_NOALLOC_BYTES)
        return refuse(PKB_EINVAL, "columns too large for the fixed staging (T * n * (5 + 4/qb) bytes, "
                                  "each part rounded up to 256, must fit in PKB_NOALLOC_BYTES)");

    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    // the device this thread's host-pointer calls run on
    // (pkb_set_thread_device), made current as every host-pointer call does
    const int dev = pkb::thread_device();
    if (dev < 0 || dev >= MAX_DEV) return refuse(PKB_ENODEV, "device out of range");
    if (cudaSetDevice(dev) != cudaSuccess) return refuse(PKB_ENODEV, "cudaSetDevice failed");
    int sms = 0;
    uint32_t* err_word = nullptr;
    // the library's own set-up of the device (kernel attributes, the error
    // word's address), once per device; allocates nothing
    if (const int rc = pkb::current_device_info(&sms, &err_word)) return rc;
    if (!g_noalloc_ready[dev]) {
        // once per device, with it current: the array's device address
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p)
            return refuse(PKB_ECUDA, "cudaGetSymbolAddress of the fixed staging failed");
        g_noalloc_ptr[dev] = static_cast<unsigned char*>(p);
        g_noalloc_ready[dev] = true;
    }
    unsigned char* base = g_noalloc_ptr[dev];
    float* dx = reinterpret_cast<float*>(base);
    int8_t* dq = reinterpret_cast<int8_t*>(base + off_q);
    float* dd = reinterpret_cast<float*>(base + off_d);
    cudaStream_t s = cudaStreamPerThread;
    // the columns, n floats each, straight from the caller's memory
    cudaError_t e = cudaMemcpy2DAsync(dx, static_cast<size_t>(n) * 4, x, xs * 4, static_cast<size_t>(n) * 4, T,
                                      cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) {
        e = pkb::launch_quantize(dq, dd, dx, n, T, n, qb, rmode, sms, s);
        if (e == cudaSuccess) pkb::count_launch();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(q, dq, qbytes, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d, dd, dbytes, cudaMemcpyDeviceToHost, s);
    // the device's error word, as every host-pointer call reads it
    uint32_t word = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&word, err_word, sizeof word, cudaMemcpyDeviceToHost, s);
    // on every path, the GPU work this call enqueued ends before the lock is
    // dropped: another call must not find the array still in use
    const cudaError_t e_sync = cudaStreamSynchronize(s);
    if (e == cudaSuccess) e = e_sync;
    if (e != cudaSuccess) return pkb::set_error(PKB_ECUDA, "quantize (no allocation): %s", cudaGetErrorString(e));
    pkb::count_host_bytes(static_cast<size_t>(T) * n * 4, qbytes + dbytes + sizeof word);
    if (word) {
        const uint32_t zero = 0;
        cudaMemcpy(err_word, &zero, sizeof zero, cudaMemcpyHostToDevice);
        return pkb::set_error(PKB_ETIMEOUT, "quantize (no allocation): device error word 0x%x", word);
    }
    return PKB_OK;
}
