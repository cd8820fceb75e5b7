// The host-pointer contract of libpktito's backend table
// (backend/kernels.h:47-78): pkb_quantize_host, pkb_gemm_q8_host,
// pkb_forget, pkb_set_thread_device.
//
// A call gets host pointers and returns when its results are in host memory,
// so its cost is mostly copies: the inputs up over PCIe, the results back. A
// call is cut into chunks of frames and run as a pipeline over two slots of
// pinned and device staging: while chunk c's inputs go up (one stream) and
// chunk c-1's results come down (another), the kernels of the chunk between
// run on a third, and the host copies the next chunk's inputs into pinned
// memory and the last chunk's results out of it. The host copies are split
// over a pool of worker threads (one thread's memcpy reaches about a fifth of
// what a B200 host's memory and PCIe can move).
//
// Where the caller's activations and results are page-locked (cudaMallocHost
// or cudaHostRegister: an engine whose buffers live as long as it does can
// pin them once), a call skips the host copies: each chunk is copied by DMA
// straight from and into the caller's memory, and the call's only host-side
// wait is the last.
//
// Calls arrive synchronously from any number of the caller's threads at once
// (the reference's pool calls a backend from every worker, core/pool.c:
// 115-122, on disjoint outputs): each calling thread has its own streams and
// staging, grown as needed and kept; matrices are uploaded once per device
// and shared, indexed by host address range, the slices of one matrix
// absorbed into one device copy, and every call checks sampled lines of its
// weights against the bytes uploaded (the matrices section below).

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <functional>
#include <memory>
#include <map>
#include <mutex>
#include <shared_mutex>
#include <thread>
#include <vector>

#include "../../include/pktito_b200.h"
#include "pkb_internal.h"

namespace pkb {
namespace {

constexpr int MAX_DEV = 16;

int cuda_err(cudaError_t e, const char* what) {
    return set_error(e == cudaErrorMemoryAllocation ? PKB_ENOMEM : PKB_ECUDA, "%s: %s", what,
                     cudaGetErrorString(e));
}

#define HOST_CUDA(call, what)                                \
    do {                                                     \
        cudaError_t e_ = (call);                             \
        if (e_ != cudaSuccess) return cuda_err(e_, what);    \
    } while (0)

size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

// ------------------------------------------------------------- copy pool --

// Worker threads that split a large host copy (or comparison) between them
// and the calling thread. Jobs from several calling threads queue up.
class CopyPool {
  public:
    static CopyPool& get() {
        static CopyPool pool;
        return pool;
    }

    // rows of `bytes` each from src (pitch spitch) to dst (pitch dpitch)
    void copy2d(void* dst, size_t dpitch, const void* src, size_t spitch, size_t bytes, size_t rows) {
        const size_t total = bytes * rows;
        if (!rows || !bytes) return;
        if (dpitch == bytes && spitch == bytes) {  // one run
            copy(dst, src, total);
            return;
        }
        const int parts = split(total, rows);
        run(parts, [=](int p) {
            const size_t r0 = rows * p / parts, r1 = rows * (p + 1) / parts;
            for (size_t r = r0; r < r1; r++)
                memcpy(static_cast<char*>(dst) + r * dpitch, static_cast<const char*>(src) + r * spitch, bytes);
        });
    }

    void copy(void* dst, const void* src, size_t bytes) {
        const int parts = split(bytes, bytes / 4096 + 1);
        run(parts, [=](int p) {
            const size_t b0 = (bytes * p / parts) & ~size_t(63), b1 = p + 1 == parts ? bytes : (bytes * (p + 1) / parts) & ~size_t(63);
            memcpy(static_cast<char*>(dst) + b0, static_cast<const char*>(src) + b0, b1 - b0);
        });
    }

    bool equal(const void* a, const void* b, size_t bytes) {
        std::atomic<bool> same{true};
        const int parts = split(bytes, bytes / 4096 + 1);
        run(parts, [&](int p) {
            const size_t b0 = (bytes * p / parts) & ~size_t(63), b1 = p + 1 == parts ? bytes : (bytes * (p + 1) / parts) & ~size_t(63);
            if (same.load(std::memory_order_relaxed) &&
                memcmp(static_cast<const char*>(a) + b0, static_cast<const char*>(b) + b0, b1 - b0))
                same = false;
        });
        return same;
    }

  private:
    struct Job {
        std::function<void(int)> fn;
        int parts;
        std::atomic<int> next{0}, done{0};
    };

    std::vector<std::thread> workers_;
    std::mutex mu_;
    std::condition_variable cv_;
    std::deque<std::shared_ptr<Job>> queue_;
    int nthreads_ = 0;

    CopyPool() {
        unsigned hw = std::thread::hardware_concurrency();
        int n = hw ? static_cast<int>(hw) : 4;
        if (n > 16) n = 16;
        if (const char* e = getenv("PKB_HOST_THREADS")) n = atoi(e);
        if (n < 1) n = 1;
        nthreads_ = n;
        for (int i = 1; i < n; i++) workers_.emplace_back([this] { work(); });  // the caller is the n-th
    }
    ~CopyPool() {
        {
            std::lock_guard<std::mutex> lock(mu_);
            queue_.push_back(nullptr);  // stop
        }
        cv_.notify_all();
        for (auto& t : workers_) t.join();
    }

    // parts worth splitting into: about 1 MB each, at most one per thread
    int split(size_t bytes, size_t units) const {
        size_t parts = bytes / (1u << 20);
        if (parts > static_cast<size_t>(nthreads_)) parts = nthreads_;
        if (parts > units) parts = units;
        return parts < 1 ? 1 : static_cast<int>(parts);
    }

    static void take(Job& j) {
        for (int p; (p = j.next.fetch_add(1)) < j.parts;) {
            j.fn(p);
            j.done.fetch_add(1, std::memory_order_acq_rel);
        }
    }

    void run(int parts, std::function<void(int)> fn) {
        if (parts <= 1 || workers_.empty()) {
            fn(0);
            return;
        }
        auto job = std::make_shared<Job>();
        job->fn = std::move(fn);
        job->parts = parts;
        {
            std::lock_guard<std::mutex> lock(mu_);
            queue_.push_back(job);
        }
        cv_.notify_all();
        take(*job);
        while (job->done.load(std::memory_order_acquire) < parts) std::this_thread::yield();
        std::lock_guard<std::mutex> lock(mu_);
        for (auto it = queue_.begin(); it != queue_.end(); ++it)
            if (*it == job) {
                queue_.erase(it);
                break;
            }
    }

    void work() {
        for (;;) {
            std::shared_ptr<Job> job;
            {
                std::unique_lock<std::mutex> lock(mu_);
                cv_.wait(lock, [this] {
                    if (!queue_.empty() && !queue_.front()) return true;
                    for (auto& j : queue_)
                        if (j && j->next.load() < j->parts) return true;
                    return false;
                });
                if (!queue_.front()) return;
                for (auto& j : queue_)
                    if (j && j->next.load() < j->parts) {
                        job = j;
                        break;
                    }
            }
            if (job) take(*job);
        }
    }
};

// ------------------------------------------------------------- staging --

// One calling thread's pipeline on its device: three streams, two slots of
// pinned and device staging each way, and the events that order them.
struct Pipe {
    int dev = -1;
    cudaStream_t s_in = nullptr, s_comp = nullptr, s_out = nullptr;
    cudaEvent_t ev_in[2] = {}, ev_comp[2] = {}, ev_out[2] = {};
    uint8_t* pin_in[2] = {};
    uint8_t* pin_out[2] = {};
    uint8_t* dev_in[2] = {};
    uint8_t* dev_out[2] = {};
    size_t in_cap = 0, out_cap = 0;
    uint8_t* pin_vec = nullptr;  // row scales and biases going up
    uint8_t* dev_vec = nullptr;
    size_t vec_cap = 0;
    uint32_t* herr = nullptr;    // the device error word, read back

    ~Pipe() { release(); }

    void release() {
        if (dev < 0) return;
        int cur = -1;
        if (cudaGetDevice(&cur) != cudaSuccess) return;  // the runtime is gone at exit
        cudaSetDevice(dev);
        for (cudaStream_t s : {s_in, s_comp, s_out})
            if (s) cudaStreamDestroy(s);
        for (int i = 0; i < 2; i++) {
            for (cudaEvent_t e : {ev_in[i], ev_comp[i], ev_out[i]})
                if (e) cudaEventDestroy(e);
            if (pin_in[i]) cudaFreeHost(pin_in[i]);
            if (pin_out[i]) cudaFreeHost(pin_out[i]);
            if (dev_in[i]) cudaFree(dev_in[i]);
            if (dev_out[i]) cudaFree(dev_out[i]);
        }
        if (pin_vec) cudaFreeHost(pin_vec);
        if (dev_vec) cudaFree(dev_vec);
        if (herr) cudaFreeHost(herr);
        *this = Pipe();
        if (cur >= 0) cudaSetDevice(cur);
    }

    int open(int device) {
        if (dev == device) return PKB_OK;
        release();
        HOST_CUDA(cudaSetDevice(device), "cudaSetDevice");
        dev = device;
        for (cudaStream_t* s : {&s_in, &s_comp, &s_out})
            HOST_CUDA(cudaStreamCreateWithFlags(s, cudaStreamNonBlocking), "cudaStreamCreate");
        for (int i = 0; i < 2; i++)
            for (cudaEvent_t* e : {&ev_in[i], &ev_comp[i], &ev_out[i]})
                HOST_CUDA(cudaEventCreateWithFlags(e, cudaEventDisableTiming), "cudaEventCreate");
        HOST_CUDA(cudaMallocHost(&herr, sizeof(uint32_t)), "cudaMallocHost");
        // the activation copies come from the device's stream-ordered pool:
        // it keeps what is freed instead of returning it at every sync
        cudaMemPool_t pool;
        if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
            uint64_t keep_all = UINT64_MAX;
            cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep_all);
        }
        return PKB_OK;
    }

    // slots of at least in_bytes / out_bytes each way, and vec_bytes of vectors
    int reserve(size_t in_bytes, size_t out_bytes, size_t vec_bytes) {
        if (in_bytes > in_cap) {
            const size_t want = up256(in_bytes + in_bytes / 4);
            for (int i = 0; i < 2; i++) {
                if (pin_in[i]) cudaFreeHost(pin_in[i]);
                if (dev_in[i]) cudaFree(dev_in[i]);
                pin_in[i] = dev_in[i] = nullptr;
            }
            in_cap = 0;
            for (int i = 0; i < 2; i++) {
                HOST_CUDA(cudaMallocHost(&pin_in[i], want), "cudaMallocHost (staging)");
                HOST_CUDA(cudaMalloc(&dev_in[i], want), "cudaMalloc (staging)");
            }
            in_cap = want;
        }
        if (out_bytes > out_cap) {
            const size_t want = up256(out_bytes + out_bytes / 4);
            for (int i = 0; i < 2; i++) {
                if (pin_out[i]) cudaFreeHost(pin_out[i]);
                if (dev_out[i]) cudaFree(dev_out[i]);
                pin_out[i] = dev_out[i] = nullptr;
            }
            out_cap = 0;
            for (int i = 0; i < 2; i++) {
                HOST_CUDA(cudaMallocHost(&pin_out[i], want), "cudaMallocHost (staging)");
                HOST_CUDA(cudaMalloc(&dev_out[i], want), "cudaMalloc (staging)");
            }
            out_cap = want;
        }
        if (vec_bytes > vec_cap) {
            const size_t want = up256(vec_bytes + vec_bytes / 4);
            if (pin_vec) cudaFreeHost(pin_vec);
            if (dev_vec) cudaFree(dev_vec);
            pin_vec = dev_vec = nullptr;
            vec_cap = 0;
            HOST_CUDA(cudaMallocHost(&pin_vec, want), "cudaMallocHost (staging)");
            HOST_CUDA(cudaMalloc(&dev_vec, want), "cudaMalloc (staging)");
            vec_cap = want;
        }
        return PKB_OK;
    }

    // All three streams drained; the device error word read and cleared.
    int finish(uint32_t* err_word) {
        HOST_CUDA(cudaMemcpyAsync(herr, err_word, sizeof(uint32_t), cudaMemcpyDeviceToHost, s_out), "error word read");
        count_host_bytes(0, sizeof(uint32_t));
        HOST_CUDA(cudaStreamSynchronize(s_in), "cudaStreamSynchronize");
        HOST_CUDA(cudaStreamSynchronize(s_comp), "cudaStreamSynchronize");
        HOST_CUDA(cudaStreamSynchronize(s_out), "cudaStreamSynchronize");
        if (*herr) {
            const uint32_t w = *herr;
            cudaMemsetAsync(err_word, 0, sizeof(uint32_t), s_out);
            cudaStreamSynchronize(s_out);
            return set_error(PKB_ETIMEOUT, "a kernel gave up waiting (device error word 0x%x)", w);
        }
        return PKB_OK;
    }
};

thread_local int tl_device = 0;
thread_local Pipe tl_pipe;

// Drains a pipe's streams when a call returns early (an error after work
// was enqueued), so that nothing the call enqueued still runs when the
// memory it uses (an activation copy, weights) may be freed.
struct DrainOnReturn {
    Pipe* p;
    ~DrainOnReturn() {
        if (!p) return;
        for (cudaStream_t st : {p->s_in, p->s_comp, p->s_out})
            if (st) cudaStreamSynchronize(st);
    }
};

// Whether [p, p + bytes) is page-locked host memory (both of its ends: a
// range that is not wholly so is still copied correctly, only not at DMA
// speed).
bool pinned(const void* p, size_t bytes) {
    if (!p || !bytes) return false;
    for (const void* q : {p, static_cast<const void*>(static_cast<const char*>(p) + bytes - 1)}) {
        cudaPointerAttributes a;
        if (cudaPointerGetAttributes(&a, q) != cudaSuccess) {
            cudaGetLastError();  // clears the error it may leave
            return false;
        }
        if (a.type != cudaMemoryTypeHost) return false;
    }
    return true;
}

// A chunk's frames: its input and output bytes per frame kept near these
// sizes, in whole tiles of 128 frames where the call has that many.
#ifndef PKB_CHUNK_MB
#define PKB_CHUNK_MB 16
#endif
constexpr size_t CHUNK_IN = size_t(PKB_CHUNK_MB) << 20, CHUNK_OUT = size_t(2 * PKB_CHUNK_MB) << 20;

uint32_t chunk_frames(uint32_t T, size_t in_per_frame, size_t out_per_frame) {
    size_t tc = CHUNK_IN / (in_per_frame ? in_per_frame : 1);
    const size_t to = CHUNK_OUT / (out_per_frame ? out_per_frame : 1);
    if (to < tc) tc = to;
    tc = tc / 128 * 128;
    if (tc < 128) tc = 128;
    return tc >= T ? T : static_cast<uint32_t>(tc);
}

// ------------------------------------------------------------- matrices --
//
// Weights are uploaded once per device and kept. A call names a run of whole
// 16-row panels (w at a panel boundary, rows a multiple of 16) of a PK_Q8
// matrix in host memory, often from inside it (the reference's passes call
// with w + r0 * cols, core/passes.c:60-72). The repack is panel-local: the
// rows of panel p, repacked, occupy the same bytes the panel did. So a device
// copy of host bytes [lo, hi) serves any call whose range lies inside it in
// the same panel phase, and the slices of one matrix, whatever their order
// and size, are absorbed into one device copy as they arrive: a slice next
// to or over an existing copy makes a copy of the union, the old rows moved
// device to device, only the new slice's bytes uploaded.
//
// Each call checks that its host bytes are still the ones uploaded by
// comparing sampled 64-byte lines with the host copy kept at upload (a
// fixed number a call, at positions that move from call to call, so the
// cost is O(1) and repeated calls cover the whole range; ranges up to
// FULL_CHECK bytes are compared whole). Bytes that differ retire the copy
// and the call uploads its range again. The reference's weights are a
// read-only mapping of the model file that lives until the model is freed;
// a caller that rewrites weights in place, or unmaps them, calls pkb_forget
// first.

constexpr size_t LINE = 64;              // bytes a sampled line
constexpr int SAMPLES = 32;              // lines checked a call
constexpr size_t FULL_CHECK = 256 << 10; // ranges compared whole up to this

// Device memory freed when the last call that uses it returns.
struct DevBuf {
    int dev = -1;
    int8_t* p = nullptr;
    ~DevBuf() {
        if (!p) return;
        int cur = -1;
        if (cudaGetDevice(&cur) != cudaSuccess) return;  // the runtime is gone at exit
        cudaSetDevice(dev);
        cudaFree(p);
        cudaSetDevice(cur);
    }
};

// A device copy of host bytes [lo, hi): panels of 16 rows of n, repacked.
struct Matrix {
    uintptr_t lo, hi;
    uint32_t n;
    std::shared_ptr<DevBuf> buf;
    std::atomic<uint32_t> probe{0};  // moves the sampled lines from call to call
};

// Host bytes as they were uploaded, in pieces over disjoint ranges.
struct Piece {
    uintptr_t hi;
    std::shared_ptr<std::vector<int8_t>> bytes;
};

struct DeviceCache {
    std::shared_mutex mu;  // the two maps
    std::map<uintptr_t, std::shared_ptr<Matrix>> mats;  // by lo; disjoint
    std::map<uintptr_t, Piece> pieces;                  // by lo; disjoint
    std::mutex upload_mu;  // one upload at a time on the device
};

DeviceCache g_cache[MAX_DEV];

// The matrix copy holding [a, a + bytes) of n-input rows in its panel
// phase, or null. Under at least a shared lock.
std::shared_ptr<Matrix> find_copy(DeviceCache& c, uintptr_t a, size_t bytes, uint32_t n) {
    auto it = c.mats.upper_bound(a);
    if (it == c.mats.begin()) return nullptr;
    --it;
    const std::shared_ptr<Matrix>& m = it->second;
    if (m->n != n || a + bytes > m->hi || (a - m->lo) % (16 * static_cast<size_t>(n))) return nullptr;
    return m;
}

// Whether host bytes [p, p + len) equal the uploaded ones. Under at least a
// shared lock.
bool same_as_uploaded(DeviceCache& c, uintptr_t p, size_t len) {
    while (len) {
        auto it = c.pieces.upper_bound(p);
        if (it == c.pieces.begin()) return false;
        --it;
        if (p >= it->second.hi) return false;
        const size_t take = std::min(len, static_cast<size_t>(it->second.hi - p));
        if (memcmp(reinterpret_cast<const void*>(p), it->second.bytes->data() + (p - it->first), take)) return false;
        p += take;
        len -= take;
    }
    return true;
}

bool still_uploaded(DeviceCache& c, Matrix& m, uintptr_t a, size_t bytes) {
    if (bytes <= FULL_CHECK) return same_as_uploaded(c, a, bytes);
    const size_t lines = bytes / LINE;
    const uint32_t k = m.probe.fetch_add(1, std::memory_order_relaxed);
    // the first and last lines, and lines spread evenly from an offset that
    // advances by a large odd step each call
    if (!same_as_uploaded(c, a, LINE) || !same_as_uploaded(c, a + bytes - LINE, LINE)) return false;
    const size_t stride = lines / (SAMPLES - 2);
    const size_t off = (static_cast<size_t>(k) * 0x9E3779B1u) % (stride ? stride : 1);
    for (int i = 0; i < SAMPLES - 2; i++) {
        const size_t line = off + i * stride;
        if (line >= lines) break;
        if (!same_as_uploaded(c, a + line * LINE, LINE)) return false;
    }
    return true;
}

// Drops the pieces' bytes over [lo, hi), keeping what lies outside. Under
// the exclusive lock.
void drop_pieces(DeviceCache& c, uintptr_t lo, uintptr_t hi) {
    auto it = c.pieces.upper_bound(lo);
    if (it != c.pieces.begin()) --it;
    std::vector<std::pair<uintptr_t, Piece>> keep;
    while (it != c.pieces.end() && it->first < hi) {
        const uintptr_t plo = it->first, phi = it->second.hi;
        if (phi <= lo) {
            ++it;
            continue;
        }
        const int8_t* src = it->second.bytes->data();
        if (plo < lo)
            keep.push_back({plo, Piece{lo, std::make_shared<std::vector<int8_t>>(src, src + (lo - plo))}});
        if (phi > hi)
            keep.push_back({hi, Piece{phi, std::make_shared<std::vector<int8_t>>(src + (hi - plo), src + (phi - plo))}});
        it = c.pieces.erase(it);
    }
    for (auto& k : keep) c.pieces.emplace(k.first, std::move(k.second));
}

// The device rows for `rows` rows of the PK_Q8 matrix at host address w (a
// run of whole panels, possibly from inside a matrix), and the copy that
// holds them, which the caller keeps until its kernels have run.
int weights_for(Pipe& p, const int8_t* w, uint32_t rows, uint32_t n, const int8_t** wpack,
                std::shared_ptr<Matrix>* hold) {
    DeviceCache& c = g_cache[p.dev];
    const uintptr_t a = reinterpret_cast<uintptr_t>(w);
    const size_t bytes = static_cast<size_t>(rows) * n, panel = 16 * static_cast<size_t>(n);
    {
        std::shared_lock<std::shared_mutex> lock(c.mu);
        std::shared_ptr<Matrix> m = find_copy(c, a, bytes, n);
        if (m && still_uploaded(c, *m, a, bytes)) {
            *wpack = m->buf->p + (a - m->lo);
            *hold = std::move(m);
            return PKB_OK;
        }
    }
    std::lock_guard<std::mutex> up(c.upload_mu);
    std::vector<std::shared_ptr<Matrix>> merge;  // the copies the new one absorbs
    {
        std::unique_lock<std::shared_mutex> lock(c.mu);
        // another thread may have uploaded it meanwhile
        std::shared_ptr<Matrix> m = find_copy(c, a, bytes, n);
        if (m && still_uploaded(c, *m, a, bytes)) {
            *wpack = m->buf->p + (a - m->lo);
            *hold = std::move(m);
            return PKB_OK;
        }
        if (m) {  // its bytes changed: retire the copy and what was kept of its bytes
            drop_pieces(c, m->lo, m->hi);
            c.mats.erase(m->lo);
        }
        // copies that overlap or touch [a, a + bytes) in its panel phase
        // join it; any other overlapping copy (another n or phase) is retired
        auto it = c.mats.upper_bound(a);
        if (it != c.mats.begin()) --it;
        while (it != c.mats.end() && it->first <= a + bytes) {
            const std::shared_ptr<Matrix>& o = it->second;
            if (o->hi < a) {
                ++it;
                continue;
            }
            const bool joins = o->n == n && (a > o->lo ? a - o->lo : o->lo - a) % panel == 0;
            const bool overlaps = o->lo < a + bytes && a < o->hi;
            if (joins) {
                merge.push_back(o);
                it = c.mats.erase(it);
            } else if (overlaps) {
                drop_pieces(c, o->lo, o->hi);
                it = c.mats.erase(it);
            } else {
                ++it;
            }
        }
    }
    uintptr_t lo = a, hi = a + bytes;
    for (auto& o : merge) {
        lo = std::min(lo, o->lo);
        hi = std::max(hi, o->hi);
    }
    auto m = std::make_shared<Matrix>();
    m->lo = lo;
    m->hi = hi;
    m->n = n;
    m->buf = std::make_shared<DevBuf>();
    m->buf->dev = p.dev;
    HOST_CUDA(cudaMalloc(&m->buf->p, hi - lo), "cudaMalloc (weights)");
    // the absorbed copies' rows, device to device, then this range's panels
    // through slot 0's staging, repacked into place
    int rc = p.reserve(bytes, 0, 0);
    if (rc) return rc;
    HOST_CUDA(cudaStreamSynchronize(p.s_in), "cudaStreamSynchronize");
    HOST_CUDA(cudaStreamSynchronize(p.s_comp), "cudaStreamSynchronize");
    for (auto& o : merge)
        HOST_CUDA(cudaMemcpyAsync(m->buf->p + (o->lo - lo), o->buf->p, o->hi - o->lo, cudaMemcpyDeviceToDevice,
                                  p.s_comp),
                  "weights move");
    auto shadow = std::make_shared<std::vector<int8_t>>(bytes);
    CopyPool::get().copy(shadow->data(), w, bytes);
    CopyPool::get().copy(p.pin_in[0], shadow->data(), bytes);
    HOST_CUDA(cudaMemcpyAsync(p.dev_in[0], p.pin_in[0], bytes, cudaMemcpyHostToDevice, p.s_comp), "weights upload");
    count_host_bytes(bytes, 0);
    if ((rc = pkb_repack_q8_dev(p.s_comp, m->buf->p + (a - lo), reinterpret_cast<int8_t*>(p.dev_in[0]), rows, n)))
        return rc;
    HOST_CUDA(cudaStreamSynchronize(p.s_comp), "weights upload");
    {
        std::unique_lock<std::shared_mutex> lock(c.mu);
        drop_pieces(c, a, a + bytes);
        c.pieces.emplace(a, Piece{a + bytes, std::move(shadow)});
        c.mats.emplace(lo, m);
    }
    *wpack = m->buf->p + (a - lo);
    *hold = std::move(m);
    return PKB_OK;
}

// ----------------------------------------------------------- activations --
//
// A product reads activations that a quantize call of this library wrote a
// moment before: the reference's engine quantizes an input and then hands
// the same host q and d to every product (and every slice of a product,
// core/passes.c:60-109) that reads it. Each quantize call therefore keeps its
// result on the device, with a host copy of the bytes and scales it wrote;
// a product whose q and d lie inside one such result, at the same frames,
// compares the caller's bytes with that copy (the whole range, split over
// the copy pool) and, where they are the same, reads the device copy instead
// of uploading them again. Bytes that differ (anything else wrote there) fail
// the comparison and the call uploads them as usual, so the result is the
// same either way; what the cache saves is PCIe traffic, paid for with host
// memory reads. A new quantize call over the same host bytes replaces the
// old result. The device copies are capped (PKB_ACT_CACHE_MB, default 4096;
// 0 turns the cache off), the oldest dropped first; a dropped copy no call
// uses keeps its memory as a spare (capped the same) that a later quantize
// call of a size it holds takes over.
//
// A call whose frames lie inside those of a call still in progress that
// compared (or was itself covered so) skips the comparison: the caller may
// not change the inputs of a call before it returns, so those bytes are
// still the ones compared. The engine's slices of one column chunk (the
// same frames, other rows) then compare the chunk once.

struct ActCopy {
    uintptr_t q0, d0;      // host addresses of frame 0's bytes and scales
    uint32_t n, nb, T;
    int8_t* dq = nullptr;  // device [T][n]
    float* dd = nullptr;   // device [T][nb]
    size_t cap_q = 0, cap_d = 0;  // their sizes in bytes
    int dev = -1;
    std::vector<int8_t> hq;  // the host bytes and scales as written
    std::vector<float> hd;
    std::mutex live_mu;     // frame ranges [first, second) of the calls in progress that read this copy
    std::vector<std::pair<uint32_t, uint32_t>> live;
    ~ActCopy() {
        int cur = -1;
        if (cudaGetDevice(&cur) != cudaSuccess) return;
        cudaSetDevice(dev);
        if (dq) cudaFreeAsync(dq, cudaStreamPerThread);
        if (dd) cudaFreeAsync(dd, cudaStreamPerThread);
        cudaSetDevice(cur);
    }
};

struct ActCache {
    std::shared_mutex mu;
    std::map<uintptr_t, std::shared_ptr<ActCopy>> by_q;  // by q0; disjoint host ranges
    // insertion order, for eviction: each entry with the copy it named, so a
    // key inserted again is not evicted for its older self
    std::deque<std::pair<uintptr_t, const ActCopy*>> order;
    size_t bytes = 0;
    // Copies that left the cache while no call used them, kept with their
    // device and host memory for the next quantize call to take over: an
    // encoder quantizes the same shapes every forward pass, and a step's
    // results can outgrow the cap (FIFO then evicts every result before its
    // next use), so without this each step would allocate its copies again
    // and fault in and zero-fill fresh host pages for their comparison copies.
    std::deque<std::shared_ptr<ActCopy>> spares;  // oldest first
    size_t spare_bytes = 0;
};

ActCache g_acts[MAX_DEV];

size_t act_cache_cap() {
    static const size_t cap = [] {
        const char* e = getenv("PKB_ACT_CACHE_MB");
        return (e ? static_cast<size_t>(atoll(e)) : size_t(4096)) << 20;
    }();
    return cap;
}

size_t act_bytes(const ActCopy& a) { return static_cast<size_t>(a.T) * (a.n + 4 * a.nb); }
size_t act_held(const ActCopy& a) { return a.cap_q + a.cap_d + a.hq.capacity() + 4 * a.hd.capacity(); }

// A copy that left the cache (c.mu held): kept as a spare where no call
// uses it (the spares' memory capped as the cache is, the oldest freed
// first), else freed by the last call that does.
void act_retire(ActCache& c, std::shared_ptr<ActCopy> a) {
    if (!a || a.use_count() != 1 || !a->dq) return;
    c.spare_bytes += act_held(*a);
    c.spares.push_back(std::move(a));
    while (c.spare_bytes > act_cache_cap() && !c.spares.empty()) {
        c.spare_bytes -= act_held(*c.spares.front());
        c.spares.pop_front();
    }
}

// The smallest spare whose device memory holds qbytes of bytes and dbytes
// of scales, taken out of the spares; null where none does.
std::shared_ptr<ActCopy> act_take_spare(ActCache& c, size_t qbytes, size_t dbytes) {
    std::unique_lock<std::shared_mutex> lock(c.mu);
    auto best = c.spares.end();
    for (auto it = c.spares.begin(); it != c.spares.end(); ++it)
        if ((*it)->cap_q >= qbytes && (*it)->cap_d >= dbytes &&
            (best == c.spares.end() || (*it)->cap_q + (*it)->cap_d < (*best)->cap_q + (*best)->cap_d))
            best = it;
    if (best == c.spares.end()) return nullptr;
    std::shared_ptr<ActCopy> a = std::move(*best);
    c.spares.erase(best);
    c.spare_bytes -= act_held(*a);
    return a;
}

// Drops the results overlapping host bytes [q, q + qbytes) or scales
// [d, d + dbytes); those no call still uses become spares.
void act_forget(ActCache& c, uintptr_t q, size_t qbytes, uintptr_t d, size_t dbytes) {
    std::unique_lock<std::shared_mutex> lock(c.mu);
    for (auto it = c.by_q.begin(); it != c.by_q.end();) {
        const ActCopy& a = *it->second;
        const uintptr_t aq1 = a.q0 + static_cast<size_t>(a.T) * a.n, ad1 = a.d0 + static_cast<size_t>(a.T) * a.nb * 4;
        if ((a.q0 < q + qbytes && q < aq1) || (a.d0 < d + dbytes && d < ad1)) {
            c.bytes -= act_bytes(a);
            std::shared_ptr<ActCopy> gone = std::move(it->second);
            it = c.by_q.erase(it);
            act_retire(c, std::move(gone));
        } else {
            ++it;
        }
    }
}

// A call's hold on frames [f0, f0 + T) of a device copy, released when the
// call returns.
struct ActHold {
    std::shared_ptr<ActCopy> a;
    std::pair<uint32_t, uint32_t> range;
    ~ActHold() {
        if (!a) return;
        std::lock_guard<std::mutex> lock(a->live_mu);
        for (auto it = a->live.begin(); it != a->live.end(); ++it)
            if (*it == range) {
                a->live.erase(it);
                break;
            }
    }
};

// The device copy holding frames [f0, f0 + T) of q and d, after the caller's
// bytes there were found to be the ones written; null otherwise.
std::shared_ptr<ActCopy> act_find(int dev, const int8_t* q, const float* d, uint32_t n, uint32_t nb, uint32_t T,
                                  uint32_t* f0, ActHold* hold) {
    if (!act_cache_cap()) return nullptr;
    ActCache& c = g_acts[dev];
    std::shared_ptr<ActCopy> a;
    {
        std::shared_lock<std::shared_mutex> lock(c.mu);
        auto it = c.by_q.upper_bound(reinterpret_cast<uintptr_t>(q));
        if (it == c.by_q.begin()) return nullptr;
        a = std::prev(it)->second;
    }
    const uintptr_t qa = reinterpret_cast<uintptr_t>(q);
    if (a->n != n || a->nb != nb || (qa - a->q0) % n) return nullptr;
    const size_t f = (qa - a->q0) / n;
    if (f + T > a->T || reinterpret_cast<uintptr_t>(d) != a->d0 + f * nb * 4) return nullptr;
    const std::pair<uint32_t, uint32_t> range(static_cast<uint32_t>(f), static_cast<uint32_t>(f + T));
    bool covered = false;
    {
        std::lock_guard<std::mutex> lock(a->live_mu);
        for (const auto& r : a->live)
            if (r.first <= range.first && range.second <= r.second) covered = true;
        if (covered) a->live.push_back(range);
    }
    if (!covered) {
        // the caller's bytes and scales against the ones written
        CopyPool& pool = CopyPool::get();
        if (!pool.equal(q, a->hq.data() + f * n, static_cast<size_t>(T) * n) ||
            !pool.equal(d, a->hd.data() + f * nb, static_cast<size_t>(T) * nb * 4))
            return nullptr;
        std::lock_guard<std::mutex> lock(a->live_mu);
        a->live.push_back(range);
    }
    hold->a = a;
    hold->range = range;
    *f0 = static_cast<uint32_t>(f);
    return a;
}

int open_pipe(Pipe** out, uint32_t** err_word) {
    Pipe& p = tl_pipe;
    int rc = p.open(tl_device);
    if (rc) return rc;
    HOST_CUDA(cudaSetDevice(p.dev), "cudaSetDevice");
    int sms;
    if ((rc = current_device_info(&sms, err_word))) return rc;
    *out = &p;
    return PKB_OK;
}

int check_shape(uint32_t n, uint32_t qb, int rmode) {
    if (n == 0 || n % 32 || n > PKB_MAX_N) return set_error(PKB_EINVAL, "n = %u: a multiple of 32 up to %u", n, PKB_MAX_N);
    if (qb == 0 || qb % 32 || n % qb) return set_error(PKB_EINVAL, "qb = %u: a multiple of 32 dividing n = %u", qb, n);
    if (rmode < PKB_RN || rmode > PKB_RZ) return set_error(PKB_EINVAL, "rounding mode %d", rmode);
    return PKB_OK;
}

}  // namespace

int thread_device() { return tl_device; }

}  // namespace pkb

using namespace pkb;

extern "C" {

int pkb_set_thread_device(int device) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n || device >= MAX_DEV)
        return set_error(PKB_ENODEV, "device %d is not present", device);
    tl_device = device;
    return PKB_OK;
}

int pkb_quantize_host(int8_t* q, float* d, uint32_t n, uint32_t qb, uint32_t T, const float* x, size_t xs,
                      int rmode) {
    int rc = check_shape(n, qb, rmode);
    if (rc) return rc;
    if (!T) return PKB_OK;
    if (!q || !d || !x) return set_error(PKB_EINVAL, "quantize: null pointer");
    // column t at x + t xs: one column reads no stride
    if (T > 1 && xs < n) return set_error(PKB_EINVAL, "quantize: column stride %zu below n = %u", xs, n);
    if (T == 1) xs = n;
    Pipe* p;
    uint32_t* err;
    if ((rc = open_pipe(&p, &err))) return rc;
    const uint32_t nb = n / qb;
    const size_t xrow = static_cast<size_t>(n) * 4, qrow = n, drow = static_cast<size_t>(nb) * 4;
    const uint32_t TC = chunk_frames(T, xrow, qrow + drow);
    const size_t off_d = up256(static_cast<size_t>(TC) * qrow);
    if ((rc = p->reserve(static_cast<size_t>(TC) * xrow, off_d + static_cast<size_t>(TC) * drow, 0))) return rc;
    CopyPool& pool = CopyPool::get();
    const uint32_t nchunks = (T + TC - 1) / TC;
    auto frames = [&](uint32_t c) { return std::min(TC, T - c * TC); };
    // the host bytes this call rewrites: older results over them are stale
    ActCache& ac = g_acts[p->dev];
    act_forget(ac, reinterpret_cast<uintptr_t>(q), T * qrow, reinterpret_cast<uintptr_t>(d), T * drow);
    // the result's device copy, kept for the products that read it: a spare
    // copy's memory where one is large enough (no allocation, no fresh host
    // pages), else new device memory
    std::shared_ptr<ActCopy> keep;
    if (act_cache_cap() && T * (qrow + drow) <= act_cache_cap()) {
        keep = act_take_spare(ac, T * qrow, T * drow);
        if (!keep) {
            keep = std::make_shared<ActCopy>();
            keep->dev = p->dev;
            if (cudaMallocAsync(&keep->dq, T * qrow, p->s_comp) != cudaSuccess ||
                cudaMallocAsync(&keep->dd, T * drow, p->s_comp) != cudaSuccess) {
                cudaGetLastError();
                keep.reset();  // no room: the call works as without the cache
            } else {
                keep->cap_q = T * qrow;
                keep->cap_d = T * drow;
            }
        }
    }
    if (keep) {
        keep->q0 = reinterpret_cast<uintptr_t>(q);
        keep->d0 = reinterpret_cast<uintptr_t>(d);
        keep->n = n;
        keep->nb = nb;
        keep->T = T;
        // the host copy of what the call writes
        if (keep->hq.size() < T * qrow) keep->hq.resize(T * qrow);
        if (keep->hd.size() < static_cast<size_t>(T) * nb) keep->hd.resize(static_cast<size_t>(T) * nb);
    }
    // declared after keep, so drained before keep's memory can go
    DrainOnReturn drain{p};
    // where chunk c's bytes and scales are made on the device
    auto dq_of = [&](uint32_t c) -> int8_t* {
        return keep ? keep->dq + static_cast<size_t>(c) * TC * qrow : reinterpret_cast<int8_t*>(p->dev_out[c & 1]);
    };
    auto dd_of = [&](uint32_t c) -> float* {
        return keep ? keep->dd + static_cast<size_t>(c) * TC * nb : reinterpret_cast<float*>(p->dev_out[c & 1] + off_d);
    };
    // chunk c's bytes and scales, once in the caller's memory, into the host copy
    auto shadow = [&](uint32_t c) {
        if (!keep) return;
        const size_t t0 = static_cast<size_t>(c) * TC;
        pool.copy(keep->hq.data() + t0 * qrow, q + t0 * qrow, frames(c) * qrow);
        pool.copy(keep->hd.data() + t0 * nb, d + t0 * nb, frames(c) * drow);
    };
    // after the call's last copy: the entry, the oldest ones evicted past the cap
    auto remember = [&]() {
        if (!keep) return;
        std::unique_lock<std::shared_mutex> lock(ac.mu);
        const size_t sz = act_bytes(*keep);
        while (ac.bytes + sz > act_cache_cap() && !ac.order.empty()) {
            const auto old = ac.order.front();
            ac.order.pop_front();
            auto it = ac.by_q.find(old.first);
            if (it != ac.by_q.end() && it->second.get() == old.second) {
                ac.bytes -= act_bytes(*it->second);
                std::shared_ptr<ActCopy> gone = std::move(it->second);
                ac.by_q.erase(it);
                act_retire(ac, std::move(gone));
            }
        }
        ac.by_q[keep->q0] = keep;
        ac.order.emplace_back(keep->q0, keep.get());
        ac.bytes += sz;
    };
    if (pinned(x, ((T - 1) * xs + n) * 4) && pinned(q, T * qrow) && pinned(d, T * drow)) {
        // page-locked: every chunk by DMA straight from x and into q and d
        for (uint32_t c = 0; c < nchunks; c++) {
            const int s = c & 1;
            const uint32_t tc = frames(c);
            const size_t t0 = static_cast<size_t>(c) * TC;
            if (c >= 2) HOST_CUDA(cudaStreamWaitEvent(p->s_in, p->ev_comp[s], 0), "cudaStreamWaitEvent");
            HOST_CUDA(cudaMemcpy2DAsync(p->dev_in[s], xrow, x + t0 * xs, xs * 4, xrow, tc, cudaMemcpyHostToDevice,
                                        p->s_in),
                      "upload");
            HOST_CUDA(cudaEventRecord(p->ev_in[s], p->s_in), "cudaEventRecord");
            HOST_CUDA(cudaStreamWaitEvent(p->s_comp, p->ev_in[s], 0), "cudaStreamWaitEvent");
            if (c >= 2) HOST_CUDA(cudaStreamWaitEvent(p->s_comp, p->ev_out[s], 0), "cudaStreamWaitEvent");
            if ((rc = pkb_quantize_dev(p->s_comp, dq_of(c), dd_of(c), reinterpret_cast<const float*>(p->dev_in[s]), n,
                                       tc, n, qb, rmode)))
                return rc;
            HOST_CUDA(cudaEventRecord(p->ev_comp[s], p->s_comp), "cudaEventRecord");
            HOST_CUDA(cudaStreamWaitEvent(p->s_out, p->ev_comp[s], 0), "cudaStreamWaitEvent");
            HOST_CUDA(cudaMemcpyAsync(q + t0 * qrow, dq_of(c), tc * qrow, cudaMemcpyDeviceToHost, p->s_out), "download");
            HOST_CUDA(cudaMemcpyAsync(d + t0 * nb, dd_of(c), tc * drow, cudaMemcpyDeviceToHost, p->s_out), "download");
            HOST_CUDA(cudaEventRecord(p->ev_out[s], p->s_out), "cudaEventRecord");
        }
        count_host_bytes(T * xrow, T * (qrow + drow));
        if ((rc = p->finish(err))) return rc;
        // the host copy after the last chunk (a chunk at a time during the
        // loop would hold the next chunk's enqueue behind a copy that waits
        // for the copy pool, which other calls' comparisons keep busy: the
        // uploads then starve, measured on B200)
        for (uint32_t c = 0; c < nchunks; c++) shadow(c);
        remember();
        return PKB_OK;
    }
    auto take_out = [&](uint32_t c) -> int {  // chunk c's bytes and scales to the caller
        const int s = c & 1;
        HOST_CUDA(cudaEventSynchronize(p->ev_out[s]), "cudaEventSynchronize");
        pool.copy(q + static_cast<size_t>(c) * TC * qrow, p->pin_out[s], frames(c) * qrow);
        pool.copy(d + static_cast<size_t>(c) * TC * nb, p->pin_out[s] + off_d, frames(c) * drow);
        shadow(c);
        return PKB_OK;
    };
    for (uint32_t c = 0; c < nchunks; c++) {
        const int s = c & 1;
        const uint32_t tc = frames(c);
        if (c >= 2) HOST_CUDA(cudaEventSynchronize(p->ev_in[s]), "cudaEventSynchronize");
        pool.copy2d(p->pin_in[s], xrow, x + static_cast<size_t>(c) * TC * xs, xs * 4, xrow, tc);
        if (c >= 2) HOST_CUDA(cudaStreamWaitEvent(p->s_in, p->ev_comp[s], 0), "cudaStreamWaitEvent");
        HOST_CUDA(cudaMemcpyAsync(p->dev_in[s], p->pin_in[s], tc * xrow, cudaMemcpyHostToDevice, p->s_in), "upload");
        HOST_CUDA(cudaEventRecord(p->ev_in[s], p->s_in), "cudaEventRecord");
        HOST_CUDA(cudaStreamWaitEvent(p->s_comp, p->ev_in[s], 0), "cudaStreamWaitEvent");
        if (c >= 2) HOST_CUDA(cudaStreamWaitEvent(p->s_comp, p->ev_out[s], 0), "cudaStreamWaitEvent");
        if ((rc = pkb_quantize_dev(p->s_comp, dq_of(c), dd_of(c), reinterpret_cast<const float*>(p->dev_in[s]), n, tc,
                                   n, qb, rmode)))
            return rc;
        HOST_CUDA(cudaEventRecord(p->ev_comp[s], p->s_comp), "cudaEventRecord");
        HOST_CUDA(cudaStreamWaitEvent(p->s_out, p->ev_comp[s], 0), "cudaStreamWaitEvent");
        HOST_CUDA(cudaMemcpyAsync(p->pin_out[s], dq_of(c), tc * qrow, cudaMemcpyDeviceToHost, p->s_out), "download");
        HOST_CUDA(cudaMemcpyAsync(p->pin_out[s] + off_d, dd_of(c), tc * drow, cudaMemcpyDeviceToHost, p->s_out),
                  "download");
        HOST_CUDA(cudaEventRecord(p->ev_out[s], p->s_out), "cudaEventRecord");
        if (c >= 1 && (rc = take_out(c - 1))) return rc;
    }
    count_host_bytes(T * xrow, T * (qrow + drow));
    if ((rc = p->finish(err))) return rc;
    if ((rc = take_out(nchunks - 1))) return rc;
    remember();
    return PKB_OK;
}

int pkb_gemm_q8_host(float* out, size_t os, const int8_t* w, const float* ws, const float* bias, uint32_t rows,
                     const int8_t* q, const float* d, uint32_t n, uint32_t qb, uint32_t T, int add, int rmode) {
    int rc = check_shape(n, qb, rmode);
    if (rc) return rc;
    if (rows % 16) return set_error(PKB_EINVAL, "rows = %u: a multiple of 16", rows);
    // out[t os + r]: one column of results reads no stride (the reference's
    // decoder passes os 0 for its gemvs, core/decoder.c:56-63)
    if (T > 1 && os < rows) return set_error(PKB_EINVAL, "output stride %zu below rows = %u", os, rows);
    if (!T || !rows) return PKB_OK;
    if (T == 1) os = rows;
    if (!out || !w || !ws || !q || !d) return set_error(PKB_EINVAL, "gemm_q8: null pointer");
    Pipe* p;
    uint32_t* err;
    if ((rc = open_pipe(&p, &err))) return rc;
    const int8_t* wpack;
    std::shared_ptr<Matrix> held;  // the weights' device copy, kept for the call
    if ((rc = weights_for(*p, w, rows, n, &wpack, &held))) return rc;
    const uint32_t nb = n / qb;
    const size_t qrow = n, drow = static_cast<size_t>(nb) * 4, orow = static_cast<size_t>(rows) * 4;
    const uint32_t TC = chunk_frames(T, qrow + drow + (add ? orow : 0), orow);
    const size_t off_d = up256(static_cast<size_t>(TC) * qrow);
    const size_t in_bytes = off_d + static_cast<size_t>(TC) * drow;
    if ((rc = p->reserve(in_bytes, static_cast<size_t>(TC) * orow, 2 * up256(orow)))) return rc;
    CopyPool& pool = CopyPool::get();
    // the row scales and biases, once a call
    memcpy(p->pin_vec, ws, orow);
    if (bias) memcpy(p->pin_vec + up256(orow), bias, orow);
    HOST_CUDA(cudaMemcpyAsync(p->dev_vec, p->pin_vec, up256(orow) + orow, cudaMemcpyHostToDevice, p->s_comp),
              "upload");
    count_host_bytes(up256(orow) + orow, 0);
    const float* dws = reinterpret_cast<const float*>(p->dev_vec);
    const float* dbias = bias ? reinterpret_cast<const float*>(p->dev_vec + up256(orow)) : nullptr;
    const uint32_t nchunks = (T + TC - 1) / TC;
    auto frames = [&](uint32_t c) { return std::min(TC, T - c * TC); };
    // activations this library quantized and that are still the caller's
    // bytes: read from their device copy, not uploaded again
    uint32_t f0 = 0;
    ActHold act_hold;
    const std::shared_ptr<ActCopy> cached = act_find(p->dev, q, d, n, nb, T, &f0, &act_hold);
    // declared after the holds on the weights and the activations, so drained before they go
    DrainOnReturn drain{p};
    auto qsrc = [&](uint32_t c) -> const int8_t* {
        return cached ? cached->dq + (static_cast<size_t>(f0) + static_cast<size_t>(c) * TC) * qrow
                      : reinterpret_cast<const int8_t*>(p->dev_in[c & 1]);
    };
    auto dsrc = [&](uint32_t c) -> const float* {
        return cached ? cached->dd + (static_cast<size_t>(f0) + static_cast<size_t>(c) * TC) * nb
                      : reinterpret_cast<const float*>(p->dev_in[c & 1] + off_d);
    };
    if (pinned(q, T * qrow) && pinned(d, T * drow) && pinned(out, ((T - 1) * os + rows) * 4)) {
        // page-locked: every chunk by DMA straight from q, d (and the rows
        // added to) and into out at its stride
        for (uint32_t c = 0; c < nchunks; c++) {
            const int s = c & 1;
            const uint32_t tc = frames(c);
            const size_t t0 = static_cast<size_t>(c) * TC;
            if (c >= 2) {
                HOST_CUDA(cudaStreamWaitEvent(p->s_in, p->ev_comp[s], 0), "cudaStreamWaitEvent");
                HOST_CUDA(cudaStreamWaitEvent(p->s_in, p->ev_out[s], 0), "cudaStreamWaitEvent");
            }
            if (!cached) {
                HOST_CUDA(cudaMemcpyAsync(p->dev_in[s], q + t0 * qrow, tc * qrow, cudaMemcpyHostToDevice, p->s_in),
                          "upload");
                HOST_CUDA(cudaMemcpyAsync(p->dev_in[s] + off_d, d + t0 * nb, tc * drow, cudaMemcpyHostToDevice, p->s_in),
                          "upload");
            }
            if (add)
                HOST_CUDA(cudaMemcpy2DAsync(p->dev_out[s], orow, out + t0 * os, os * 4, orow, tc,
                                            cudaMemcpyHostToDevice, p->s_in),
                          "upload");
            HOST_CUDA(cudaEventRecord(p->ev_in[s], p->s_in), "cudaEventRecord");
            HOST_CUDA(cudaStreamWaitEvent(p->s_comp, p->ev_in[s], 0), "cudaStreamWaitEvent");
            if (c >= 2) HOST_CUDA(cudaStreamWaitEvent(p->s_comp, p->ev_out[s], 0), "cudaStreamWaitEvent");
            if ((rc = pkb_gemm_q8_dev(p->s_comp, reinterpret_cast<float*>(p->dev_out[s]), rows, wpack, dws, dbias,
                                      rows, qsrc(c), dsrc(c), n, qb, tc, add, rmode)))
                return rc;
            HOST_CUDA(cudaEventRecord(p->ev_comp[s], p->s_comp), "cudaEventRecord");
            HOST_CUDA(cudaStreamWaitEvent(p->s_out, p->ev_comp[s], 0), "cudaStreamWaitEvent");
            HOST_CUDA(cudaMemcpy2DAsync(out + t0 * os, os * 4, p->dev_out[s], orow, orow, tc, cudaMemcpyDeviceToHost,
                                        p->s_out),
                      "download");
            HOST_CUDA(cudaEventRecord(p->ev_out[s], p->s_out), "cudaEventRecord");
        }
        count_host_bytes(T * ((cached ? 0 : qrow + drow) + (add ? orow : 0)), T * orow);
        return p->finish(err);
    }
    auto take_out = [&](uint32_t c) -> int {  // chunk c's rows of out, at the caller's stride
        const int s = c & 1;
        HOST_CUDA(cudaEventSynchronize(p->ev_out[s]), "cudaEventSynchronize");
        pool.copy2d(out + static_cast<size_t>(c) * TC * os, os * 4, p->pin_out[s], orow, orow, frames(c));
        return PKB_OK;
    };
    for (uint32_t c = 0; c < nchunks; c++) {
        const int s = c & 1;
        const uint32_t tc = frames(c);
        const size_t t0 = static_cast<size_t>(c) * TC;
        if (c >= 2) HOST_CUDA(cudaEventSynchronize(p->ev_in[s]), "cudaEventSynchronize");
        if (!cached) {
            pool.copy(p->pin_in[s], q + t0 * qrow, tc * qrow);
            pool.copy(p->pin_in[s] + off_d, d + t0 * nb, tc * drow);
        }
        if (add) {
            // the residual the product adds to: its rows, packed, into the
            // output slot (its previous chunk there was taken out already)
            pool.copy2d(p->pin_out[s], orow, out + t0 * os, os * 4, orow, tc);
        }
        if (c >= 2) {
            HOST_CUDA(cudaStreamWaitEvent(p->s_in, p->ev_comp[s], 0), "cudaStreamWaitEvent");
            HOST_CUDA(cudaStreamWaitEvent(p->s_in, p->ev_out[s], 0), "cudaStreamWaitEvent");
        }
        if (!cached)
            HOST_CUDA(cudaMemcpyAsync(p->dev_in[s], p->pin_in[s], off_d + tc * drow, cudaMemcpyHostToDevice, p->s_in),
                      "upload");
        if (add)
            HOST_CUDA(cudaMemcpyAsync(p->dev_out[s], p->pin_out[s], tc * orow, cudaMemcpyHostToDevice, p->s_in),
                      "upload");
        HOST_CUDA(cudaEventRecord(p->ev_in[s], p->s_in), "cudaEventRecord");
        HOST_CUDA(cudaStreamWaitEvent(p->s_comp, p->ev_in[s], 0), "cudaStreamWaitEvent");
        if (c >= 2) HOST_CUDA(cudaStreamWaitEvent(p->s_comp, p->ev_out[s], 0), "cudaStreamWaitEvent");
        if ((rc = pkb_gemm_q8_dev(p->s_comp, reinterpret_cast<float*>(p->dev_out[s]), rows, wpack, dws, dbias, rows,
                                  qsrc(c), dsrc(c), n, qb, tc, add, rmode)))
            return rc;
        HOST_CUDA(cudaEventRecord(p->ev_comp[s], p->s_comp), "cudaEventRecord");
        HOST_CUDA(cudaStreamWaitEvent(p->s_out, p->ev_comp[s], 0), "cudaStreamWaitEvent");
        HOST_CUDA(cudaMemcpyAsync(p->pin_out[s], p->dev_out[s], tc * orow, cudaMemcpyDeviceToHost, p->s_out),
                  "download");
        HOST_CUDA(cudaEventRecord(p->ev_out[s], p->s_out), "cudaEventRecord");
        if (c >= 1 && (rc = take_out(c - 1))) return rc;
    }
    count_host_bytes(T * ((cached ? 0 : qrow + drow) + (add ? orow : 0)), T * orow);
    if ((rc = p->finish(err))) return rc;
    return take_out(nchunks - 1);
}

// pk_k_gemm_f32 on host memory: the run of panels, the columns, the biases
// (or, where out is the bias, out's rows) up, the product on the device, the
// results' rows back at their stride (only [t os, t os + rows): the engine's
// other threads may write the rest of those rows at the same time).
int pkb_gemm_f32_host(float* out, size_t os, const float* w, uint32_t ld, uint32_t rows, uint32_t n, const float* x,
                      size_t xs, uint32_t T, const float* bias, size_t bs, int relu, int rmode) {
    if (rmode < PKB_RN || rmode > PKB_RZ) return set_error(PKB_EINVAL, "rounding mode %d", rmode);
    if (rows % 16) return set_error(PKB_EINVAL, "gemm_f32: rows = %u, a multiple of 16", rows);
    if (n > ld) return set_error(PKB_EINVAL, "gemm_f32: n = %u beyond the panels' ld = %u", n, ld);
    if (!T || !rows) return PKB_OK;
    if (!out || !w || (n && !x)) return set_error(PKB_EINVAL, "gemm_f32: null pointer");
    // column t at x + t xs, out + t os, bias + t bs: one column reads no stride
    if (T == 1) os = xs = bs = 0;
    if (T > 1 && os < rows) return set_error(PKB_EINVAL, "gemm_f32: output stride %zu below rows = %u", os, rows);
    if (T > 1 && xs < n) return set_error(PKB_EINVAL, "gemm_f32: column stride %zu below n = %u", xs, n);
    if (T > 1 && bias && bs && bs < rows) return set_error(PKB_EINVAL, "gemm_f32: bias stride %zu below rows = %u", bs, rows);
    const bool alias = bias && bias == out;
    if (alias && bs != os) return set_error(PKB_EINVAL, "gemm_f32: out is the bias but bs %zu != os %zu", bs, os);
    Pipe* p;
    uint32_t* err;
    int rc;
    if ((rc = open_pipe(&p, &err))) return rc;
    DrainOnReturn drain{p};
    const size_t orow = static_cast<size_t>(rows) * 4;
    const size_t wbytes = n ? ((static_cast<size_t>(rows / 16) - 1) * ld + n) * 64 : 0;
    const size_t xbytes = n ? ((static_cast<size_t>(T) - 1) * xs + n) * 4 : 0;
    const size_t bbytes = bias && !alias ? ((bs ? (static_cast<size_t>(T) - 1) * bs : 0) + rows) * 4 : 0;
    const size_t off_x = up256(wbytes), off_b = off_x + up256(xbytes);
    if ((rc = p->reserve(off_b + bbytes, static_cast<size_t>(T) * orow, 0))) return rc;
    const cudaStream_t s = p->s_comp;
    if (wbytes) HOST_CUDA(cudaMemcpyAsync(p->dev_in[0], w, wbytes, cudaMemcpyHostToDevice, s), "upload");
    if (xbytes) HOST_CUDA(cudaMemcpyAsync(p->dev_in[0] + off_x, x, xbytes, cudaMemcpyHostToDevice, s), "upload");
    if (bbytes) HOST_CUDA(cudaMemcpyAsync(p->dev_in[0] + off_b, bias, bbytes, cudaMemcpyHostToDevice, s), "upload");
    float* dout = reinterpret_cast<float*>(p->dev_out[0]);
    if (alias)  // the biases are out's rows: up into the results' slot, packed
        HOST_CUDA(cudaMemcpy2DAsync(dout, orow, out, os * 4, orow, T, cudaMemcpyHostToDevice, s), "upload");
    const float* dbias = alias ? dout : bias ? reinterpret_cast<const float*>(p->dev_in[0] + off_b) : nullptr;
    const size_t dbs = alias ? rows : bs;
    if ((rc = pkb_gemm_f32_dev(s, dout, rows, reinterpret_cast<const float*>(p->dev_in[0]), ld, rows, n,
                               reinterpret_cast<const float*>(p->dev_in[0] + off_x), T > 1 ? xs : n, T, dbias, dbs, relu,
                               rmode)))
        return rc;
    HOST_CUDA(cudaMemcpy2DAsync(out, (T > 1 ? os : rows) * 4, dout, orow, orow, T, cudaMemcpyDeviceToHost, s),
              "download");
    count_host_bytes(wbytes + xbytes + bbytes + (alias ? T * orow : 0), T * orow);
    return p->finish(err);
}

// pk_k_softmax on one row of host memory, in place.
int pkb_softmax_host(float* x, uint32_t n, float scale, int rmode) {
    if (rmode < PKB_RN || rmode > PKB_RZ) return set_error(PKB_EINVAL, "rounding mode %d", rmode);
    if (!n) return PKB_OK;
    if (!x) return set_error(PKB_EINVAL, "softmax: null pointer");
    Pipe* p;
    uint32_t* err;
    int rc;
    if ((rc = open_pipe(&p, &err))) return rc;
    DrainOnReturn drain{p};
    const size_t bytes = static_cast<size_t>(n) * 4;
    if ((rc = p->reserve(0, bytes, 0))) return rc;
    const cudaStream_t s = p->s_comp;
    float* dx = reinterpret_cast<float*>(p->dev_out[0]);
    HOST_CUDA(cudaMemcpyAsync(dx, x, bytes, cudaMemcpyHostToDevice, s), "upload");
    if ((rc = pkb_softmax_dev(s, dx, n, 1, n, scale, rmode))) return rc;
    HOST_CUDA(cudaMemcpyAsync(x, dx, bytes, cudaMemcpyDeviceToHost, s), "download");
    count_host_bytes(bytes, bytes);
    return p->finish(err);
}

int pkb_forget(const void* ptr, size_t bytes) {
    // the copies overlapping the range leave the cache at once; their device
    // memory goes when the last call still using it returns
    const uintptr_t lo = reinterpret_cast<uintptr_t>(ptr), hi = lo + bytes;
    std::vector<std::shared_ptr<Matrix>> drop;
    for (DeviceCache& c : g_cache) {
        std::unique_lock<std::shared_mutex> lock(c.mu);
        for (auto it = c.mats.begin(); it != c.mats.end();) {
            if (it->second->lo < hi && lo < it->second->hi) {
                drop_pieces(c, it->second->lo, it->second->hi);
                drop.push_back(std::move(it->second));
                it = c.mats.erase(it);
            } else {
                ++it;
            }
        }
        drop_pieces(c, lo, hi);
    }
    for (ActCache& c : g_acts) act_forget(c, lo, bytes, lo, bytes);
    return PKB_OK;
}

}  // extern "C"
