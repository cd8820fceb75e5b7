// The device side of the C ABI of libpktito_b200 (include/pktito_b200.h):
// argument checks, device set-up, tensor maps and launches.
//
// The host-pointer entry points are in pkb_host.cu.

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/pktito_b200.h"
#include "pkb_internal.h"

namespace pkb {

__device__ uint32_t g_device_error;  // the device-side error word (pkb_device_errors)

namespace {

constexpr int MAX_DEV = 16;

thread_local char tl_err[512];
std::atomic<uint64_t> g_launches{0};
std::atomic<uint64_t> g_up{0}, g_down{0};

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(tl_err, sizeof tl_err, fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    const int code = e == cudaErrorMemoryAllocation ? PKB_ENOMEM : PKB_ECUDA;
    return fail(code, "%s: %s", what, cudaGetErrorString(e));
}

#define PKB_CUDA(call, what)                          \
    do {                                              \
        cudaError_t e_ = (call);                      \
        if (e_ != cudaSuccess) return cuda_fail(e_, what); \
    } while (0)

// --------------------------------------------------------------- devices --

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct Device {
    bool ready = false;
    int sms = 0;
    uint32_t* err = nullptr;  // device address of g_device_error
};

std::mutex g_dev_mu;
Device g_dev[MAX_DEV];
EncodeTiledFn g_encode = nullptr;
long long g_timeout = 0;

long long wait_limit() {
    if (!g_timeout) {
        const char* e = getenv("PKB_WAIT_CYCLES");
        long long v = e ? atoll(e) : 0;
        g_timeout = v > 0 ? v : (1ll << 31);  // about a second at B200's clocks
    }
    return g_timeout;
}

// The device that is current on this thread, checked to be an sm_100 one
// and set up once.
int current_device(Device** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(PKB_ENODEV, "no CUDA device: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= MAX_DEV) return fail(PKB_ENODEV, "device %d out of range", dev);
    Device& d = g_dev[dev];
    if (!d.ready) {
        std::lock_guard<std::mutex> lock(g_dev_mu);
        if (!d.ready) {
            cudaDeviceProp prop;
            PKB_CUDA(cudaGetDeviceProperties(&prop, dev), "cudaGetDeviceProperties");
            if (prop.major != 10)
                return fail(PKB_ENODEV, "device %d is sm_%d%d; libpktito_b200 runs on sm_100 (B200)", dev, prop.major,
                            prop.minor);
            if (!g_encode) {
                void* fn = nullptr;
                cudaDriverEntryPointQueryResult q;
                PKB_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q),
                         "cudaGetDriverEntryPoint");
                if (!fn || q != cudaDriverEntryPointSuccess)
                    return fail(PKB_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
                g_encode = reinterpret_cast<EncodeTiledFn>(fn);
            }
            void* sym = nullptr;
            PKB_CUDA(cudaGetSymbolAddress(&sym, g_device_error), "cudaGetSymbolAddress");
            d.err = static_cast<uint32_t*>(sym);
            PKB_CUDA(prepare_gemm_q8(), "kernel attributes");
            PKB_CUDA(prepare_attention(), "kernel attributes");
            prepare_quantize();
            d.sms = prop.multiProcessorCount;
            wait_limit();
            d.ready = true;
        }
    }
    *out = &d;
    return PKB_OK;
}

// A 2-D tensor map over rows x cols int8 (row stride cols bytes), with the
// product's boxes and the 128-byte swizzle; rows and cols beyond the
// tensor read as zeros.
int make_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows, uint32_t box_cols) {
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(PKB_ECUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return PKB_OK;
}

int check_act_shape(uint32_t n, uint32_t qb) {
    if (n == 0 || n % 32 || n > PKB_MAX_N)
        return fail(PKB_EINVAL, "n = %u: a multiple of 32 up to %u", n, PKB_MAX_N);
    if (qb == 0 || qb % 32 || n % qb)
        return fail(PKB_EINVAL, "qb = %u: a multiple of 32 dividing n = %u", qb, n);
    return PKB_OK;
}

int check_rmode(int rmode) {
    if (rmode < PKB_RN || rmode > PKB_RZ) return fail(PKB_EINVAL, "rounding mode %d", rmode);
    return PKB_OK;
}

bool aligned(const void* p, size_t a) { return reinterpret_cast<uintptr_t>(p) % a == 0; }

// ------------------------------------------------------- device entries --

int quantize_dev(cudaStream_t stream, int8_t* q, float* d, const float* x, size_t xs, uint32_t T, uint32_t n,
                 uint32_t qb, int rmode) {
    int rc = check_act_shape(n, qb);
    if (rc) return rc;
    if ((rc = check_rmode(rmode))) return rc;
    if (!T) return PKB_OK;
    if (!q || !d || !x) return fail(PKB_EINVAL, "quantize: null pointer");
    // the contract reads column t at x + t xs: one column reads no stride
    // (the reference's decoder passes its gemv's input so)
    if (T > 1 && xs < n) return fail(PKB_EINVAL, "quantize: column stride %zu below n = %u", xs, n);
    if (T == 1) xs = n;
    if (!aligned(q, 4) || !aligned(d, 4) || !aligned(x, 4)) return fail(PKB_EINVAL, "quantize: misaligned buffer");
    Device* dev;
    if ((rc = current_device(&dev))) return rc;
    PKB_CUDA(launch_quantize(q, d, x, xs, T, n, qb, rmode, dev->sms, stream), "quantize launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return PKB_OK;
}

// A tensor map of the block scales d [T][nb] (nb a multiple of 4, d 16-byte
// aligned): boxes of gemm_scale_box() blocks by gemm_tile_rows() frames.
int make_scale_map(CUtensorMap* md, const float* d, uint32_t nb, uint32_t T) {
    cuuint32_t estr[2] = {1, 1};
    cuuint64_t ddims[2] = {nb, T};
    cuuint64_t dstrides[1] = {static_cast<cuuint64_t>(nb) * 4};
    cuuint32_t dbox[2] = {static_cast<cuuint32_t>(gemm_scale_box()), static_cast<cuuint32_t>(gemm_tile_rows())};
    CUresult r = g_encode(md, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(d), ddims, dstrides, dbox, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(PKB_ECUDA, "cuTensorMapEncodeTiled (scales) failed (%d)", static_cast<int>(r));
    return PKB_OK;
}

int gemm_dev(cudaStream_t stream, float* out, size_t os, const int8_t* wpack, const float* ws, const float* bias,
             uint32_t rows, const int8_t* q, const float* d, uint32_t n, uint32_t qb, uint32_t T, int add, int rmode) {
    int rc = check_act_shape(n, qb);
    if (rc) return rc;
    if ((rc = check_rmode(rmode))) return rc;
    if (rows % 16) return fail(PKB_EINVAL, "rows = %u: a multiple of 16", rows);
    // out[t os + r]: one column of results reads no stride (the reference's
    // decoder passes os 0 for its gemvs, core/decoder.c:56-63)
    if (T > 1 && os < rows) return fail(PKB_EINVAL, "output stride %zu below rows = %u", os, rows);
    if (!T || !rows) return PKB_OK;
    if (T == 1) os = rows;
    if (!out || !wpack || !ws || !q || !d) return fail(PKB_EINVAL, "gemm_q8: null pointer");
    if (!aligned(q, 16) || !aligned(wpack, 16))
        return fail(PKB_EINVAL, "gemm_q8: activations and weights must be 16-byte aligned");
    if (!aligned(d, 4) || !aligned(out, 4) || !aligned(ws, 4) || (bias && !aligned(bias, 4)))
        return fail(PKB_EINVAL, "gemm_q8: misaligned float buffer");
    Device* dev;
    if ((rc = current_device(&dev))) return rc;
    CUtensorMap ma, mb;
    if ((rc = make_map(&ma, q, T, n, gemm_tile_rows(), gemm_box_k()))) return rc;
    if ((rc = make_map(&mb, wpack, rows, n, gemm_tile_cols(), gemm_box_k()))) return rc;
    GemmArgs g;
    g.out = out;
    g.ws = ws;
    g.bias = bias;
    g.d = d;
    g.err = dev->err;
    g.os = os;
    g.rows = rows;
    g.n = n;
    g.qb = qb;
    g.T = T;
    g.add = add ? 1u : 0u;
    g.tiles_m = (T + gemm_tile_rows() - 1) / gemm_tile_rows();
    g.tiles_n = (rows + gemm_tile_cols() - 1) / gemm_tile_cols();
    g.timeout = wait_limit();
    g.pmode = 0;
    g.dk = 0;
    g.tpad = T;
    g.ps = 0;
    // row scales, biases and results through TMA where their rows are whole
    // 16-byte units; the block scales too, except for blocks of whole boxes
    CUtensorMap md, mo;
    const CUtensorMap* mdp = nullptr;
    const CUtensorMap* mop = nullptr;
    const uint32_t nb = n / qb;
    const bool wide = gemm_wide_blocks(n, qb);
    if ((wide || (nb % 4 == 0 && aligned(d, 16))) && os % 4 == 0 && aligned(out, 16) && aligned(ws, 16) &&
        (!bias || aligned(bias, 16))) {
        if (!wide) {
            if ((rc = make_scale_map(&md, d, nb, T))) return rc;
            mdp = &md;
        }
        cuuint32_t estr[2] = {1, 1};
        cuuint64_t odims[2] = {rows, T};
        cuuint64_t ostrides[1] = {static_cast<cuuint64_t>(os) * 4};
        cuuint32_t obox[2] = {static_cast<cuuint32_t>(gemm_out_box()), static_cast<cuuint32_t>(gemm_out_box())};
        CUresult r = g_encode(&mo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, out, odims, ostrides, obox, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(PKB_ECUDA, "cuTensorMapEncodeTiled (results) failed (%d)", static_cast<int>(r));
        mop = &mo;
    }
    PKB_CUDA(launch_gemm_q8(ma, mb, mdp, mop, g, dev->sms, rmode, stream), "gemm_q8 launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return PKB_OK;
}

// ------------------------------------------------------ fused producers --

int check_fused_qb(uint32_t qb) {
    if (qb != 32 && qb != 64) return fail(PKB_EINVAL, "qb = %u: 32 or 64, the encoder's blocks", qb);
    return PKB_OK;
}

int layernorm_quantize_dev(cudaStream_t stream, int8_t* q, float* d, const float* x, size_t xs, uint32_t T,
                           uint32_t n, uint32_t qb, const float* w, const float* b, float eps, int rmode) {
    int rc;
    if ((rc = check_rmode(rmode)) || (rc = check_fused_qb(qb))) return rc;
    if (n == 0 || n % qb || n > PKB_LN_MAX_N)
        return fail(PKB_EINVAL, "layernorm_quantize: n = %u, a multiple of qb up to %u", n, PKB_LN_MAX_N);
    if (!T) return PKB_OK;
    if (!q || !d || !x || !w || !b) return fail(PKB_EINVAL, "layernorm_quantize: null pointer");
    if (xs < n) return fail(PKB_EINVAL, "layernorm_quantize: row stride %zu below n = %u", xs, n);
    if (!aligned(q, 4) || !aligned(d, 4) || !aligned(x, 4) || !aligned(w, 4) || !aligned(b, 4))
        return fail(PKB_EINVAL, "layernorm_quantize: misaligned buffer");
    Device* dev;
    if ((rc = current_device(&dev))) return rc;
    PKB_CUDA(launch_layernorm_quantize(q, d, x, xs, T, n, qb, w, b, eps, rmode, dev->sms, stream),
             "layernorm_quantize launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return PKB_OK;
}

int layernorm_dev(cudaStream_t stream, float* out, size_t os, const float* x, size_t xs, uint32_t T, uint32_t n,
                  const float* w, const float* b, float eps, int rmode) {
    int rc;
    if ((rc = check_rmode(rmode))) return rc;
    if (n == 0 || n % 32 || n > PKB_LN_MAX_N)
        return fail(PKB_EINVAL, "layernorm: n = %u, a multiple of 32 up to %u", n, PKB_LN_MAX_N);
    if (!T) return PKB_OK;
    if (!out || !x || !w || !b) return fail(PKB_EINVAL, "layernorm: null pointer");
    if (T > 1 && (xs < n || os < n)) return fail(PKB_EINVAL, "layernorm: a row stride below n = %u", n);
    if (T == 1) xs = os = n;
    if (!aligned(out, 4) || !aligned(x, 4) || !aligned(w, 4) || !aligned(b, 4))
        return fail(PKB_EINVAL, "layernorm: misaligned buffer");
    if (out != x) {
        const uintptr_t x0 = reinterpret_cast<uintptr_t>(x), x1 = x0 + ((T - 1) * xs + n) * sizeof(float);
        const uintptr_t o0 = reinterpret_cast<uintptr_t>(out), o1 = o0 + ((T - 1) * os + n) * sizeof(float);
        if (o0 < x1 && x0 < o1) return fail(PKB_EINVAL, "layernorm: out overlaps x (only out == x is allowed)");
    } else if (os != xs) {
        return fail(PKB_EINVAL, "layernorm: in place with os %zu != xs %zu", os, xs);
    }
    Device* dev;
    if ((rc = current_device(&dev))) return rc;
    PKB_CUDA(launch_layernorm(out, os, x, xs, T, n, w, b, eps, rmode, dev->sms, stream), "layernorm launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return PKB_OK;
}

int silu_quantize_dev(cudaStream_t stream, int8_t* q, float* d, const float* u, size_t us, uint32_t T, uint32_t n,
                      uint32_t qb, int rmode) {
    int rc;
    if ((rc = check_rmode(rmode)) || (rc = check_fused_qb(qb)) || (rc = check_act_shape(n, qb))) return rc;
    if (!T) return PKB_OK;
    if (!q || !d || !u) return fail(PKB_EINVAL, "silu_quantize: null pointer");
    if (us < n) return fail(PKB_EINVAL, "silu_quantize: row stride %zu below n = %u", us, n);
    if (!aligned(q, 4) || !aligned(d, 4) || !aligned(u, 4)) return fail(PKB_EINVAL, "silu_quantize: misaligned buffer");
    Device* dev;
    if ((rc = current_device(&dev))) return rc;
    PKB_CUDA(launch_silu_quantize(q, d, u, us, T, n, qb, rmode, dev->sms, stream), "silu_quantize launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return PKB_OK;
}

int dwconv_quantize_dev(cudaStream_t stream, int8_t* q, float* d, float* out, size_t os, const float* x, size_t xs,
                        uint32_t T, uint32_t C, const float* w, const float* b, uint32_t K, int glu, uint32_t qb,
                        int rmode) {
    int rc;
    if ((rc = check_rmode(rmode)) || (rc = check_fused_qb(qb))) return rc;
    if (C == 0 || C % qb || C > PKB_MAX_N)
        return fail(PKB_EINVAL, "dwconv_quantize: C = %u, a multiple of qb up to %u", C, PKB_MAX_N);
    if (K % 2 == 0 || K > 63) return fail(PKB_EINVAL, "dwconv_quantize: K = %u, odd and at most 63", K);
    if (!T) return PKB_OK;
    if (!q || !d || !x || !w || !b) return fail(PKB_EINVAL, "dwconv_quantize: null pointer");
    const size_t width = glu ? 2 * static_cast<size_t>(C) : C;
    if (xs < width) return fail(PKB_EINVAL, "dwconv_quantize: frame stride %zu below %zu", xs, width);
    if (!aligned(q, 4) || !aligned(d, 4) || !aligned(x, 4) || !aligned(w, 4) || !aligned(b, 4) ||
        (out && !aligned(out, 4)))
        return fail(PKB_EINVAL, "dwconv_quantize: misaligned buffer");
    if (out) {
        if (os < C) return fail(PKB_EINVAL, "dwconv_quantize: out stride %zu below C = %u", os, C);
        const uintptr_t x0 = reinterpret_cast<uintptr_t>(x), x1 = x0 + ((T - 1) * xs + width) * sizeof(float);
        const uintptr_t o0 = reinterpret_cast<uintptr_t>(out), o1 = o0 + ((T - 1) * os + C) * sizeof(float);
        if (o0 < x1 && x0 < o1) return fail(PKB_EINVAL, "dwconv_quantize: out overlaps x");
    }
    Device* dev;
    if ((rc = current_device(&dev))) return rc;
    PKB_CUDA(launch_dwconv_quantize(q, d, out, os, x, xs, T, C, w, b, K, glu != 0, qb, rmode, stream),
             "dwconv_quantize launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return PKB_OK;
}

// The product straight into the attention's panels (kind PKB_PANELS_V or
// PKB_PANELS_KP): no bias, nothing added, as the reference's V, K and P
// products. Where n / qb is a multiple of 4 and the buffers (and V's panel
// stride) whole 16-byte units, the results leave through TMA stores of a
// panel-shaped map: V as (row in panel 16, frame T, panel rows/16), boxes of
// 16 x 32 x 2 with a 64-byte swizzle; K/P as (frame in panel 16, dimension
// dk, panel tpad/16, head rows/dk), boxes of 16 x 16 x 2 x 1, so a box never
// crosses a head and the map clips the frames past tpad. Otherwise the
// plain-store path, its index per kind.
int gemm_panels_dev(cudaStream_t stream, float* panels, int kind, size_t ps, uint32_t dk, uint32_t tpad,
                    const int8_t* wpack, const float* ws, uint32_t rows, const int8_t* q, const float* d, uint32_t n,
                    uint32_t qb, uint32_t T, int rmode) {
    int rc = check_act_shape(n, qb);
    if (rc) return rc;
    if ((rc = check_rmode(rmode))) return rc;
    if (kind != PKB_PANELS_V && kind != PKB_PANELS_KP) return fail(PKB_EINVAL, "panels: kind %d", kind);
    if (rows % 16) return fail(PKB_EINVAL, "rows = %u: a multiple of 16", rows);
    if (kind == PKB_PANELS_V && ps < 16 * static_cast<size_t>(T))
        return fail(PKB_EINVAL, "V panels: panel stride %zu below 16 T = %zu", ps, 16 * static_cast<size_t>(T));
    if (kind == PKB_PANELS_KP) {
        if (dk == 0 || dk % 16 || rows % dk)
            return fail(PKB_EINVAL, "K/P panels: dk = %u, a multiple of 16 dividing rows = %u", dk, rows);
        if (tpad < T || tpad % 16)
            return fail(PKB_EINVAL, "K/P panels: tpad = %u, a multiple of 16 from T = %u", tpad, T);
    }
    if (!T || !rows) return PKB_OK;
    if (!panels || !wpack || !ws || !q || !d) return fail(PKB_EINVAL, "panels: null pointer");
    if (!aligned(q, 16) || !aligned(wpack, 16))
        return fail(PKB_EINVAL, "panels: activations and weights must be 16-byte aligned");
    if (!aligned(d, 4) || !aligned(panels, 4) || !aligned(ws, 4))
        return fail(PKB_EINVAL, "panels: misaligned float buffer");
    Device* dev;
    if ((rc = current_device(&dev))) return rc;
    CUtensorMap ma, mb;
    if ((rc = make_map(&ma, q, T, n, gemm_tile_rows(), gemm_box_k()))) return rc;
    if ((rc = make_map(&mb, wpack, rows, n, gemm_tile_cols(), gemm_box_k()))) return rc;
    GemmArgs g;
    g.out = panels;
    g.ws = ws;
    g.bias = nullptr;
    g.d = d;
    g.err = dev->err;
    g.os = rows;
    g.rows = rows;
    g.n = n;
    g.qb = qb;
    g.T = T;
    g.add = 0;
    g.pmode = kind == PKB_PANELS_V ? 1u : 2u;
    g.dk = dk;
    g.tpad = kind == PKB_PANELS_KP ? tpad : T;
    g.ps = ps;
    // K/P's tiles reach its padding, whose frames it writes as zeros
    g.tiles_m = (g.tpad + gemm_tile_rows() - 1) / gemm_tile_rows();
    g.tiles_n = (rows + gemm_tile_cols() - 1) / gemm_tile_cols();
    g.timeout = wait_limit();
    CUtensorMap md, mo;
    const CUtensorMap* mdp = nullptr;
    const CUtensorMap* mop = nullptr;
    const uint32_t nb = n / qb;
    const bool wide = gemm_wide_blocks(n, qb);
    if ((wide || (nb % 4 == 0 && aligned(d, 16))) && aligned(panels, 16) && aligned(ws, 16) &&
        (kind == PKB_PANELS_KP || ps % 4 == 0)) {
        if (!wide) {
            if ((rc = make_scale_map(&md, d, nb, T))) return rc;
            mdp = &md;
        }
        cuuint32_t estr[4] = {1, 1, 1, 1};
        CUresult r;
        if (kind == PKB_PANELS_V) {
            cuuint64_t odims[3] = {16, T, rows / 16};
            cuuint64_t ostrides[2] = {64, static_cast<cuuint64_t>(ps) * 4};
            cuuint32_t obox[3] = {16, 32, 2};
            r = g_encode(&mo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, panels, odims, ostrides, obox, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        } else {
            cuuint64_t odims[4] = {16, dk, tpad / 16, rows / dk};
            cuuint64_t ostrides[3] = {64, 64 * static_cast<cuuint64_t>(dk),
                                      4 * static_cast<cuuint64_t>(tpad) * dk};
            cuuint32_t obox[4] = {16, 16, 2, 1};
            r = g_encode(&mo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, panels, odims, ostrides, obox, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        }
        if (r != CUDA_SUCCESS) return fail(PKB_ECUDA, "cuTensorMapEncodeTiled (panels) failed (%d)", static_cast<int>(r));
        mop = &mo;
    }
    PKB_CUDA(launch_gemm_q8(ma, mb, mdp, mop, g, dev->sms, rmode, stream), "panels launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return PKB_OK;
}

int repack_dev(cudaStream_t stream, int8_t* wpack, const int8_t* w_pk, uint32_t rows, uint32_t n) {
    if (rows % 16 || n % 32 || n == 0) return fail(PKB_EINVAL, "repack: rows %u (16s) by n %u (32s)", rows, n);
    if (!rows) return PKB_OK;
    if (!wpack || !w_pk || !aligned(wpack, 4) || !aligned(w_pk, 4))
        return fail(PKB_EINVAL, "repack: null or misaligned buffer");
    Device* dev;
    int rc = current_device(&dev);
    if (rc) return rc;
    PKB_CUDA(launch_repack_q8(wpack, w_pk, rows, n, dev->sms, stream), "repack launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return PKB_OK;
}

// ------------------------------------------------ the attention's floats --

int gemm_f32_dev(cudaStream_t stream, float* out, size_t os, const float* w, uint32_t ld, uint32_t rows, uint32_t n,
                 const float* x, size_t xs, uint32_t T, const float* bias, size_t bs, int relu, int rmode) {
    int rc;
    if ((rc = check_rmode(rmode))) return rc;
    if (rows % 16) return fail(PKB_EINVAL, "gemm_f32: rows = %u, a multiple of 16", rows);
    if (n > ld) return fail(PKB_EINVAL, "gemm_f32: n = %u beyond the panels' ld = %u", n, ld);
    if (!T || !rows) return PKB_OK;
    if (!out || (n && (!w || !x))) return fail(PKB_EINVAL, "gemm_f32: null pointer");
    if (T > 1 && os < rows) return fail(PKB_EINVAL, "gemm_f32: output stride %zu below rows = %u", os, rows);
    if (T > 1 && xs < n) return fail(PKB_EINVAL, "gemm_f32: column stride %zu below n = %u", xs, n);
    if (bias && bs && bs < rows) return fail(PKB_EINVAL, "gemm_f32: bias stride %zu below rows = %u", bs, rows);
    if (T == 1) os = xs = rows;  // one column reads no stride
    if (!aligned(out, 4) || !aligned(w, 4) || !aligned(x, 4) || (bias && !aligned(bias, 4)))
        return fail(PKB_EINVAL, "gemm_f32: misaligned buffer");
    if (T > 65535u * 32u) return fail(PKB_EINVAL, "gemm_f32: T = %u columns, at most %u", T, 65535u * 32u);
    Device* dev;
    if ((rc = current_device(&dev))) return rc;
    PKB_CUDA(launch_gemm_f32(out, os, w, ld, rows, n, x, T == 1 ? n : xs, T, bias, bs, relu, rmode, stream),
             "gemm_f32 launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return PKB_OK;
}

int softmax_dev(cudaStream_t stream, float* x, size_t xs, uint32_t T, uint32_t n, float scale, int rmode) {
    int rc;
    if ((rc = check_rmode(rmode))) return rc;
    if (!T || !n) return PKB_OK;
    if (!x) return fail(PKB_EINVAL, "softmax: null pointer");
    if (T > 1 && xs < n) return fail(PKB_EINVAL, "softmax: row stride %zu below n = %u", xs, n);
    if (!aligned(x, 4)) return fail(PKB_EINVAL, "softmax: misaligned buffer");
    Device* dev;
    if ((rc = current_device(&dev))) return rc;
    PKB_CUDA(launch_softmax(x, T == 1 ? n : xs, T, n, scale, rmode, dev->sms, stream), "softmax launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return PKB_OK;
}

// The attention over segments (panels: one segment in the reference's
// panel layouts; else rows), in launches of up to ATT_MAX_SEG segments, one
// CTA a head and block of queries.
int attention_dev(cudaStream_t stream, bool panels, float* o, size_t os, const float* q, size_t qs, const float* k,
                  size_t ks, const float* v, size_t vs, const float* p, size_t ps, const float* bias_u,
                  const float* bias_v, uint32_t D, uint32_t H, const pkb_att_segment* segs, uint32_t nseg, int rmode) {
    int rc;
    if ((rc = check_rmode(rmode))) return rc;
    if (!H || !D || D % H || (D / H) % 16 || D / H > 256)
        return fail(PKB_EINVAL, "attention: D = %u, H = %u: heads of a multiple of 16 up to 256", D, H);
    if (!nseg) return PKB_OK;
    if (!segs || !o || !q || !k || !v || !p || !bias_u || !bias_v) return fail(PKB_EINVAL, "attention: null pointer");
    if (!aligned(o, 4) || !aligned(q, 4) || !aligned(bias_u, 4) || !aligned(bias_v, 4) || !aligned(k, 16) ||
        !aligned(v, 16) || !aligned(p, 16))
        return fail(PKB_EINVAL, "attention: misaligned buffer (K, P and V 16-byte aligned)");
    if (!panels && (ks % 4 || vs % 4 || ps % 4))
        return fail(PKB_EINVAL, "attention: K, V and P row strides must be multiples of 4 floats");
    const uint32_t dk = D / H;
    Device* dev;
    if ((rc = current_device(&dev))) return rc;
    const size_t smem_max = attention_smem_max();
    for (uint32_t s0 = 0; s0 < nseg; s0 += ATT_MAX_SEG) {
        AttArgs a = {};
        a.o = o;
        a.q = q;
        a.k = k;
        a.p = p;
        a.v = v;
        a.bu = bias_u;
        a.bv = bias_v;
        a.os = os;
        a.qs = qs;
        a.ks = ks;
        a.ps = ps;
        a.vs = vs;
        a.dk = dk;
        uint32_t tmax = 0;
        uint64_t items = 0;
        for (uint32_t s = s0; s < nseg && s < s0 + ATT_MAX_SEG; s++) {
            const pkb_att_segment& g = segs[s];
            if (!g.T) continue;
            if (g.T > 1 && (os < D || qs < D || (!panels && (ks < D || vs < D))))
                return fail(PKB_EINVAL, "attention: a row stride below D = %u", D);
            if (!panels && 2 * static_cast<uint64_t>(g.T) - 1 > 1 && ps < D)
                return fail(PKB_EINVAL, "attention: P's row stride %zu below D = %u", ps, D);
            a.seg[a.nseg] = AttSeg{g.T, g.f, g.p, static_cast<uint32_t>(items)};
            a.nseg++;
            items += static_cast<uint64_t>(H) * ((g.T + attention_block() - 1) / attention_block());
            tmax = g.T > tmax ? g.T : tmax;
        }
        if (!a.nseg) continue;
        if (items >= (1ull << 31)) return fail(PKB_EINVAL, "attention: %llu blocks in one launch", (unsigned long long)items);
        a.items = static_cast<uint32_t>(items);
        a.sp = (tmax + 15) & ~15u;  // the scores' rows hold T
        const size_t smem = attention_smem(dk, a.sp);
        if (smem > smem_max)
            return fail(PKB_EINVAL, "attention: T = %u needs %zu bytes of shared memory a block, above %zu", tmax, smem,
                        smem_max);
        PKB_CUDA(launch_attention(a, panels, rmode, stream), "attention launch");
        g_launches.fetch_add(1, std::memory_order_relaxed);
    }
    return PKB_OK;
}

// ------------------------------------------------------------- TDT search --

#ifndef PKB_TDT_GRAPH
#define PKB_TDT_GRAPH 1
#endif

// The work area's pieces, 256-byte aligned, in the order TdtArgs lists them.
struct TdtLayout {
    size_t seg, T, f0, qembed, dembed, qx, dx, h, c, qh, dh, gates, gp, gpn, qz, dz, logits, keys, bar, total;
};

TdtLayout tdt_layout(const pkb_tdt_model& m, uint32_t S) {
    TdtLayout o = {};
    size_t at = 0;
    auto take = [&](size_t bytes) {
        const size_t here = at;
        at += (bytes + 255) & ~size_t(255);
        return here;
    };
    const size_t P = m.P, J = m.J, L = m.L, V1 = m.V + 1;
    o.seg = take(S * tdt_seg_bytes());
    o.T = take(S * 4);
    o.f0 = take(S * 4);
    o.qembed = take(V1 * P);
    o.dembed = take(V1 * 4);
    o.qx = take(S * P);
    o.dx = take(S * 4);
    o.h = take(L * S * P * 4);
    o.c = take(L * S * P * 4);
    o.qh = take(L * S * P);
    o.dh = take(L * S * 4);
    o.gates = take(S * 4 * P * 4);
    o.gp = take(S * J * 4);
    o.gpn = take(S * J * 4);
    o.qz = take(S * J);
    o.dz = take(S * 4);
    o.logits = take(S * size_t(m.n_out_pad) * 4);
    o.keys = take(2 * S * 2 * 8);  // the persistent search's argmax keys, two rounds' worth
    o.bar = take(8);  // its barrier count and abort flag
    o.total = at;
    return o;
}

int check_tdt(const pkb_tdt_model* m) {
    if (!m) return fail(PKB_EINVAL, "tdt: null model");
    if (!m->P || m->P % 32 || m->P > PKB_MAX_N || !m->J || m->J % 32 || m->J > PKB_MAX_N)
        return fail(PKB_EINVAL, "tdt: P = %u and J = %u, multiples of 32 up to %u", m->P, m->J, PKB_MAX_N);
    if (!m->L || m->L > PKB_TDT_MAX_LAYERS) return fail(PKB_EINVAL, "tdt: %u LSTM layers", m->L);
    if (!m->n_dur || m->n_dur > PKB_TDT_MAX_DUR) return fail(PKB_EINVAL, "tdt: %u durations", m->n_dur);
    if (m->n_out_pad % 16 || m->n_out_pad < m->V + 1 + m->n_dur)
        return fail(PKB_EINVAL, "tdt: n_out_pad = %u for %u tokens and %u durations", m->n_out_pad, m->V + 1, m->n_dur);
    if (!m->max_symbols) return fail(PKB_EINVAL, "tdt: max_symbols 0");
    if (!m->embed || !m->jpred || !m->jpreds || !m->jout || !m->jouts)
        return fail(PKB_EINVAL, "tdt: null weights");
    for (uint32_t l = 0; l < m->L; l++)
        if (!m->wx[l] || !m->wh[l] || !m->wxs[l] || !m->whs[l] || !m->lb[l])
            return fail(PKB_EINVAL, "tdt: null weights of layer %u", l);
    return PKB_OK;
}

// A stream of the call's own (rounds are captured into a graph, which the
// legacy default stream a caller may pass cannot be), destroyed on return.
struct OwnStream {
    cudaStream_t s = nullptr;
    ~OwnStream() {
        if (s) cudaStreamDestroy(s);
    }
};

// The rounds as launches: ROUNDS rounds as one CUDA graph, replayed until
// every search has ended (a round past a segment's end does nothing to it),
// the segments' states read back after each replay.
template <typename Round>
int tdt_rounds(Round& round, cudaStream_t st, std::vector<uint8_t>& states, const uint8_t* seg, uint32_t S, uint32_t L,
               uint64_t max_rounds) {
    constexpr uint32_t ROUNDS = 8;
#if !PKB_TDT_GRAPH
    int rc;
    for (uint64_t r = 0; r < max_rounds; r += ROUNDS) {
        for (uint32_t i = 0; i < ROUNDS; i++)
            if ((rc = round())) return rc;
        PKB_CUDA(cudaMemcpyAsync(states.data(), seg, states.size(), cudaMemcpyDeviceToHost, st), "download");
        PKB_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize");
        bool running = false;
        for (uint32_t s = 0; s < S; s++)
            if (reinterpret_cast<const uint32_t*>(states.data() + s * tdt_seg_bytes())[TDT_SEG_ACTIVE]) running = true;
        if (!running) break;
    }
#else
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    PKB_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
    int crc = PKB_OK;
    const uint64_t counted = g_launches.load();
    for (uint32_t r = 0; r < ROUNDS && !crc; r++) crc = round();
    // a captured launch runs when the graph does: counted at each replay
    g_launches.fetch_sub(g_launches.load() - counted, std::memory_order_relaxed);
    const cudaError_t ce = cudaStreamEndCapture(st, &graph);
    if (crc) {
        if (graph) cudaGraphDestroy(graph);
        return crc;
    }
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaStreamEndCapture");
    const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) return cuda_fail(ie, "cudaGraphInstantiate");
    bool running = true;
    cudaError_t le = cudaSuccess;
    for (uint64_t r = 0; running && r < max_rounds && le == cudaSuccess; r += ROUNDS) {
        le = cudaGraphLaunch(exec, st);
        if (le == cudaSuccess) le = cudaMemcpyAsync(states.data(), seg, states.size(), cudaMemcpyDeviceToHost, st);
        if (le == cudaSuccess) le = cudaStreamSynchronize(st);
        g_launches.fetch_add(ROUNDS * (3 * L + 4), std::memory_order_relaxed);
        running = false;
        for (uint32_t s = 0; s < S; s++)
            if (reinterpret_cast<const uint32_t*>(states.data() + s * tdt_seg_bytes())[TDT_SEG_ACTIVE]) running = true;
    }
    cudaGraphExecDestroy(exec);
    if (le != cudaSuccess) return cuda_fail(le, "tdt rounds");
#endif
    return PKB_OK;
}

// rounds of the calling thread's last search: its longest segment's joint steps
thread_local uint64_t tl_tdt_rounds = 0;

int tdt_search_dev(cudaStream_t caller, const pkb_tdt_model* m, const float* f, const uint32_t* f0,
                   const uint32_t* T, uint32_t S, int32_t* toks, uint32_t* ntok, uint32_t cap, void* work,
                   size_t work_bytes, int rmode) {
    int rc;
    if ((rc = check_rmode(rmode)) || (rc = check_tdt(m))) return rc;
    if (!S) return PKB_OK;
    if (!f || !f0 || !T || !toks || !ntok || !work) return fail(PKB_EINVAL, "tdt: null pointer");
    const TdtLayout o = tdt_layout(*m, S);
    if (work_bytes < o.total || !aligned(work, 256))
        return fail(PKB_EINVAL, "tdt: work area of %zu bytes (%zu needed, 256-byte aligned)", work_bytes, o.total);
    Device* dev;
    if ((rc = current_device(&dev))) return rc;
    // the caller's work on f and the outputs ends first; the call's own runs
    // on its own stream and has ended when it returns
    PKB_CUDA(cudaStreamSynchronize(caller), "cudaStreamSynchronize");
    OwnStream own;
    PKB_CUDA(cudaStreamCreateWithFlags(&own.s, cudaStreamNonBlocking), "cudaStreamCreate");
    const cudaStream_t st = own.s;
    uint8_t* w = static_cast<uint8_t*>(work);
    TdtArgs a = {};
    a.S = S;
    a.P = m->P;
    a.J = m->J;
    a.V = m->V;
    a.n_dur = m->n_dur;
    a.max_symbols = m->max_symbols;
    a.nout = m->n_out_pad;
    a.cap = cap;
    for (uint32_t i = 0; i < m->n_dur; i++) a.dur[i] = m->dur[i];
    a.T = reinterpret_cast<const uint32_t*>(w + o.T);
    a.f0 = reinterpret_cast<const uint32_t*>(w + o.f0);
    a.f = f;
    a.seg = w + o.seg;
    a.ntok = ntok;
    a.toks = toks;
    a.qembed = reinterpret_cast<const int8_t*>(w + o.qembed);
    a.dembed = reinterpret_cast<const float*>(w + o.dembed);
    a.qx = reinterpret_cast<int8_t*>(w + o.qx);
    a.dx = reinterpret_cast<float*>(w + o.dx);
    a.h = reinterpret_cast<float*>(w + o.h);
    a.c = reinterpret_cast<float*>(w + o.c);
    a.qh = reinterpret_cast<int8_t*>(w + o.qh);
    a.dh = reinterpret_cast<float*>(w + o.dh);
    a.gates = reinterpret_cast<float*>(w + o.gates);
    a.gp = reinterpret_cast<float*>(w + o.gp);
    a.gpn = reinterpret_cast<float*>(w + o.gpn);
    a.qz = reinterpret_cast<int8_t*>(w + o.qz);
    a.dz = reinterpret_cast<float*>(w + o.dz);
    a.logits = reinterpret_cast<float*>(w + o.logits);
    // a zero state: h, c and h quantized (a block of zeros quantizes to
    // zeros with scale 0), and the joint's halves
    PKB_CUDA(cudaMemsetAsync(w + o.h, 0, o.gates - o.h, st), "cudaMemsetAsync");
    PKB_CUDA(cudaMemsetAsync(w + o.gp, 0, o.qz - o.gp, st), "cudaMemsetAsync");
    PKB_CUDA(cudaMemcpyAsync(w + o.T, T, S * 4, cudaMemcpyHostToDevice, st), "upload");
    PKB_CUDA(cudaMemcpyAsync(w + o.f0, f0, S * 4, cudaMemcpyHostToDevice, st), "upload");
    uint32_t tmax = 0;
    for (uint32_t s = 0; s < S; s++) tmax = T[s] > tmax ? T[s] : tmax;
    // the embedding quantized once a row, as gemv quantizes its input
    if ((rc = quantize_dev(st, reinterpret_cast<int8_t*>(w + o.qembed), reinterpret_cast<float*>(w + o.dembed),
                           m->embed, m->P, m->V + 1, m->P, m->P, rmode)))
        return rc;
    PKB_CUDA(launch_tdt_init(a, st), "tdt launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    const uint32_t P = m->P, J = m->J, L = m->L;
    auto product = [&](float* out, uint32_t rows, const int8_t* wq, const float* ws, const float* bias,
                       const int8_t* q, const float* d, uint32_t n, int add) {
        return gemm_dev(st, out, rows, wq, ws, bias, rows, q, d, n, n, S, add, rmode);
    };
    auto tdt = [&](int phase, uint32_t l) -> int {
        PKB_CUDA(launch_tdt(a, phase, l, rmode, st), "tdt launch");
        g_launches.fetch_add(1, std::memory_order_relaxed);
        return PKB_OK;
    };
    // one round: the prediction network of the segments that emitted (all of
    // them at the first round: the blank's; the other columns' results are
    // not used), then the joint at each running segment's frame and the
    // search's step
    auto round = [&]() -> int {
        for (uint32_t l = 0; l < L; l++) {
            const int8_t* qin = l ? a.qh + static_cast<size_t>(l - 1) * S * P : a.qx;
            const float* din = l ? a.dh + static_cast<size_t>(l - 1) * S : a.dx;
            if ((rc = product(a.gates, 4 * P, m->wx[l], m->wxs[l], m->lb[l], qin, din, P, 0))) return rc;
            if ((rc = product(a.gates, 4 * P, m->wh[l], m->whs[l], nullptr, a.qh + static_cast<size_t>(l) * S * P,
                              a.dh + static_cast<size_t>(l) * S, P, 1)))
                return rc;
            if ((rc = tdt(TDT_LSTM, l))) return rc;
        }
        if ((rc = product(a.gpn, J, m->jpred, m->jpreds, m->jpredb, a.qh + static_cast<size_t>(L - 1) * S * P,
                          a.dh + static_cast<size_t>(L - 1) * S, P, 0)))
            return rc;
        if ((rc = tdt(TDT_JOINT_IN, 0))) return rc;
        if ((rc = product(a.logits, m->n_out_pad, m->jout, m->jouts, m->joutb, a.qz, a.dz, J, 0))) return rc;
        return tdt(TDT_STEP, 0);
    };
    // each round takes every running segment one joint step further or one
    // token on, so T (max_symbols + 1) + 1 rounds end every search
    const uint64_t max_rounds = static_cast<uint64_t>(tmax) * (m->max_symbols + 1) + 2;
    std::vector<uint8_t> states(S * tdt_seg_bytes());
    // The whole search as one cooperative launch where its shared memory
    // fits and the grid can be resident at once (pkb_tdt.cu); otherwise
    // the rounds' launches below.
    const size_t psmem = L <= TDT_MAX_L && max_rounds < (1ull << 31) ? tdt_persist_smem(a, attention_smem_max()) : 0;
    const int pgrid = psmem ? tdt_persist_grid(a, rmode, dev->sms, psmem) : 0;
    bool searched = false;
    if (pgrid > 0) {
        TdtPersist pp = {};
        pp.L = L;
        for (uint32_t l = 0; l < L; l++) {
            pp.wx[l] = m->wx[l];
            pp.wh[l] = m->wh[l];
            pp.wxs[l] = m->wxs[l];
            pp.whs[l] = m->whs[l];
            pp.lb[l] = m->lb[l];
        }
        pp.jpred = m->jpred;
        pp.jpreds = m->jpreds;
        pp.jpredb = m->jpredb;
        pp.jout = m->jout;
        pp.jouts = m->jouts;
        pp.joutb = m->joutb;
        pp.keys = reinterpret_cast<unsigned long long*>(w + o.keys);
        pp.bar = reinterpret_cast<unsigned*>(w + o.bar);
        pp.abort = reinterpret_cast<int*>(w + o.bar + 4);
        pp.err = dev->err;
        pp.timeout = wait_limit();
        pp.max_rounds = static_cast<uint32_t>(max_rounds);
        PKB_CUDA(cudaMemsetAsync(w + o.bar, 0, 8, st), "cudaMemsetAsync");
        const cudaError_t le = launch_tdt_persist(a, pp, rmode, pgrid, psmem, st);
        if (le == cudaErrorCooperativeLaunchTooLarge || le == cudaErrorNotSupported) {
            // the grid cannot be resident at once here (another context's
            // work, a restricted device): the rounds' launches instead
            cudaGetLastError();
        } else {
            PKB_CUDA(le, "tdt launch");
            searched = true;
        }
    }
    if (searched) {
        g_launches.fetch_add(1, std::memory_order_relaxed);
        uint32_t word = 0;
        PKB_CUDA(cudaMemcpyAsync(&word, dev->err, sizeof word, cudaMemcpyDeviceToHost, st), "download");
        PKB_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize");
        if (word) {
            PKB_CUDA(cudaMemsetAsync(dev->err, 0, sizeof word, st), "cudaMemsetAsync");
            PKB_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize");
            return fail(PKB_ETIMEOUT, "tdt: a barrier of the search gave up waiting (device error word 0x%x)", word);
        }
    } else {
        if ((rc = tdt_rounds(round, st, states, w + o.seg, S, L, max_rounds))) return rc;
    }
    PKB_CUDA(cudaMemcpyAsync(states.data(), w + o.seg, states.size(), cudaMemcpyDeviceToHost, st), "download");
    PKB_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    tl_tdt_rounds = 0;
    for (uint32_t s = 0; s < S; s++) {
        const uint32_t* g = reinterpret_cast<const uint32_t*>(states.data() + s * tdt_seg_bytes());
        if (g[TDT_SEG_STEPS] > tl_tdt_rounds) tl_tdt_rounds = g[TDT_SEG_STEPS];
        if (g[TDT_SEG_OVER]) return fail(PKB_EINVAL, "tdt: segment %u found more than %u tokens", s, cap);
        if (g[TDT_SEG_ACTIVE]) return fail(PKB_ETIMEOUT, "tdt: segment %u still searching after %llu rounds", s,
                              static_cast<unsigned long long>(max_rounds));
    }
    return PKB_OK;
}



}  // namespace

int current_device_info(int* sms, uint32_t** err_word) {
    Device* d;
    const int rc = current_device(&d);
    if (rc) return rc;
    *sms = d->sms;
    *err_word = d->err;
    return PKB_OK;
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void count_host_bytes(size_t up, size_t down) {
    g_up.fetch_add(up, std::memory_order_relaxed);
    g_down.fetch_add(down, std::memory_order_relaxed);
}

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(tl_err, sizeof tl_err, fmt, ap);
    va_end(ap);
    return code;
}

}  // namespace pkb

using namespace pkb;

extern "C" {

const char* pkb_last_error(void) { return tl_err; }

int pkb_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    int ok = 0;
    for (int i = 0; i < n; i++) {
        cudaDeviceProp prop;
        if (cudaGetDeviceProperties(&prop, i) == cudaSuccess && prop.major == 10) ok++;
    }
    return ok;
}

int pkb_device_errors(int device, uint32_t* word) {
    int cur = -1;
    PKB_CUDA(cudaGetDevice(&cur), "cudaGetDevice");
    PKB_CUDA(cudaSetDevice(device), "cudaSetDevice");
    uint32_t w = 0;
    const uint32_t zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&w, g_device_error, sizeof w);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof zero);
    cudaSetDevice(cur);
    if (e != cudaSuccess) return cuda_fail(e, "error word read");
    if (word) *word = w;
    return PKB_OK;
}

uint64_t pkb_launch_count(void) { return g_launches.load(); }

void pkb_host_bytes(uint64_t* up, uint64_t* down) {
    if (up) *up = g_up.load();
    if (down) *down = g_down.load();
}

size_t pkb_wpack_bytes(uint32_t rows, uint32_t n) { return static_cast<size_t>(rows) * n; }

int pkb_layernorm_quantize_dev(void* stream, int8_t* q, float* d, const float* x, size_t xs, uint32_t T, uint32_t n,
                               uint32_t qb, const float* w, const float* b, float eps, int rmode) {
    return pkb::layernorm_quantize_dev(static_cast<cudaStream_t>(stream), q, d, x, xs, T, n, qb, w, b, eps, rmode);
}

int pkb_layernorm_dev(void* stream, float* out, size_t os, const float* x, size_t xs, uint32_t T, uint32_t n,
                      const float* w, const float* b, float eps, int rmode) {
    return pkb::layernorm_dev(static_cast<cudaStream_t>(stream), out, os, x, xs, T, n, w, b, eps, rmode);
}

int pkb_silu_quantize_dev(void* stream, int8_t* q, float* d, const float* u, size_t us, uint32_t T, uint32_t n,
                          uint32_t qb, int rmode) {
    return pkb::silu_quantize_dev(static_cast<cudaStream_t>(stream), q, d, u, us, T, n, qb, rmode);
}

int pkb_dwconv_quantize_dev(void* stream, int8_t* q, float* d, float* out, size_t os, const float* x, size_t xs,
                            uint32_t T, uint32_t C, const float* w, const float* b, uint32_t K, int glu, uint32_t qb,
                            int rmode) {
    return pkb::dwconv_quantize_dev(static_cast<cudaStream_t>(stream), q, d, out, os, x, xs, T, C, w, b, K, glu, qb,
                                    rmode);
}

int pkb_gemm_f32_dev(void* stream, float* out, size_t os, const float* w, uint32_t ld, uint32_t rows, uint32_t n,
                     const float* x, size_t xs, uint32_t T, const float* bias, size_t bs, int relu, int rmode) {
    return pkb::gemm_f32_dev(static_cast<cudaStream_t>(stream), out, os, w, ld, rows, n, x, xs, T, bias, bs, relu,
                             rmode);
}

int pkb_softmax_dev(void* stream, float* x, size_t xs, uint32_t T, uint32_t n, float scale, int rmode) {
    return pkb::softmax_dev(static_cast<cudaStream_t>(stream), x, xs, T, n, scale, rmode);
}

int pkb_attention_dev(void* stream, float* o, size_t os, const float* q, size_t qs, const float* kp, const float* pp,
                      const float* vp, const float* bias_u, const float* bias_v, uint32_t T, uint32_t D, uint32_t H,
                      int rmode) {
    const pkb_att_segment seg = {T, 0, 0};
    return pkb::attention_dev(static_cast<cudaStream_t>(stream), true, o, os, q, qs, kp, 0, vp, 0, pp, 0, bias_u,
                              bias_v, D, H, &seg, 1, rmode);
}

int pkb_attention_rows_dev(void* stream, float* o, size_t os, const float* q, size_t qs, const float* k, size_t ks,
                           const float* v, size_t vs, const float* p, size_t ps, const float* bias_u,
                           const float* bias_v, uint32_t D, uint32_t H, const pkb_att_segment* segs, uint32_t nseg,
                           int rmode) {
    return pkb::attention_dev(static_cast<cudaStream_t>(stream), false, o, os, q, qs, k, ks, v, vs, p, ps, bias_u,
                              bias_v, D, H, segs, nseg, rmode);
}

uint64_t pkb_tdt_last_rounds(void) { return pkb::tl_tdt_rounds; }

size_t pkb_tdt_work_bytes(const pkb_tdt_model* m, uint32_t S) {
    return m && S ? pkb::tdt_layout(*m, S).total : 0;
}

int pkb_tdt_search_dev(void* stream, const pkb_tdt_model* m, const float* f, const uint32_t* f0, const uint32_t* T,
                       uint32_t S, int32_t* toks, uint32_t* ntok, uint32_t cap, void* work, size_t work_bytes,
                       int rmode) {
    return pkb::tdt_search_dev(static_cast<cudaStream_t>(stream), m, f, f0, T, S, toks, ntok, cap, work, work_bytes,
                               rmode);
}

int pkb_gemm_q8_panels_dev(void* stream, float* panels, int kind, size_t ps, uint32_t dk, uint32_t tpad,
                           const int8_t* wpack, const float* ws, uint32_t rows, const int8_t* q, const float* d,
                           uint32_t n, uint32_t qb, uint32_t T, int rmode) {
    return gemm_panels_dev(static_cast<cudaStream_t>(stream), panels, kind, ps, dk, tpad, wpack, ws, rows, q, d, n, qb,
                           T, rmode);
}

int pkb_repack_q8_dev(void* stream, int8_t* wpack, const int8_t* w_pk, uint32_t rows, uint32_t n) {
    return repack_dev(static_cast<cudaStream_t>(stream), wpack, w_pk, rows, n);
}

int pkb_quantize_dev(void* stream, int8_t* q, float* d, const float* x, size_t xs, uint32_t T, uint32_t n,
                     uint32_t qb, int rmode) {
    return quantize_dev(static_cast<cudaStream_t>(stream), q, d, x, xs, T, n, qb, rmode);
}

int pkb_gemm_q8_dev(void* stream, float* out, size_t os, const int8_t* wpack, const float* ws, const float* bias,
                    uint32_t rows, const int8_t* q, const float* d, uint32_t n, uint32_t qb, uint32_t T, int add,
                    int rmode) {
    return gemm_dev(static_cast<cudaStream_t>(stream), out, os, wpack, ws, bias, rows, q, d, n, qb, T, add, rmode);
}

}  // extern "C"
