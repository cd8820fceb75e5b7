// The producers of the product's int8 inputs, fused with the float step
// that makes each input, sm_100a. The reference's encoder makes each such
// input as a float row in thread scratch and quantizes it at once; here the
// row never leaves the SM.
//
//   layernorm_quantize  normq (core/encoder.c:112-130): k_layernorm
//                       (backend/ref/kernels.c:109-131) into a row, then
//                       pk_quant_part (core/passes.c:114-118) of the row
//   SiLU, quantize      siluq_tile (core/encoder.c:150-158): in
//                       pkb_quantize.cu, the quantizer's SILU form
//   dwconv_quantize     glu_item + dw_item (core/encoder.c:160-183): k_glu
//                       (backend/ref/kernels.c:157-161) where asked, k_dwconv
//                       (:163-177), then pk_quant_part a frame at a time
//
// Every float operation is the reference's, in its order, rounded once in
// the mode RM; the quantization is k_quantize's (backend/ref/kernels.c:24-58)
// on blocks of 32 or 64 (the encoder's qb(), core/encoder.c:56).

#include "pkb_device.cuh"
#include "pkb_internal.h"
#include "pkb_vmath.cuh"

namespace pkb {

namespace {

// ------------------------------------------------------ layer norm, quantize --

// The reference's lanes_sum (backend/ref/kernels.c:109-113) over the 16
// lanes of a half-warp, lane j holding acc[j]: acc[i] += acc[i + h] for h =
// 8, 4, 2, 1, then acc[0] to every lane of the half.
template <int RM>
__device__ __forceinline__ float fold16(float a) {
#pragma unroll
    for (int h = 8; h >= 1; h >>= 1) a = add_r<RM>(a, __shfl_down_sync(0xffffffffu, a, h, 16));
    return __shfl_sync(0xffffffffu, a, 0, 16);
}

// Rows of n floats (n a multiple of QB, QB 32 or 64), two a warp, a
// half-warp each, the row staged in shared memory. The two sums are the
// reference's 16 lane sums exactly: lane j adds inputs j, j + 16, j + 32, ...
// in order, then the fold. The normalized row is then quantized a block at
// a time, lane j taking 8 consecutive inputs at 8j + 128k (QB / 8 lanes a
// block, reduced by shuffles).
template <int RM, int QB>
__global__ void __launch_bounds__(256) layernorm_quantize(int8_t* __restrict__ q, float* __restrict__ d,
                                                          const float* __restrict__ x, size_t xs, uint32_t T,
                                                          uint32_t n, const float* __restrict__ w,
                                                          const float* __restrict__ b, float eps, bool xvec,
                                                          bool wvec, bool q8) {
    extern __shared__ float4 ln_smem[];
    pdl_trigger();
    pdl_wait();
    constexpr uint32_t GL = QB / 8;  // lanes a block
    const uint32_t lane = threadIdx.x & 31, half = lane >> 4, j = lane & 15, warp = threadIdx.x >> 5;
    const uint32_t wpb = blockDim.x >> 5;
    const uint32_t pitch = n + 16;  // the halves' rows 16 banks apart
    float* row = reinterpret_cast<float*>(ln_smem) + static_cast<size_t>(2 * warp + half) * pitch;
    const uint32_t nb = n / QB;
    const float fn = static_cast<float>(n);  // exact: n <= 2^24
    for (uint32_t t0 = 2 * (blockIdx.x * wpb + warp); t0 < T; t0 += 2 * gridDim.x * wpb) {  // warp-uniform
        const uint32_t t = t0 + half;
        const bool live = t < T;
        const float* xr = x + static_cast<size_t>(live ? t : t0) * xs;  // a dead half reads its twin's row
        if (xvec) {
            for (uint32_t i = 4 * j; i < n; i += 64)
                *reinterpret_cast<float4*>(row + i) = __ldg(reinterpret_cast<const float4*>(xr + i));
        } else {
            for (uint32_t i = j; i < n; i += 16) row[i] = __ldg(xr + i);
        }
        __syncwarp();

        // mean = sum / n; var = sum((x - mean)^2) / n; r = 1 / sqrt(var + eps)
        float acc = 0.0f;
        for (uint32_t i = j; i < n; i += 16) acc = add_r<RM>(acc, row[i]);
        const float mean = div_r<RM>(fold16<RM>(acc), fn);
        acc = 0.0f;
        for (uint32_t i = j; i < n; i += 16) {
            const float c = sub_r<RM>(row[i], mean);
            acc = add_r<RM>(acc, mul_r<RM>(c, c));
        }
        const float var = div_r<RM>(fold16<RM>(acc), fn);
        const float rs = div_r<RM>(1.0f, sqrt_r<RM>(add_r<RM>(var, eps)));

        // out = (x - mean) * r * w + b, left to right; then its blocks
        for (uint32_t k0 = 0; k0 < n; k0 += 128) {  // the same trip count on every lane
            const uint32_t i0 = k0 + 8 * j;
            const bool in = i0 < n;  // a block is all in or all out (n a multiple of QB)
            float v[8];
            uint32_t m = 0;
            if (in) {
                float xv[8], wv[8], bv[8];
                *reinterpret_cast<float4*>(xv) = *reinterpret_cast<const float4*>(row + i0);
                *reinterpret_cast<float4*>(xv + 4) = *reinterpret_cast<const float4*>(row + i0 + 4);
                if (wvec) {
                    *reinterpret_cast<float4*>(wv) = __ldg(reinterpret_cast<const float4*>(w + i0));
                    *reinterpret_cast<float4*>(wv + 4) = __ldg(reinterpret_cast<const float4*>(w + i0 + 4));
                    *reinterpret_cast<float4*>(bv) = __ldg(reinterpret_cast<const float4*>(b + i0));
                    *reinterpret_cast<float4*>(bv + 4) = __ldg(reinterpret_cast<const float4*>(b + i0 + 4));
                } else {
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        wv[e] = __ldg(w + i0 + e);
                        bv[e] = __ldg(b + i0 + e);
                    }
                }
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    v[e] = add_r<RM>(mul_r<RM>(mul_r<RM>(sub_r<RM>(xv[e], mean), rs), wv[e]), bv[e]);
                    m = max(m, abs_bits(v[e]));
                }
            }
#pragma unroll
            for (uint32_t off = GL / 2; off >= 1; off >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, off));
            if (in && live) {
                uint32_t p0 = 0, p1 = 0;
                float scale = 0.0f;
                if (block_scaled(m)) {
                    const float amax = __uint_as_float(m);
                    scale = div_r<RM>(amax, 127.0f);
                    const float id = div_r<RM>(127.0f, amax);
                    p0 = quant4<RM>(make_float4(v[0], v[1], v[2], v[3]), id);
                    p1 = quant4<RM>(make_float4(v[4], v[5], v[6], v[7]), id);
                }
                int8_t* qo = q + static_cast<size_t>(t) * n + i0;
                if (q8) {
                    *reinterpret_cast<uint2*>(qo) = make_uint2(p0, p1);
                } else {
                    *reinterpret_cast<uint32_t*>(qo) = p0;
                    *reinterpret_cast<uint32_t*>(qo + 4) = p1;
                }
                if (j % GL == 0) d[static_cast<size_t>(t) * nb + i0 / QB] = scale;
            }
        }
        __syncwarp();  // the row buffer is refilled next
    }
}

// -------------------------------------------- (GLU,) dwconv, SiLU, quantize --

constexpr int DW_FRAMES = 32;  // output frames a CTA
constexpr int DW_CH = 64;      // channels a CTA, two a lane
constexpr int DW_THREADS = 256;

// A tile of DW_FRAMES frames by 64 channels a CTA. The input rows its taps
// reach (its frames and K/2 either side) are staged in shared memory, made
// from pw1's output by the reference's GLU on the way in where GLU; the
// tile's taps are staged tap-major. Then a warp takes a frame at a time,
// two adjacent channels a lane: the taps in order, each reading padding
// skipped as the reference skips it (an fma with a zero is not the same
// bits: -0 under RD, NaN for an infinite tap), + bias, SiLU, and the frame's
// blocks of QB channels reduced across QB / 2 lanes.
template <int RM, int QB, bool GLU>
__global__ void __launch_bounds__(DW_THREADS) dwconv_quantize(int8_t* __restrict__ q, float* __restrict__ d,
                                                              float* __restrict__ out, size_t os,
                                                              const float* __restrict__ x, size_t xs, uint32_t T,
                                                              uint32_t C, const float* __restrict__ w,
                                                              const float* __restrict__ bias, uint32_t K) {
    extern __shared__ float4 dw_smem[];
    pdl_trigger();
    pdl_wait();
    const uint32_t rows = DW_FRAMES + K - 1;
    float* tile = reinterpret_cast<float*>(dw_smem);  // [rows][DW_CH]
    float* taps = tile + rows * DW_CH;                // [K][DW_CH]
    const uint32_t t0 = blockIdx.x * DW_FRAMES, c0 = blockIdx.y * DW_CH;
    const int64_t hk = K / 2;
    for (uint32_t i = threadIdx.x; i < rows * DW_CH; i += DW_THREADS) {
        const uint32_t r = i / DW_CH, c = i % DW_CH;
        const int64_t s = static_cast<int64_t>(t0) + r - hk;
        float v = 0.0f;  // never read: the taps past either end are skipped
        if (s >= 0 && s < T && c0 + c < C) {
            const float* xr = x + static_cast<size_t>(s) * xs + c0 + c;
            if constexpr (GLU)
                v = mul_r<RM>(__ldg(xr), pk_sigmoid<RM>(__ldg(xr + C)));  // out[i] = a[i] * sigmoid(a[i + n])
            else
                v = __ldg(xr);
        }
        tile[i] = v;
    }
    for (uint32_t i = threadIdx.x; i < K * DW_CH; i += DW_THREADS) {
        const uint32_t jt = i / DW_CH, c = i % DW_CH;
        taps[i] = c0 + c < C ? __ldg(w + static_cast<size_t>(c0 + c) * K + jt) : 0.0f;
    }
    __syncthreads();

    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t cl = 2 * lane, ca = c0 + cl;
    const bool cin = ca < C;  // C even: both of the lane's channels, or neither
    const float b0 = cin ? __ldg(bias + ca) : 0.0f, b1 = cin ? __ldg(bias + ca + 1) : 0.0f;
    const uint32_t nb = C / QB;
    for (uint32_t f = warp; f < DW_FRAMES; f += DW_THREADS / 32) {
        const uint32_t t = t0 + f;
        if (t >= T) break;  // warp-uniform
        float a0 = 0.0f, a1 = 0.0f;
        for (uint32_t jt = 0; jt < K; jt++) {
            const int64_t s = static_cast<int64_t>(t) + jt - hk;
            if (s < 0 || s >= T) continue;  // warp-uniform
            const float2 xv = *reinterpret_cast<const float2*>(tile + (f + jt) * DW_CH + cl);
            const float2 wv = *reinterpret_cast<const float2*>(taps + jt * DW_CH + cl);
            a0 = fma_r<RM>(wv.x, xv.x, a0);
            a1 = fma_r<RM>(wv.y, xv.y, a1);
        }
        const float v0 = add_r<RM>(a0, b0), v1 = add_r<RM>(a1, b1);
        const float o0 = mul_r<RM>(v0, pk_sigmoid<RM>(v0)), o1 = mul_r<RM>(v1, pk_sigmoid<RM>(v1));
        if (out && cin) {
            out[static_cast<size_t>(t) * os + ca] = o0;
            out[static_cast<size_t>(t) * os + ca + 1] = o1;
        }
        uint32_t m = cin ? max(abs_bits(o0), abs_bits(o1)) : 0u;
        if constexpr (QB == 64) {
            m = __reduce_max_sync(0xffffffffu, m);
        } else {
#pragma unroll
            for (uint32_t off = 8; off >= 1; off >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, off));
        }
        if (cin) {
            uint32_t pq = 0;
            float scale = 0.0f;
            if (block_scaled(m)) {
                const float amax = __uint_as_float(m);
                scale = div_r<RM>(amax, 127.0f);
                const float id = div_r<RM>(127.0f, amax);
                pq = quant1<RM>(o0, id) | (quant1<RM>(o1, id) << 8);
            }
            *reinterpret_cast<uint16_t*>(q + static_cast<size_t>(t) * C + ca) = static_cast<uint16_t>(pq);
            if (lane % (QB / 2) == 0) d[static_cast<size_t>(t) * nb + ca / QB] = scale;
        }
    }
}

// --------------------------------------------------------------- launches --

constexpr size_t LN_SMEM_CAP = 96 * 1024;

template <int RM, int QB>
cudaError_t ln_launch(int8_t* q, float* d, const float* x, size_t xs, uint32_t T, uint32_t n, const float* w,
                      const float* b, float eps, int num_sms, cudaStream_t stream) {
    const size_t per_warp = 2 * static_cast<size_t>(n + 16) * sizeof(float);
    size_t warps = LN_SMEM_CAP / per_warp;
    if (warps > 8) warps = 8;
    if (warps < 1) return cudaErrorInvalidValue;  // n beyond the checked maximum
    const size_t smem = warps * per_warp;
    auto kern = layernorm_quantize<RM, QB>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const size_t pairs = (static_cast<size_t>(T) + 1) / 2;
    size_t grid = (pairs + warps - 1) / warps;
    const size_t cap = static_cast<size_t>(num_sms) * (LN_SMEM_CAP * 2 / smem + 1);
    if (grid > cap) grid = cap;
    const bool xvec = reinterpret_cast<uintptr_t>(x) % 16 == 0 && xs % 4 == 0;
    const bool wvec = reinterpret_cast<uintptr_t>(w) % 16 == 0 && reinterpret_cast<uintptr_t>(b) % 16 == 0;
    const bool q8 = reinterpret_cast<uintptr_t>(q) % 8 == 0;
    return launch_pdl(kern, dim3(static_cast<unsigned>(grid)), dim3(static_cast<unsigned>(32 * warps)), smem, stream,
                      q, d, x, xs, T, n, w, b, eps, xvec, wvec, q8);
}

template <int RM, int QB>
cudaError_t dw_launch(int8_t* q, float* d, float* out, size_t os, const float* x, size_t xs, uint32_t T, uint32_t C,
                      const float* w, const float* bias, uint32_t K, bool glu, cudaStream_t stream) {
    const size_t smem = (static_cast<size_t>(DW_FRAMES + K - 1) + K) * DW_CH * sizeof(float);
    const dim3 grid((T + DW_FRAMES - 1) / DW_FRAMES, (C + DW_CH - 1) / DW_CH);
    if (glu)
        return launch_pdl(dwconv_quantize<RM, QB, true>, grid, dim3(DW_THREADS), smem, stream, q, d, out, os, x, xs,
                          T, C, w, bias, K);
    return launch_pdl(dwconv_quantize<RM, QB, false>, grid, dim3(DW_THREADS), smem, stream, q, d, out, os, x, xs, T,
                      C, w, bias, K);
}

template <int RM>
cudaError_t ln_rm(int8_t* q, float* d, const float* x, size_t xs, uint32_t T, uint32_t n, uint32_t qb,
                  const float* w, const float* b, float eps, int num_sms, cudaStream_t stream) {
    if (qb == 32) return ln_launch<RM, 32>(q, d, x, xs, T, n, w, b, eps, num_sms, stream);
    if (qb == 64) return ln_launch<RM, 64>(q, d, x, xs, T, n, w, b, eps, num_sms, stream);
    return cudaErrorInvalidValue;
}

template <int RM>
cudaError_t dw_rm(int8_t* q, float* d, float* out, size_t os, const float* x, size_t xs, uint32_t T, uint32_t C,
                  const float* w, const float* bias, uint32_t K, bool glu, uint32_t qb, cudaStream_t stream) {
    if (qb == 32) return dw_launch<RM, 32>(q, d, out, os, x, xs, T, C, w, bias, K, glu, stream);
    if (qb == 64) return dw_launch<RM, 64>(q, d, out, os, x, xs, T, C, w, bias, K, glu, stream);
    return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_layernorm_quantize(int8_t* q, float* d, const float* x, size_t xs, uint32_t T, uint32_t n,
                                      uint32_t qb, const float* w, const float* b, float eps, int rmode,
                                      int num_sms, cudaStream_t stream) {
    switch (rmode) {
    case 1: return ln_rm<1>(q, d, x, xs, T, n, qb, w, b, eps, num_sms, stream);
    case 2: return ln_rm<2>(q, d, x, xs, T, n, qb, w, b, eps, num_sms, stream);
    case 3: return ln_rm<3>(q, d, x, xs, T, n, qb, w, b, eps, num_sms, stream);
    default: return ln_rm<0>(q, d, x, xs, T, n, qb, w, b, eps, num_sms, stream);
    }
}

cudaError_t launch_dwconv_quantize(int8_t* q, float* d, float* out, size_t os, const float* x, size_t xs, uint32_t T,
                                   uint32_t C, const float* w, const float* bias, uint32_t K, bool glu, uint32_t qb,
                                   int rmode, cudaStream_t stream) {
    switch (rmode) {
    case 1: return dw_rm<1>(q, d, out, os, x, xs, T, C, w, bias, K, glu, qb, stream);
    case 2: return dw_rm<2>(q, d, out, os, x, xs, T, C, w, bias, K, glu, qb, stream);
    case 3: return dw_rm<3>(q, d, out, os, x, xs, T, C, w, bias, K, glu, qb, stream);
    default: return dw_rm<0>(q, d, out, os, x, xs, T, C, w, bias, K, glu, qb, stream);
    }
}

}  // namespace pkb
