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

#include <type_traits>

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

// A row in shared memory: float i at i + 4 (i / 32), four floats of gap a
// run of 32. Reads of 16 consecutive floats (the sums' lanes) and 16-byte
// reads of one run by each of 8 lanes (a block a lane) are then both free of
// bank conflicts, and every run starts 16-byte aligned.
__device__ __forceinline__ uint32_t ln_at(uint32_t i) { return i + 4 * (i >> 5); }
__host__ __device__ constexpr uint32_t ln_padded(uint32_t n) { return n + 4 * (n / 32); }
// floats a staged row takes: its padded length rounded so that the two rows
// of a warp sit 16 banks apart
__host__ __device__ constexpr uint32_t ln_pitch(uint32_t n) { return (ln_padded(n) + 31) / 32 * 32 + 16; }

// NC: n / 16 where n is 1024 (the FastConformer's d_model), compiled with
// the row's sums in registers; 0 for any other n, summed from shared memory
constexpr uint32_t LN_NC = 64;

// Block k of ROWS staged rows (the second pitch floats after the first, for
// frames t0 and t0 + 1; the second only if live1): (x - mean) * r * w + b,
// left to right, each chunk's w and b read once for the rows; then each
// row's block quantized, its bytes stored 16 at a time where q16 (FOUT: the
// floats stored instead, at out + t os, 16 bytes at a time where ov).
template <int RM, int QB, int ROWS, bool FOUT>
__device__ __forceinline__ void ln_block(int8_t* __restrict__ q, float* __restrict__ d, float* out, size_t os,
                                         const float* rows, uint32_t pitch, const float* ws, const float* bs,
                                         uint32_t k, uint32_t t0, bool live1, uint32_t n, uint32_t nb, float mean0,
                                         float rs0, float mean1, float rs1, bool q16) {
    float4 v[ROWS][QB / 4];
    uint32_t m[ROWS] = {};
    const uint64_t nm[2] = {pack2(-mean0, -mean0), pack2(-mean1, -mean1)};
    const uint64_t rs[2] = {pack2(rs0, rs0), pack2(rs1, rs1)};
#pragma unroll
    for (int c = 0; c < QB / 4; c++) {
        const uint32_t at = ln_at(k * QB + 4 * c);
        const float4 wv = *reinterpret_cast<const float4*>(ws + at);
        const float4 bv = *reinterpret_cast<const float4*>(bs + at);
#pragma unroll
        for (int r = 0; r < ROWS; r++) {
            const float4 xv = *reinterpret_cast<const float4*>(rows + r * pitch + at);
            // (x - mean) * r on pairs; the multiply by w and the add of b one
            // at a time, so that the two never fuse
            float a0, a1, a2, a3;
            unpack2(mul2_r<RM>(add2_r<RM>(pack2(xv.x, xv.y), nm[r]), rs[r]), a0, a1);
            unpack2(mul2_r<RM>(add2_r<RM>(pack2(xv.z, xv.w), nm[r]), rs[r]), a2, a3);
            v[r][c] = make_float4(add_r<RM>(mul_r<RM>(a0, wv.x), bv.x), add_r<RM>(mul_r<RM>(a1, wv.y), bv.y),
                                  add_r<RM>(mul_r<RM>(a2, wv.z), bv.z), add_r<RM>(mul_r<RM>(a3, wv.w), bv.w));
            m[r] = max(m[r], max(max(abs_bits(v[r][c].x), abs_bits(v[r][c].y)),
                                 max(abs_bits(v[r][c].z), abs_bits(v[r][c].w))));
        }
    }
    if constexpr (FOUT) {
#pragma unroll
        for (int r = 0; r < ROWS; r++) {
            if (r == 1 && !live1) break;
            float* o = out + static_cast<size_t>(t0 + r) * os + k * QB;
            if (q16) {  // out 16-byte aligned, os a multiple of 4
#pragma unroll
                for (int c = 0; c < QB / 4; c++) *reinterpret_cast<float4*>(o + 4 * c) = v[r][c];
            } else {
#pragma unroll
                for (int c = 0; c < QB / 4; c++) {
                    o[4 * c] = v[r][c].x;
                    o[4 * c + 1] = v[r][c].y;
                    o[4 * c + 2] = v[r][c].z;
                    o[4 * c + 3] = v[r][c].w;
                }
            }
        }
        return;
    }
#pragma unroll
    for (int r = 0; r < ROWS; r++) {
        if (r == 1 && !live1) break;
        uint32_t packed[QB / 4];
        float scale = 0.0f;
        if (block_scaled(m[r])) {
            const float amax = __uint_as_float(m[r]);
            scale = div_r<RM>(amax, 127.0f);
            const float id = div_r<RM>(127.0f, amax);
#pragma unroll
            for (int c = 0; c < QB / 4; c++) packed[c] = quant4<RM>(v[r][c], id);
        } else {
#pragma unroll
            for (int c = 0; c < QB / 4; c++) packed[c] = 0;
        }
        const size_t t = t0 + r;
        int8_t* qo = q + t * n + k * QB;
        if (q16) {
#pragma unroll
            for (int c = 0; c < QB / 16; c++)
                *reinterpret_cast<uint4*>(qo + 16 * c) =
                    make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
        } else {
#pragma unroll
            for (int c = 0; c < QB / 4; c++) *reinterpret_cast<uint32_t*>(qo + 4 * c) = packed[c];
        }
        d[t * nb + k] = scale;
    }
}

// Rows of n floats (n a multiple of QB, QB 32 or 64), two a warp. w and b
// are staged once a CTA; each warp's pair of rows comes in by asynchronous
// copies into one of two buffers while the warp works on the pair before.
//
// The sums: a half-warp a row, lane j adding inputs j, j + 16, j + 32, ...
// in order (the reference's 16 lanes, backend/ref/kernels.c:119-129), then
// the fold. The normalized values and their quantization: a lane a block,
// so that a block's maximum and its two divisions stay in one thread, the
// arithmetic on pairs of inputs (f32x2, each half rounded as the scalar
// operation), the bytes stored 16 at a time where q allows.
//
// FOUT: k_layernorm alone, the normalized floats stored at out + t os
// instead of quantized. out may be x itself (the reference's out norm runs
// in place): a row is read only by the asynchronous copies into shared
// memory, which complete before the warp stores any of its floats, and no
// other warp touches it.
template <int RM, int QB, uint32_t NC, bool FOUT>
__global__ void __launch_bounds__(256) layernorm_quantize(int8_t* __restrict__ q, float* __restrict__ d, float* out,
                                                          size_t os, const float* x, size_t xs, uint32_t T,
                                                          uint32_t n, const float* __restrict__ w,
                                                          const float* __restrict__ b, float eps, bool xvec,
                                                          bool q16) {
    extern __shared__ float4 ln_smem[];
    pdl_trigger();
    pdl_wait();
    const uint32_t lane = threadIdx.x & 31, half = lane >> 4, j = lane & 15, warp = threadIdx.x >> 5;
    const uint32_t wpb = blockDim.x >> 5;
    const uint32_t padded = ln_padded(n), pitch = ln_pitch(n);
    float* ws = reinterpret_cast<float*>(ln_smem);
    float* bs = ws + padded;
    float* bufs = bs + padded + static_cast<size_t>(warp) * 4 * pitch;  // [stage][row][pitch]
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        ws[ln_at(i)] = __ldg(w + i);
        bs[ln_at(i)] = __ldg(b + i);
    }
    __syncthreads();

    const uint32_t pairs = (T + 1) / 2, nb = n / QB;
    const float fn = static_cast<float>(n);  // exact: n <= 2^24
    // the pair's two rows into stage st: lane j of half h copies row h's
    // chunks 4j, 4j + 64, ... (a dead second row copies the first again)
    auto stage_in = [&](uint32_t pr, uint32_t st) {
        const uint32_t t = 2 * pr + half < T ? 2 * pr + half : 2 * pr;
        const float* xr = x + static_cast<size_t>(t) * xs;
        float* row = bufs + (2 * st + half) * pitch;
        if (xvec) {
            for (uint32_t i = 4 * j; i < n; i += 64) cp_async16(row + ln_at(i), xr + i);
        } else {
            for (uint32_t i = j; i < n; i += 16) cp_async4(row + ln_at(i), xr + i);
        }
    };
    uint32_t pr = blockIdx.x * wpb + warp;
    const uint32_t stride = gridDim.x * wpb;
    if (pr < pairs) stage_in(pr, 0);
    cp_async_commit();
    for (uint32_t st = 0; pr < pairs; pr += stride, st ^= 1) {  // warp-uniform
        if (pr + stride < pairs) stage_in(pr + stride, st ^ 1);
        cp_async_commit();
        cp_async_wait<1>();  // this pair's copies (every lane's) have landed
        __syncwarp();
        const float* rows = bufs + 2 * st * pitch;
        const float* row = rows + half * pitch;

        // mean = sum / n; var = sum((x - mean)^2) / n; r = 1 / sqrt(var + eps)
        float acc = 0.0f, mean, var;
        if (NC > 0) {
            // n = 16 NC, known at compile time: the lane's NC inputs held in
            // registers between the two sums
            float xv[NC > 0 ? NC : 1];
#pragma unroll
            for (uint32_t k = 0; k < NC; k++) {
                xv[k] = row[ln_at(16 * k + j)];
                acc = add_r<RM>(acc, xv[k]);
            }
            mean = div_r<RM>(fold16<RM>(acc), fn);
            acc = 0.0f;
#pragma unroll
            for (uint32_t k = 0; k < NC; k++) {
                const float c = sub_r<RM>(xv[k], mean);
                acc = add_r<RM>(acc, mul_r<RM>(c, c));
            }
        } else {
#pragma unroll 8
            for (uint32_t i = j; i < n; i += 16) acc = add_r<RM>(acc, row[ln_at(i)]);
            mean = div_r<RM>(fold16<RM>(acc), fn);
            acc = 0.0f;
#pragma unroll 8
            for (uint32_t i = j; i < n; i += 16) {
                const float c = sub_r<RM>(row[ln_at(i)], mean);
                acc = add_r<RM>(acc, mul_r<RM>(c, c));
            }
        }
        var = div_r<RM>(fold16<RM>(acc), fn);
        const float rs = div_r<RM>(1.0f, sqrt_r<RM>(add_r<RM>(var, eps)));
        const float mean0 = __shfl_sync(0xffffffffu, mean, 0), mean1 = __shfl_sync(0xffffffffu, mean, 16);
        const float rs0 = __shfl_sync(0xffffffffu, rs, 0), rs1 = __shfl_sync(0xffffffffu, rs, 16);

        // out = (x - mean) * r * w + b, left to right, a block a lane. With
        // 32 blocks a row or more (and blocks of 32), lane l takes block l
        // (l + 32, ...) of both rows, reading its w and b once for the two;
        // otherwise the pair's 2 nb blocks are dealt over the lanes.
        const bool live1 = 2 * pr + 1 < T;
        if (QB == 32 && nb >= 32) {
            for (uint32_t k = lane; k < nb; k += 32)
                ln_block<RM, QB, 2, FOUT>(q, d, out, os, rows, pitch, ws, bs, k, 2 * pr, live1, n, nb, mean0, rs0,
                                          mean1, rs1, q16);
        } else {
            for (uint32_t item = lane; item < 2 * nb; item += 32) {
                const uint32_t r = item >= nb, k = item - r * nb;
                if (r && !live1) continue;
                ln_block<RM, QB, 1, FOUT>(q, d, out, os, rows + r * pitch, pitch, ws, bs, k, 2 * pr + r, false, n,
                                          nb, r ? mean1 : mean0, r ? rs1 : rs0, 0.0f, 0.0f, q16);
            }
        }
        __syncwarp();  // the stage is refilled two pairs on
    }
    cp_async_wait<0>();
}

// -------------------------------------------- (GLU,) dwconv, SiLU, quantize --

constexpr int DW_FRAMES = 32;  // output frames a CTA
constexpr int DW_CH = 64;      // channels a CTA, two a lane
constexpr int DW_THREADS = 256;

// A tile of DW_FRAMES frames by 64 channels a CTA. The input rows its taps
// reach (its frames and K/2 either side) are staged in shared memory, two
// channels a thread, made from pw1's output by the reference's GLU on the
// way in where GLU; the tile's taps are staged tap-major. Then a warp takes
// a frame at a time, two adjacent channels a lane: the taps in order as one
// fused multiply-add on the pair (f32x2: each half the reference's fmaf),
// those reading past either end skipped as the reference skips them (an fma
// with a zero is not the same bits: -0 under RD, NaN for an infinite tap),
// + bias, SiLU, and the frame's blocks of QB channels reduced across QB / 2
// lanes. KC: the tap count where it is known at compile time (9, the
// FastConformer's kernel: the taps then stay in registers and the staging's
// loads all go out before any is used), or 0.
template <int RM, int QB, bool GLU, int KC>
__global__ void __launch_bounds__(DW_THREADS) dwconv_quantize(int8_t* __restrict__ q, float* __restrict__ d,
                                                              float* __restrict__ out, size_t os,
                                                              const float* __restrict__ x, size_t xs, uint32_t T,
                                                              uint32_t C, const float* __restrict__ w,
                                                              const float* __restrict__ bias, uint32_t Krt, bool xv2) {
    extern __shared__ float4 dw_smem[];
    pdl_trigger();
    pdl_wait();
    const uint32_t K = KC ? KC : Krt;
    const uint32_t rows = DW_FRAMES + K - 1;
    float* tile = reinterpret_cast<float*>(dw_smem);  // [rows][DW_CH]
    float* taps = tile + rows * DW_CH;                // [K][DW_CH]
    const uint32_t t0 = blockIdx.x * DW_FRAMES, c0 = blockIdx.y * DW_CH;
    const uint32_t hk = K / 2;
    constexpr uint32_t PR = DW_CH / 2;  // channel pairs a row

    // the staged input, a channel pair at a time: GLU or a copy
    auto load2 = [&](const float* p) -> float2 {
        return xv2 ? __ldg(reinterpret_cast<const float2*>(p)) : make_float2(__ldg(p), __ldg(p + 1));
    };
    auto live = [&](uint32_t i, const float*& xr) -> bool {
        const uint32_t r = i / PR, c = c0 + 2 * (i % PR);
        const int64_t s = static_cast<int64_t>(t0) + r - static_cast<int64_t>(hk);
        const bool ok = i < rows * PR && s >= 0 && s < T && c < C;
        xr = ok ? x + static_cast<size_t>(s) * xs + c : x;  // only a live row's address is formed
        return ok;
    };
    // items a thread stages, its pairs' values a and gates g (GLU) as one
    // batch: out[i] = a[i] * sigmoid(a[i + n]); rows past either end are
    // left 0 and never read (the taps there are skipped)
    auto stage = [&](auto items_tag, uint32_t first) {
        constexpr uint32_t ITEMS = decltype(items_tag)::value;
        float2 a[ITEMS];
        float gv[2 * ITEMS];
        bool ok[ITEMS];
#pragma unroll
        for (uint32_t k = 0; k < ITEMS; k++) {
            const float* xr;
            ok[k] = live(first + k * DW_THREADS, xr);
            a[k] = ok[k] ? load2(xr) : make_float2(0.0f, 0.0f);
            const float2 g = (GLU && ok[k]) ? load2(xr + C) : make_float2(0.0f, 0.0f);
            gv[2 * k] = g.x;
            gv[2 * k + 1] = g.y;
        }
        float sg[2 * ITEMS];
        if constexpr (GLU) sigmoid_batch<RM, 2 * ITEMS>(gv, sg);
#pragma unroll
        for (uint32_t k = 0; k < ITEMS; k++) {
            const uint32_t i = first + k * DW_THREADS;
            float2 v = make_float2(0.0f, 0.0f);
            if (ok[k]) v = GLU ? make_float2(mul_r<RM>(a[k].x, sg[2 * k]), mul_r<RM>(a[k].y, sg[2 * k + 1])) : a[k];
            if (i < rows * PR) *reinterpret_cast<float2*>(tile + (i / PR) * DW_CH + 2 * (i % PR)) = v;
        }
    };
    if constexpr (KC > 0) {
        stage(std::integral_constant<uint32_t, ((DW_FRAMES + KC - 1) * PR + DW_THREADS - 1) / DW_THREADS>{},
              threadIdx.x);
    } else {
        // every thread runs the same passes (the batch's vote needs the warp)
        for (uint32_t first = threadIdx.x; first - threadIdx.x < rows * PR; first += DW_THREADS)
            stage(std::integral_constant<uint32_t, 1>{}, first);
    }
    for (uint32_t i = threadIdx.x; i < K * DW_CH; i += DW_THREADS) {
        const uint32_t jt = i / DW_CH, c = i % DW_CH;
        taps[i] = c0 + c < C ? __ldg(w + static_cast<size_t>(c0 + c) * K + jt) : 0.0f;
    }
    __syncthreads();

    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t cl = 2 * lane, ca = c0 + cl;
    const bool cin = ca < C;  // C even: both of the lane's channels, or neither
    const uint64_t b2 = cin ? pack2(__ldg(bias + ca), __ldg(bias + ca + 1)) : pack2(0.0f, 0.0f);
    float2 wr[KC > 0 ? KC : 1];
    if constexpr (KC > 0) {
#pragma unroll
        for (uint32_t jt = 0; jt < KC; jt++) wr[jt] = *reinterpret_cast<const float2*>(taps + jt * DW_CH + cl);
    }
    const uint32_t nb = C / QB;
    for (uint32_t f = warp; f < DW_FRAMES; f += DW_THREADS / 32) {
        const uint32_t t = t0 + f;
        if (t >= T) break;  // warp-uniform
        // the taps reading rows 0 .. T-1, in order: jt from hk - t (if
        // positive) up to T - 1 - t + hk (if below K)
        const uint32_t j0 = t >= hk ? 0u : hk - t;
        const uint64_t jend = static_cast<uint64_t>(T) - t + hk;
        const uint32_t j1 = jend < K ? static_cast<uint32_t>(jend) : K;
        uint64_t acc = pack2(0.0f, 0.0f);
        if constexpr (KC > 0) {
            if (j0 == 0 && j1 == KC) {  // an interior frame: every tap (warp-uniform)
#pragma unroll
                for (uint32_t jt = 0; jt < KC; jt++) {
                    const float2 xv = *reinterpret_cast<const float2*>(tile + (f + jt) * DW_CH + cl);
                    acc = fma2_r<RM>(pack2(wr[jt].x, wr[jt].y), pack2(xv.x, xv.y), acc);
                }
            } else {
#pragma unroll
                for (uint32_t jt = 0; jt < KC; jt++)
                    if (jt >= j0 && jt < j1) {
                        const float2 xv = *reinterpret_cast<const float2*>(tile + (f + jt) * DW_CH + cl);
                        acc = fma2_r<RM>(pack2(wr[jt].x, wr[jt].y), pack2(xv.x, xv.y), acc);
                    }
            }
        } else {
            for (uint32_t jt = j0; jt < j1; jt++) {
                const float2 xv = *reinterpret_cast<const float2*>(tile + (f + jt) * DW_CH + cl);
                const float2 wv = *reinterpret_cast<const float2*>(taps + jt * DW_CH + cl);
                acc = fma2_r<RM>(pack2(wv.x, wv.y), pack2(xv.x, xv.y), acc);
            }
        }
        float o[2];
        unpack2(add2_r<RM>(acc, b2), o[0], o[1]);  // v = acc + b
        silu_batch<RM, 2>(o);                        // v * sigmoid(v)
        const float o0 = o[0], o1 = o[1];
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
                pq = __byte_perm(quant1<RM>(o0, id), quant1<RM>(o1, id), 0x0040);  // the two low bytes
            }
            *reinterpret_cast<uint16_t*>(q + static_cast<size_t>(t) * C + ca) = static_cast<uint16_t>(pq);
            if (lane % (QB / 2) == 0) d[static_cast<size_t>(t) * nb + ca / QB] = scale;
        }
    }
}

// --------------------------------------------------------------- launches --

// Shared memory: w and b, padded, then two stages of two rows a warp. Up
// to four warps a CTA where two CTAs fit an SM; one warp up to the largest n.
constexpr size_t LN_SMEM_PAIR_CTA = 110 * 1024;
constexpr size_t LN_SMEM_MAX = 227 * 1024;

template <int RM, int QB>
cudaError_t ln_launch(int8_t* q, float* d, float* out, size_t os, const float* x, size_t xs, uint32_t T, uint32_t n,
                      const float* w, const float* b, float eps, int num_sms, cudaStream_t stream) {
    const size_t wb = 2 * static_cast<size_t>(ln_padded(n)) * sizeof(float);
    const size_t per_warp = 4 * static_cast<size_t>(ln_pitch(n)) * sizeof(float);
    size_t warps = LN_SMEM_PAIR_CTA > wb ? (LN_SMEM_PAIR_CTA - wb) / per_warp : 0;
    if (warps > 4) warps = 4;
    if (warps < 1) warps = 1;
    const size_t smem = wb + warps * per_warp;
    if (smem > LN_SMEM_MAX) return cudaErrorInvalidValue;  // n beyond the checked maximum
    auto kern = out ? (n == 16 * LN_NC ? layernorm_quantize<RM, QB, LN_NC, true> : layernorm_quantize<RM, QB, 0, true>)
                    : (n == 16 * LN_NC ? layernorm_quantize<RM, QB, LN_NC, false> : layernorm_quantize<RM, QB, 0, false>);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const size_t pairs = (static_cast<size_t>(T) + 1) / 2;
    size_t grid = (pairs + warps - 1) / warps;
    const size_t per_sm = (228 * 1024) / (smem + 1024);
    const size_t cap = static_cast<size_t>(num_sms) * (per_sm ? per_sm : 1);
    if (grid > cap) grid = cap;
    const bool xvec = reinterpret_cast<uintptr_t>(x) % 16 == 0 && xs % 4 == 0;
    const bool q16 = out ? reinterpret_cast<uintptr_t>(out) % 16 == 0 && os % 4 == 0
                         : reinterpret_cast<uintptr_t>(q) % 16 == 0;
    return launch_pdl(kern, dim3(static_cast<unsigned>(grid)), dim3(static_cast<unsigned>(32 * warps)), smem, stream,
                      q, d, out, os, x, xs, T, n, w, b, eps, xvec, q16);
}

template <int RM, int QB>
cudaError_t dw_launch(int8_t* q, float* d, float* out, size_t os, const float* x, size_t xs, uint32_t T, uint32_t C,
                      const float* w, const float* bias, uint32_t K, bool glu, cudaStream_t stream) {
    const size_t smem = (static_cast<size_t>(DW_FRAMES + K - 1) + K) * DW_CH * sizeof(float);
    const dim3 grid((T + DW_FRAMES - 1) / DW_FRAMES, (C + DW_CH - 1) / DW_CH);
    const bool xv2 = reinterpret_cast<uintptr_t>(x) % 8 == 0 && xs % 2 == 0;
    if (K == 9) {
        if (glu)
            return launch_pdl(dwconv_quantize<RM, QB, true, 9>, grid, dim3(DW_THREADS), smem, stream, q, d, out, os, x,
                              xs, T, C, w, bias, K, xv2);
        return launch_pdl(dwconv_quantize<RM, QB, false, 9>, grid, dim3(DW_THREADS), smem, stream, q, d, out, os, x,
                          xs, T, C, w, bias, K, xv2);
    }
    if (glu)
        return launch_pdl(dwconv_quantize<RM, QB, true, 0>, grid, dim3(DW_THREADS), smem, stream, q, d, out, os, x, xs,
                          T, C, w, bias, K, xv2);
    return launch_pdl(dwconv_quantize<RM, QB, false, 0>, grid, dim3(DW_THREADS), smem, stream, q, d, out, os, x, xs, T,
                      C, w, bias, K, xv2);
}

template <int RM>
cudaError_t ln_rm(int8_t* q, float* d, const float* x, size_t xs, uint32_t T, uint32_t n, uint32_t qb,
                  const float* w, const float* b, float eps, int num_sms, cudaStream_t stream) {
    if (qb == 32) return ln_launch<RM, 32>(q, d, nullptr, 0, x, xs, T, n, w, b, eps, num_sms, stream);
    if (qb == 64) return ln_launch<RM, 64>(q, d, nullptr, 0, x, xs, T, n, w, b, eps, num_sms, stream);
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

cudaError_t launch_layernorm(float* out, size_t os, const float* x, size_t xs, uint32_t T, uint32_t n, const float* w,
                             const float* b, float eps, int rmode, int num_sms, cudaStream_t stream) {
    switch (rmode) {
    case 1: return ln_launch<1, 32>(nullptr, nullptr, out, os, x, xs, T, n, w, b, eps, num_sms, stream);
    case 2: return ln_launch<2, 32>(nullptr, nullptr, out, os, x, xs, T, n, w, b, eps, num_sms, stream);
    case 3: return ln_launch<3, 32>(nullptr, nullptr, out, os, x, xs, T, n, w, b, eps, num_sms, stream);
    default: return ln_launch<0, 32>(nullptr, nullptr, out, os, x, xs, T, n, w, b, eps, num_sms, stream);
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
