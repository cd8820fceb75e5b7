// The attention's float work on the device, sm_100a: the reference's
// k_gemm_f32 (backend/ref/kernels.c:90-105), k_softmax (:134-147), and
// att_item (core/encoder.c:280-326) as one kernel over every head and block
// of queries of a batch of segments.
//
// Bit for bit the reference's: every product is its chain of fused
// multiply-adds in its order (k ascending, from +0), every other operation
// its operation, rounded once in the mode RM. A tensor core does not compute
// an IEEE chain of fused multiply-adds, so these run on the CUDA cores' FP32
// pipe (128 lane-operations a cycle per SM), which bounds them.

#include "pkb_device.cuh"
#include "pkb_internal.h"
#include "pkb_vmath.cuh"

namespace pkb {

namespace {

// -------------------------------------------------------------- gemm_f32 --

constexpr int GF_ROWS = 64;   // output rows a CTA: four 16-row panels
constexpr int GF_COLS = 32;   // columns (t) a CTA
constexpr int GF_KC = 32;     // k a staged chunk
constexpr int GF_THREADS = 256;
constexpr int GF_XS = GF_COLS + 2;  // the staged columns' k-major row stride (pairs stay 8-byte aligned)

// out[t os + r] = relu?(chain_k fma(w(r, k), x[t xs + k]) + (bias ? bias[t bs + r] : 0)),
// w(r, k) at w[(r/16) ld 16 + 16 k + r%16]. Thread (rq, cp) holds rows
// 4 rq .. 4 rq + 3 of the CTA's 64 (inside one panel) for columns 2 cp and
// 2 cp + 1: eight chains, each over k in order.
template <int RM>
__global__ void __launch_bounds__(GF_THREADS)
    gemm_f32_kernel(float* out, unsigned long long os, const float* w, uint32_t ld, uint32_t rows, uint32_t n,
                    const float* x, unsigned long long xs, uint32_t T, const float* bias, unsigned long long bs,
                    int relu) {
    __shared__ __align__(16) float sw[4][GF_KC][16];
    __shared__ __align__(16) float sx[GF_KC][GF_XS];
    const uint32_t tid = threadIdx.x;
    const uint32_t r0 = blockIdx.x * GF_ROWS, t0 = blockIdx.y * GF_COLS;
    const uint32_t rq = tid % 16, cp = tid / 16;
    const uint32_t pnl = rq / 4, pr = (rq % 4) * 4;
    float acc[2][4];
#pragma unroll
    for (int c = 0; c < 2; c++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[c][j] = 0.0f;
    for (uint32_t k0 = 0; k0 < n; k0 += GF_KC) {
        const uint32_t kc = min(static_cast<uint32_t>(GF_KC), n - k0);
        __syncthreads();  // the previous chunk is read
        for (uint32_t e = tid; e < 4 * GF_KC * 16; e += GF_THREADS) {
            const uint32_t p = e / (GF_KC * 16), kk = (e / 16) % GF_KC, r = e % 16;
            float v = 0.0f;
            if (r0 + 16 * p < rows && kk < kc)
                v = w[(static_cast<size_t>(r0 / 16 + p) * ld + k0 + kk) * 16 + r];
            sw[p][kk][r] = v;
        }
        for (uint32_t e = tid; e < GF_COLS * GF_KC; e += GF_THREADS) {
            const uint32_t c = e / GF_KC, kk = e % GF_KC;
            float v = 0.0f;
            if (t0 + c < T && kk < kc) v = x[static_cast<size_t>(t0 + c) * xs + k0 + kk];
            sx[kk][c] = v;
        }
        __syncthreads();
        for (uint32_t kk = 0; kk < kc; kk++) {
            const float4 wv = *reinterpret_cast<const float4*>(&sw[pnl][kk][pr]);
            const float2 xv = *reinterpret_cast<const float2*>(&sx[kk][2 * cp]);
            acc[0][0] = fma_r<RM>(wv.x, xv.x, acc[0][0]);
            acc[0][1] = fma_r<RM>(wv.y, xv.x, acc[0][1]);
            acc[0][2] = fma_r<RM>(wv.z, xv.x, acc[0][2]);
            acc[0][3] = fma_r<RM>(wv.w, xv.x, acc[0][3]);
            acc[1][0] = fma_r<RM>(wv.x, xv.y, acc[1][0]);
            acc[1][1] = fma_r<RM>(wv.y, xv.y, acc[1][1]);
            acc[1][2] = fma_r<RM>(wv.z, xv.y, acc[1][2]);
            acc[1][3] = fma_r<RM>(wv.w, xv.y, acc[1][3]);
        }
    }
#pragma unroll
    for (int c = 0; c < 2; c++) {
        const uint32_t t = t0 + 2 * cp + c;
        if (t >= T) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t r = r0 + 4 * rq + j;
            if (r >= rows) continue;
            // one thread reads bias[t bs + r] and then writes out[t os + r],
            // so out may be the bias itself (os == bs)
            float v = add_r<RM>(acc[c][j], bias ? bias[static_cast<size_t>(t) * bs + r] : 0.0f);
            if (relu) v = v > 0.0f ? v : 0.0f;
            out[static_cast<size_t>(t) * os + r] = v;
        }
    }
}

// --------------------------------------------------------------- softmax --

// k_softmax on one row of n in memory (global or shared; element i at
// x[i xs]) by one warp, lane i taking elements i, i + 32, ...: y = x * scale and its maximum (fmaxf
// passes a NaN over; the sign of a zero maximum changes no e below, as
// y - (+-0) is y for y != 0 and pk_expf(+-0) is 1), e = pk_expf(y - m), the
// sum of the e in the reference's 16 lanes (element i into lane i % 16, in
// order: lane l < 16 adds its own then lane l + 16's element of each 32)
// folded 8, 4, 2, 1, then e * (1 / sum).
template <int RM>
__device__ __forceinline__ void softmax_row(float* x, uint32_t xs, uint32_t n, float scale, uint32_t lane) {
    float m = -INFINITY;
    for (uint32_t i = lane; i < n; i += 32) {
        const float y = mul_r<RM>(x[i * xs], scale);
        x[i * xs] = y;
        m = fmaxf(m, y);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float acc = 0.0f;
    for (uint32_t base = 0; base < n; base += 32) {
        const uint32_t i = base + lane;
        float e = 0.0f;
        if (i < n) {
            e = pk_exp<RM>(sub_r<RM>(x[i * xs], m));
            x[i * xs] = e;
        }
        const float hi = __shfl_down_sync(0xffffffffu, e, 16);
        if (lane < 16) {
            if (i < n) acc = add_r<RM>(acc, e);
            if (i + 16 < n) acc = add_r<RM>(acc, hi);
        }
    }
#pragma unroll
    for (int h = 8; h >= 1; h >>= 1) {
        const float o = __shfl_down_sync(0xffffffffu, acc, h);
        if (lane < static_cast<uint32_t>(h)) acc = add_r<RM>(acc, o);
    }
    const float inv = rcp_r<RM>(__shfl_sync(0xffffffffu, acc, 0));
    for (uint32_t i = lane; i < n; i += 32) x[i * xs] = mul_r<RM>(x[i * xs], inv);
}

constexpr int SM_THREADS = 256;

// T rows at stride xs, a warp a row
template <int RM>
__global__ void __launch_bounds__(SM_THREADS)
    softmax_kernel(float* x, unsigned long long xs, uint32_t T, uint32_t n, float scale) {
    const uint32_t lane = threadIdx.x % 32;
    for (uint32_t t = blockIdx.x * (SM_THREADS / 32) + threadIdx.x / 32; t < T; t += gridDim.x * (SM_THREADS / 32))
        softmax_row<RM>(x + static_cast<size_t>(t) * xs, 1, n, scale, lane);
}

// ------------------------------------------------------------- attention --

constexpr int AQ = 32;           // queries a CTA (two of the reference's PK_ATT_BLOCK, core/asr.h:16)
constexpr int A_THREADS = 256;
constexpr int AKU = 128;         // keys (or positions) a unit of K (P)
constexpr int AQS = AQ + 4;      // row stride of the transposed queries and scores

// The staging: units of K and P carry DH dimensions of 128 keys, units of
// V DH keys of up to 128 dimensions, through NBUF buffers (the copies of
// NBUF - 1 units in flight while the CTA computes on one). Measured on B200
// over the benchmark's batch: DH 32 with 2 buffers 871 us, DH 16 with 2
// 1004 us, DH 16 with 3 994 us (more units, more barriers).
#ifndef PKB_ATT_DH
#define PKB_ATT_DH 32
#endif
#ifndef PKB_ATT_NBUF
#define PKB_ATT_NBUF 2
#endif
constexpr int ADH = PKB_ATT_DH, ANB = PKB_ATT_NBUF;

// the unit depth a head of dk takes: ADH where it divides dk, else 16
__host__ __device__ __forceinline__ uint32_t att_dh(uint32_t dk) { return dk % ADH ? 16 : ADH; }

// floats of one staging buffer: the larger of a K/P unit and a V unit in
// either layout, with the padding that keeps a quarter-warp's 16-byte loads
// on distinct bank groups
__host__ __device__ __forceinline__ uint32_t att_buf(uint32_t dk, uint32_t dh) {
    const uint32_t dv = dk < 128 ? dk : 128, av = dh;
    const uint32_t kp_rows = AKU * (dh + 4), kp_pan = (AKU / 16) * (16 * dh + 16);
    const uint32_t v_rows = av * (dv + 4), v_pan = (dv / 16) * (16 * av + 16);
    uint32_t m = kp_rows > kp_pan ? kp_rows : kp_pan;
    m = m > v_rows ? m : v_rows;
    return m > v_pan ? m : v_pan;
}

// One CTA: head h, queries i0 .. i0 + nq - 1 (nq <= 32) of one segment of T
// frames. Shared memory:
//
//   QT     the queries plus a position bias, transposed: dimension d of
//          query i at QT[d AQS + i] (first q + bias_u; q + bias_v once the
//          scores are done)
//   ST[2]  two staging buffers that the K, P and V units go through in
//          turn, the next unit's copies (cp.async) in flight while the CTA
//          computes on the current one
//   SC     the scores, then the weights, transposed: key k of query i at
//          SC[k AQS + i], SP rows
//
// The units, in order: K in chunks of 128 keys, each in pieces of dh
// dimensions (a score's chain runs on across the pieces, d ascending); P the
// same over the block's window of positions; V in chunks of 32 keys, in
// passes of up to 128 dimensions. Rows layout: a K/P unit is row-major (key
// j, dimension d at j (dh + 4) + d), a V unit too (k (dv + 4) + d). Panels
// layout: the reference's order, padded (16-key groups of dh x 16, 16 dh +
// 16 apart; 16-dimension panels of 32 x 16, 528 apart).
//
// Scores and position products: lane (qq, ko) of warp w takes queries
// 4 qq .. 4 qq + 3 and 4 keys of the warp's 16 (rows: 16 w + ko + 4 e;
// panels: 16 w + 4 ko + e), 16 chains over d, 4 dimensions a step: 4
// 16-byte loads of queries (8 distinct in a warp: one wavefront), 4 of K or
// P (4 distinct on distinct bank groups: one wavefront), 64 FMAs. A score is
// stored as 4 queries' 16 bytes; each position product is added to the
// score it belongs to as soon as its chain is done (the pairs (query i,
// position T-1-i+k) are one to one with the scores (i, k)). The weighted
// values: lane (vq, vo) of warp w takes queries 4 vq .. 4 vq + 3 and
// dimensions 4 (4 w + vo) .. + 3 of the pass, 16 chains over k, a key a
// step: the 4 queries' weights in one 16-byte load, 4 values in another.
template <int RM, bool PANELS, int DH, int NBUF>
__global__ void __launch_bounds__(A_THREADS, 2) attention_kernel(const __grid_constant__ AttArgs a) {
    extern __shared__ __align__(16) float sm[];
    __shared__ uint32_t s_seg;
    const uint32_t tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
    if (tid == 0) {
        // the segment whose items hold this CTA's: the last with item0 <= blockIdx.x
        uint32_t lo = 0, hi = a.nseg - 1;
        while (lo < hi) {
            const uint32_t mid = (lo + hi + 1) / 2;
            if (a.seg[mid].item0 <= blockIdx.x)
                lo = mid;
            else
                hi = mid - 1;
        }
        s_seg = lo;
    }
    __syncthreads();
    const AttSeg sg = a.seg[s_seg];
    constexpr uint32_t dh = DH, AVU = DH;
    const uint32_t T = sg.T, dk = a.dk;
    const uint32_t nh = dk / dh, BUF = att_buf(dk, dh);
    const uint32_t nqb = (T + AQ - 1) / AQ, local = blockIdx.x - sg.item0;
    const uint32_t h = local / nqb, i0 = (local % nqb) * AQ;
    const uint32_t nq = min(static_cast<uint32_t>(AQ), T - i0), i1 = i0 + nq;
    const uint32_t R = 2 * T - 1;
    // the position window: rows T - 1 - i + k for the block's queries i and
    // keys k, from a panel boundary
    const uint32_t w0 = (T - i1) & ~15u, W = ((2 * T - 1 - i0 - w0) + 15) & ~15u;
    float* QT = sm;
    float* ST = QT + dk * AQS;
    float* SC = ST + NBUF * BUF;

    const uint32_t Tp = (T + 15) & ~15u, Pp = ((R + 15) & ~15u) + 16;
    const float* kh = PANELS ? a.k + static_cast<size_t>(h) * Tp * dk : a.k + static_cast<size_t>(sg.f) * a.ks + h * dk;
    const float* ph = PANELS ? a.p + static_cast<size_t>(h) * Pp * dk : a.p + static_cast<size_t>(sg.p) * a.ps + h * dk;
    const float* vh = PANELS ? a.v + static_cast<size_t>(h) * (dk / 16) * T * 16
                             : a.v + static_cast<size_t>(sg.f) * a.vs + h * dk;

    const uint32_t nkc = (T + AKU - 1) / AKU, npc = (W + AKU - 1) / AKU, nvc = (T + AVU - 1) / AVU;
    const uint32_t npass = (dk + 127) / 128;
    const uint32_t nK = nkc * nh, nP = npc * nh, U = nK + nP + npass * nvc;

    // issues unit u's copies into buffer b; rows past the data are skipped
    // (their results are never read)
    auto issue = [&](uint32_t u, float* b) {
        if (u < nK + nP) {
            const bool isk = u < nK;
            const uint32_t cu = isk ? u : u - nK, c = cu / nh, d0 = (cu % nh) * dh;
            const uint32_t j0 = isk ? c * AKU : w0 + c * AKU;
            const float* src = isk ? kh : ph;
            if constexpr (PANELS) {
                // 16-key group g: dh x 16 floats at ((j0/16 + g) dk + d0) 16
                const uint32_t valid = isk ? Tp : Pp, n4 = dh * 4;
                for (uint32_t e = tid; e < (AKU / 16) * n4; e += A_THREADS) {
                    const uint32_t g = e / n4, o = e % n4;
                    if (j0 + 16 * g < valid)
                        cp_async16(b + g * (16 * dh + 16) + 4 * o,
                                   src + (static_cast<size_t>(j0 / 16 + g) * dk + d0) * 16 + 4 * o);
                }
            } else {
                const unsigned long long rs = isk ? a.ks : a.ps;
                const uint32_t valid = isk ? T : R, n4 = dh / 4;
                for (uint32_t e = tid; e < AKU * n4; e += A_THREADS) {
                    const uint32_t jj = e / n4, o = e % n4;
                    if (j0 + jj < valid)
                        cp_async16(b + jj * (dh + 4) + 4 * o, src + static_cast<size_t>(j0 + jj) * rs + d0 + 4 * o);
                }
            }
        } else {
            const uint32_t vu = u - nK - nP, pass = vu / nvc, c0 = (vu % nvc) * AVU;
            const uint32_t e0 = pass * 128, dv = min(128u, dk - e0);
            if constexpr (PANELS) {
                // 16-dimension panel dp: 32 x 16 floats at ((e0/16 + dp) T + c0) 16
                const uint32_t n4 = AVU * 4;
                for (uint32_t e = tid; e < (dv / 16) * n4; e += A_THREADS) {
                    const uint32_t dp = e / n4, o = e % n4;
                    if (c0 + o / 4 < T)
                        cp_async16(b + dp * (16 * AVU + 16) + 4 * o,
                                   vh + (static_cast<size_t>(e0 / 16 + dp) * T + c0) * 16 + 4 * o);
                }
            } else {
                const uint32_t n4 = dv / 4;
                for (uint32_t e = tid; e < AVU * n4; e += A_THREADS) {
                    const uint32_t kk = e / n4, o = e % n4;
                    if (c0 + kk < T)
                        cp_async16(b + kk * (dv + 4) + 4 * o, vh + static_cast<size_t>(c0 + kk) * a.vs + e0 + 4 * o);
                }
            }
        }
        cp_async_commit();
    };

    // the block's queries with a position bias, transposed (core/encoder.c:
    // 302-309); eight loads of each in flight a thread
    auto load_queries = [&](const float* bias) {
        for (uint32_t e0 = tid; e0 < AQ * dk; e0 += 8 * A_THREADS) {
            float qv[8], bv[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const uint32_t e = e0 + j * A_THREADS, i = e / dk, d = e % dk;
                qv[j] = bv[j] = 0.0f;
                if (e < AQ * dk && i < nq) {
                    qv[j] = a.q[static_cast<size_t>(sg.f + i0 + i) * a.qs + h * dk + d];
                    bv[j] = bias[h * dk + d];
                }
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const uint32_t e = e0 + j * A_THREADS, i = e / dk, d = e % dk;
                if (e < AQ * dk) QT[d * AQS + i] = i < nq ? add_r<RM>(qv[j], bv[j]) : 0.0f;
            }
        }
    };

#pragma unroll
    for (int j = 0; j < NBUF - 1; j++)
        if (j < static_cast<int>(U)) issue(j, ST + j * BUF);
    load_queries(a.bu);

    const uint32_t qq = lane % 8, ko = lane / 8;  // query quad, key (or dimension) lane group
    float acc[4][4];
    const float scale = div_r<RM>(1.0f, sqrt_r<RM>(static_cast<float>(dk)));

    for (uint32_t u = 0; u < U; u++) {
        float* b = ST + (u % NBUF) * BUF;
        // unit u + NBUF - 1 into the buffer unit u - 1 left (free since the
        // barrier ending unit u - 1); an empty group past the end keeps the
        // count of groups in flight the same
        if (u + NBUF - 1 < U)
            issue(u + NBUF - 1, ST + ((u + NBUF - 1) % NBUF) * BUF);
        else
            cp_async_commit();
        cp_async_wait<NBUF - 1>();
        if (u == nK) {
            // the scores are done with q + bias_u (the barrier ending unit
            // nK - 1): q + bias_v in its place
            load_queries(a.bv);
        }
        __syncthreads();  // unit u has landed for every thread (and the queries are in)
        if (u < nK + nP) {
            const bool isk = u < nK;
            const uint32_t cu = isk ? u : u - nK, c = cu / nh, part = cu % nh, d0 = part * dh;
            if (part == 0) {
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int e = 0; e < 4; e++) acc[i][e] = 0.0f;
            }
            // a warp whose 16 keys (positions) all lie past the data skips the unit
            const bool idle = c * AKU + 16 * warp >= (isk ? T : W);
            if (!idle) {
                const float* qb = QT + d0 * AQS + 4 * qq;
#pragma unroll
                for (uint32_t dd = 0; dd < dh; dd += 4) {
                    float4 q[4];
#pragma unroll
                    for (int t = 0; t < 4; t++) q[t] = *reinterpret_cast<const float4*>(qb + (dd + t) * AQS);
                    float4 k[4];
                    if constexpr (PANELS) {
                        // keys 16 w + 4 ko .. + 3 at dimension dd + t
#pragma unroll
                        for (int t = 0; t < 4; t++)
                            k[t] = *reinterpret_cast<const float4*>(b + warp * (16 * dh + 16) + (dd + t) * 16 + 4 * ko);
                    } else {
                        // key 16 w + ko + 4 e, dimensions dd .. dd + 3
#pragma unroll
                        for (int e = 0; e < 4; e++)
                            k[e] = *reinterpret_cast<const float4*>(b + (16 * warp + ko + 4 * e) * (dh + 4) + dd);
                    }
#pragma unroll
                    for (int t = 0; t < 4; t++) {
                        const float qv[4] = {q[t].x, q[t].y, q[t].z, q[t].w};
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            float kv;
                            if constexpr (PANELS)
                                kv = e == 0 ? k[t].x : e == 1 ? k[t].y : e == 2 ? k[t].z : k[t].w;
                            else
                                kv = t == 0 ? k[e].x : t == 1 ? k[e].y : t == 2 ? k[e].z : k[e].w;
#pragma unroll
                            for (int i = 0; i < 4; i++) acc[i][e] = fma_r<RM>(kv, qv[i], acc[i][e]);
                        }
                    }
                }
            }
            if (part == nh - 1 && !idle) {
                // the chains are done: + 0 as gemm_f32 adds its absent bias;
                // a score is stored, a position product added to its score
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const uint32_t jl = c * AKU + 16 * warp + (PANELS ? 4 * ko + e : ko + 4 * e);
                    if (isk) {
                        if (jl < T) {
                            float4 v;
                            v.x = add_r<RM>(acc[0][e], 0.0f);
                            v.y = add_r<RM>(acc[1][e], 0.0f);
                            v.z = add_r<RM>(acc[2][e], 0.0f);
                            v.w = add_r<RM>(acc[3][e], 0.0f);
                            *reinterpret_cast<float4*>(SC + jl * AQS + 4 * qq) = v;
                        }
                    } else if (jl < W) {
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            // position row w0 + jl is the score (qi, k), k = w0 + jl - (T - 1 - (i0 + qi))
                            const uint32_t qi = 4 * qq + i;
                            const int k = static_cast<int>(w0 + jl) - static_cast<int>(T - 1 - (i0 + qi));
                            if (qi < nq && k >= 0 && k < static_cast<int>(T))
                                SC[k * AQS + qi] = add_r<RM>(SC[k * AQS + qi], add_r<RM>(acc[i][e], 0.0f));
                        }
                    }
                }
            }
        } else {
            const uint32_t vu = u - nK - nP, pass = vu / nvc, cc = vu % nvc, c0 = cc * AVU;
            const uint32_t e0 = pass * 128, dv = min(128u, dk - e0), kc = min(static_cast<uint32_t>(AVU), T - c0);
            if (vu == 0) {
                // every score has its position: each query's softmax
                // (core/encoder.c:315-321), while the first V units land
                for (uint32_t i = warp; i < nq; i += A_THREADS / 32) softmax_row<RM>(SC + i, AQS, T, scale, lane);
                __syncthreads();
            }
            if (cc == 0) {
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int e = 0; e < 4; e++) acc[i][e] = 0.0f;
            }
            const uint32_t vo = ko + 4 * warp;  // dimensions 4 vo .. 4 vo + 3 of the pass
            if (vo < dv / 4) {
                const float* wr = SC + c0 * AQS + 4 * qq;
                const float* vb = PANELS ? b + (vo / 4) * (16 * AVU + 16) + 4 * (vo % 4) : b + 4 * vo;
                const uint32_t vstep = PANELS ? 16 : dv + 4;
                // a key: the 4 queries' weights, 4 values, 16 FMAs
                auto one = [&](uint32_t kk) {
                    const float4 p = *reinterpret_cast<const float4*>(wr + kk * AQS);
                    const float4 v = *reinterpret_cast<const float4*>(vb + kk * vstep);
                    const float pv[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        acc[i][0] = fma_r<RM>(v.x, pv[i], acc[i][0]);
                        acc[i][1] = fma_r<RM>(v.y, pv[i], acc[i][1]);
                        acc[i][2] = fma_r<RM>(v.z, pv[i], acc[i][2]);
                        acc[i][3] = fma_r<RM>(v.w, pv[i], acc[i][3]);
                    }
                };
                if (kc == AVU) {
#pragma unroll
                    for (uint32_t kk = 0; kk < AVU; kk++) one(kk);
                } else {
                    for (uint32_t kk = 0; kk < kc; kk++) one(kk);
                }
                if (cc == nvc - 1) {
                    // o = V^T s + 0 (core/encoder.c:323-324), this pass's dimensions
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const uint32_t qi = 4 * qq + i;
                        if (qi < nq) {
                            float* orow = a.o + static_cast<size_t>(sg.f + i0 + qi) * a.os + h * dk + e0 + 4 * vo;
#pragma unroll
                            for (int e = 0; e < 4; e++) orow[e] = add_r<RM>(acc[i][e], 0.0f);
                        }
                    }
                }
            }
        }
        __syncthreads();  // buffer u % NBUF is free for unit u + NBUF
    }
}

template <int RM>
cudaError_t gemm_f32_rm(float* out, size_t os, const float* w, uint32_t ld, uint32_t rows, uint32_t n, const float* x,
                        size_t xs, uint32_t T, const float* bias, size_t bs, int relu, cudaStream_t stream) {
    const dim3 grid((rows + GF_ROWS - 1) / GF_ROWS, (T + GF_COLS - 1) / GF_COLS);
    gemm_f32_kernel<RM><<<grid, GF_THREADS, 0, stream>>>(out, os, w, ld, rows, n, x, xs, T, bias, bs, relu);
    return cudaGetLastError();
}

template <int RM>
cudaError_t softmax_rm(float* x, size_t xs, uint32_t T, uint32_t n, float scale, int num_sms, cudaStream_t stream) {
    const uint32_t per = SM_THREADS / 32;
    const uint32_t blocks = min((T + per - 1) / per, static_cast<uint32_t>(num_sms) * 8u);
    softmax_kernel<RM><<<blocks, SM_THREADS, 0, stream>>>(x, xs, T, n, scale);
    return cudaGetLastError();
}

template <int RM, bool PANELS>
cudaError_t attention_rm(const AttArgs& a, size_t smem, cudaStream_t stream) {
    if (att_dh(a.dk) == ADH)
        attention_kernel<RM, PANELS, ADH, ANB><<<a.items, A_THREADS, smem, stream>>>(a);
    else
        attention_kernel<RM, PANELS, 16, ANB><<<a.items, A_THREADS, smem, stream>>>(a);
    return cudaGetLastError();
}

// the dynamic shared memory every attention instance may take: the
// device's opt-in limit less the kernel's own static shared memory
size_t g_att_dyn_max = 0;

template <typename Kern>
cudaError_t allow_smem(Kern kern, int optin) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return e;
    const int dyn = optin - static_cast<int>(fa.sharedSizeBytes);
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
    if (e == cudaSuccess && (g_att_dyn_max == 0 || static_cast<size_t>(dyn) < g_att_dyn_max))
        g_att_dyn_max = static_cast<size_t>(dyn);
    return e;
}

template <int RM>
cudaError_t prepare_attention_rm(int optin) {
    cudaError_t e = allow_smem(attention_kernel<RM, true, ADH, ANB>, optin);
    if (e == cudaSuccess) e = allow_smem(attention_kernel<RM, false, ADH, ANB>, optin);
    if (ADH != 16 && e == cudaSuccess) e = allow_smem(attention_kernel<RM, true, 16, ANB>, optin);
    if (ADH != 16 && e == cudaSuccess) e = allow_smem(attention_kernel<RM, false, 16, ANB>, optin);
    return e;
}

}  // namespace

cudaError_t launch_gemm_f32(float* out, size_t os, const float* w, uint32_t ld, uint32_t rows, uint32_t n,
                            const float* x, size_t xs, uint32_t T, const float* bias, size_t bs, int relu, int rmode,
                            cudaStream_t stream) {
    switch (rmode) {
    case 1: return gemm_f32_rm<1>(out, os, w, ld, rows, n, x, xs, T, bias, bs, relu, stream);
    case 2: return gemm_f32_rm<2>(out, os, w, ld, rows, n, x, xs, T, bias, bs, relu, stream);
    case 3: return gemm_f32_rm<3>(out, os, w, ld, rows, n, x, xs, T, bias, bs, relu, stream);
    default: return gemm_f32_rm<0>(out, os, w, ld, rows, n, x, xs, T, bias, bs, relu, stream);
    }
}

cudaError_t launch_softmax(float* x, size_t xs, uint32_t T, uint32_t n, float scale, int rmode, int num_sms,
                           cudaStream_t stream) {
    switch (rmode) {
    case 1: return softmax_rm<1>(x, xs, T, n, scale, num_sms, stream);
    case 2: return softmax_rm<2>(x, xs, T, n, scale, num_sms, stream);
    case 3: return softmax_rm<3>(x, xs, T, n, scale, num_sms, stream);
    default: return softmax_rm<0>(x, xs, T, n, scale, num_sms, stream);
    }
}

size_t attention_smem(uint32_t dk, uint32_t sp) {
    return (static_cast<size_t>(dk) * AQS + ANB * static_cast<size_t>(att_buf(dk, att_dh(dk))) +
            static_cast<size_t>(sp) * AQS) *
           sizeof(float);
}

uint32_t attention_block() { return AQ; }

cudaError_t prepare_attention() {
    int dev = 0, optin = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e == cudaSuccess) e = prepare_attention_rm<0>(optin);
    if (e == cudaSuccess) e = prepare_attention_rm<1>(optin);
    if (e == cudaSuccess) e = prepare_attention_rm<2>(optin);
    if (e == cudaSuccess) e = prepare_attention_rm<3>(optin);
    return e;
}

size_t attention_smem_max() { return g_att_dyn_max; }

cudaError_t launch_attention(const AttArgs& a, bool panels, int rmode, cudaStream_t stream) {
    const size_t smem = attention_smem(a.dk, a.sp);
    if (panels) {
        switch (rmode) {
        case 1: return attention_rm<1, true>(a, smem, stream);
        case 2: return attention_rm<2, true>(a, smem, stream);
        case 3: return attention_rm<3, true>(a, smem, stream);
        default: return attention_rm<0, true>(a, smem, stream);
        }
    }
    switch (rmode) {
    case 1: return attention_rm<1, false>(a, smem, stream);
    case 2: return attention_rm<2, false>(a, smem, stream);
    case 3: return attention_rm<3, false>(a, smem, stream);
    default: return attention_rm<0, false>(a, smem, stream);
    }
}

}  // namespace pkb
