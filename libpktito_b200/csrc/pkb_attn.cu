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

// k_softmax on one row of n in memory (global or shared) by one warp, lane
// i taking elements i, i + 32, ...: y = x * scale and its maximum (fmaxf
// passes a NaN over; the sign of a zero maximum changes no e below, as
// y - (+-0) is y for y != 0 and pk_expf(+-0) is 1), e = pk_expf(y - m), the
// sum of the e in the reference's 16 lanes (element i into lane i % 16, in
// order: lane l < 16 adds its own then lane l + 16's element of each 32)
// folded 8, 4, 2, 1, then e * (1 / sum).
template <int RM>
__device__ __forceinline__ void softmax_row(float* x, uint32_t n, float scale, uint32_t lane) {
    float m = -INFINITY;
    for (uint32_t i = lane; i < n; i += 32) {
        const float y = mul_r<RM>(x[i], scale);
        x[i] = y;
        m = fmaxf(m, y);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float acc = 0.0f;
    for (uint32_t base = 0; base < n; base += 32) {
        const uint32_t i = base + lane;
        float e = 0.0f;
        if (i < n) {
            e = pk_exp<RM>(sub_r<RM>(x[i], m));
            x[i] = e;
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
    for (uint32_t i = lane; i < n; i += 32) x[i] = mul_r<RM>(x[i], inv);
}

constexpr int SM_THREADS = 256;

// T rows at stride xs, a warp a row
template <int RM>
__global__ void __launch_bounds__(SM_THREADS)
    softmax_kernel(float* x, unsigned long long xs, uint32_t T, uint32_t n, float scale) {
    const uint32_t lane = threadIdx.x % 32;
    for (uint32_t t = blockIdx.x * (SM_THREADS / 32) + threadIdx.x / 32; t < T; t += gridDim.x * (SM_THREADS / 32))
        softmax_row<RM>(x + static_cast<size_t>(t) * xs, n, scale, lane);
}

// ------------------------------------------------------------- attention --

constexpr int AQ = 16;           // queries a CTA: PK_ATT_BLOCK (core/asr.h:16)
constexpr int A_THREADS = 128;
constexpr int ACH = 64;          // keys, positions or values a staged chunk

// One CTA: head h, queries i0 .. i0 + nq - 1 of one segment of T frames.
//
//   qu, qv   the queries plus each position bias, AQ rows of dk (+4)
//   ST       a chunk of 64 rows of K, P or V (row j, dimension d at
//            ST[j (dk + 4) + d]: 16-byte rows offset by one bank group, so
//            the 8 lanes of a quarter-warp reading 8 rows hit 8 groups)
//   S        the scores, then the weights: AQ rows of SP >= T
//   B        the position products over the block's window: AQ rows of BP
//
// Scores and position products: thread (kq, qp) takes queries 2 qp, 2 qp + 1
// and rows kq, kq + 16, kq + 32, kq + 48 of each chunk, 8 chains over d,
// 4 dimensions a step (two 16-byte loads of queries, four of rows, 32
// FMAs). The weighted values: tile u = (query quad, dimension quad), 4 x 4
// chains over k, 4 keys a step (four 16-byte loads of weights, four of
// values, 64 FMAs).
template <int RM, bool PANELS>
__global__ void __launch_bounds__(A_THREADS) attention_kernel(const __grid_constant__ AttArgs a) {
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
    const uint32_t T = sg.T, dk = a.dk, DS = dk + 4;
    const uint32_t nqb = (T + AQ - 1) / AQ, local = blockIdx.x - sg.item0;
    const uint32_t h = local / nqb, i0 = (local % nqb) * AQ;
    const uint32_t nq = min(static_cast<uint32_t>(AQ), T - i0), i1 = i0 + nq;
    const uint32_t R = 2 * T - 1;
    // the position window: rows T - 1 - i + k for the block's queries i and
    // keys k, from a panel boundary (as the reference takes it; a value
    // does not depend on it)
    const uint32_t w0 = (T - i1) & ~15u, W = ((2 * T - 1 - i0 - w0) + 15) & ~15u;
    float* qu = sm;
    float* qv = qu + AQ * DS;
    float* ST = qv + AQ * DS;
    float* S = ST + ACH * DS;
    float* B = S + AQ * a.sp;
    const uint32_t SP = a.sp, BP = a.bp;

    // K, P and V of this segment and head
    const uint32_t Tp = (T + 15) & ~15u, Pp = ((R + 15) & ~15u) + 16;
    const float* kh = PANELS ? a.k + static_cast<size_t>(h) * Tp * dk : a.k + static_cast<size_t>(sg.f) * a.ks + h * dk;
    const float* ph = PANELS ? a.p + static_cast<size_t>(h) * Pp * dk : a.p + static_cast<size_t>(sg.p) * a.ps + h * dk;
    const float* vh = PANELS ? a.v + static_cast<size_t>(h) * (dk / 16) * T * 16
                             : a.v + static_cast<size_t>(sg.f) * a.vs + h * dk;

    // the block's queries with each position bias (core/encoder.c:302-309)
    for (uint32_t e = tid; e < AQ * dk; e += A_THREADS) {
        const uint32_t i = e / dk, d = e % dk;
        float u = 0.0f, v = 0.0f;
        if (i < nq) {
            const float qd = a.q[static_cast<size_t>(sg.f + i0 + i) * a.qs + h * dk + d];
            u = add_r<RM>(qd, a.bu[h * dk + d]);
            v = add_r<RM>(qd, a.bv[h * dk + d]);
        }
        qu[i * DS + d] = u;
        qv[i * DS + d] = v;
    }

    // rows j0 .. j0 + 63 of K (kind 0) or P (kind 1) into ST, zeros past the end
    auto stage_kp = [&](const float* src, unsigned long long rs, uint32_t j0, uint32_t valid, uint32_t np) {
        if constexpr (PANELS) {
            // (row j, dimension d) at ((j/16) dk + d) 16 + j%16: four rows a 16-byte load
            for (uint32_t e = tid; e < (ACH / 4) * dk; e += A_THREADS) {
                const uint32_t d = e % dk, jq = e / dk, j = j0 + 4 * jq;
                float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (j < np) v = *reinterpret_cast<const float4*>(src + (static_cast<size_t>(j / 16) * dk + d) * 16 + j % 16);
                ST[(4 * jq + 0) * DS + d] = v.x;
                ST[(4 * jq + 1) * DS + d] = v.y;
                ST[(4 * jq + 2) * DS + d] = v.z;
                ST[(4 * jq + 3) * DS + d] = v.w;
            }
            (void)rs;
            (void)valid;
        } else {
            for (uint32_t e = tid; e < ACH * (dk / 4); e += A_THREADS) {
                const uint32_t d4 = e % (dk / 4), jj = e / (dk / 4), j = j0 + jj;
                float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (j < valid) v = *reinterpret_cast<const float4*>(src + static_cast<size_t>(j) * rs + 4 * d4);
                *reinterpret_cast<float4*>(&ST[jj * DS + 4 * d4]) = v;
            }
            (void)np;
        }
    };

    // scores (kind 0: against qu into S) and position products (kind 1:
    // against qv into B), each + 0 as gemm_f32 adds its absent bias
    const uint32_t kq = tid % 16, qp = tid / 16;
    for (int kind = 0; kind < 2; kind++) {
        const float* qrow = kind == 0 ? qu : qv;
        const uint32_t start = kind == 0 ? 0 : w0, count = kind == 0 ? T : W;
        float* dst = kind == 0 ? S : B;
        const uint32_t dstride = kind == 0 ? SP : BP;
        for (uint32_t c0 = 0; c0 < count; c0 += ACH) {
            __syncthreads();  // ST is free, the queries are in
            if (kind == 0)
                stage_kp(kh, a.ks, c0, T, Tp);
            else
                stage_kp(ph, a.ps, start + c0, R, Pp);
            __syncthreads();
            float acc[2][4];
#pragma unroll
            for (int q2 = 0; q2 < 2; q2++)
#pragma unroll
                for (int e = 0; e < 4; e++) acc[q2][e] = 0.0f;
            const float* q0 = qrow + (2 * qp) * DS;
            const float* q1 = q0 + DS;
            for (uint32_t d = 0; d < dk; d += 4) {
                const float4 a0 = *reinterpret_cast<const float4*>(q0 + d);
                const float4 a1 = *reinterpret_cast<const float4*>(q1 + d);
                float4 r[4];
#pragma unroll
                for (int e = 0; e < 4; e++) r[e] = *reinterpret_cast<const float4*>(&ST[(kq + 16 * e) * DS + d]);
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    acc[0][e] = fma_r<RM>(r[e].x, a0.x, acc[0][e]);
                    acc[1][e] = fma_r<RM>(r[e].x, a1.x, acc[1][e]);
                }
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    acc[0][e] = fma_r<RM>(r[e].y, a0.y, acc[0][e]);
                    acc[1][e] = fma_r<RM>(r[e].y, a1.y, acc[1][e]);
                }
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    acc[0][e] = fma_r<RM>(r[e].z, a0.z, acc[0][e]);
                    acc[1][e] = fma_r<RM>(r[e].z, a1.z, acc[1][e]);
                }
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    acc[0][e] = fma_r<RM>(r[e].w, a0.w, acc[0][e]);
                    acc[1][e] = fma_r<RM>(r[e].w, a1.w, acc[1][e]);
                }
            }
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const uint32_t j = c0 + kq + 16 * e;
                if (j < count) {
                    dst[(2 * qp) * dstride + j] = add_r<RM>(acc[0][e], 0.0f);
                    dst[(2 * qp + 1) * dstride + j] = add_r<RM>(acc[1][e], 0.0f);
                }
            }
        }
    }
    __syncthreads();

    // each query's scores plus its positions, then its softmax (core/encoder.c:315-321)
    const float scale = div_r<RM>(1.0f, sqrt_r<RM>(static_cast<float>(dk)));
    for (uint32_t i = warp; i < nq; i += A_THREADS / 32) {
        float* srow = S + i * SP;
        const float* brow = B + i * BP + (T - 1 - (i0 + i)) - w0;
        for (uint32_t k = lane; k < T; k += 32) srow[k] = add_r<RM>(srow[k], brow[k]);
        __syncwarp();
        softmax_row<RM>(srow, T, scale, lane);
    }

    // the weighted values (core/encoder.c:323-324): o = V^T s + 0
    const uint32_t ntiles = dk;  // (AQ / 4) query quads x (dk / 4) dimension quads
    float acc[2][4][4];
#pragma unroll
    for (int u = 0; u < 2; u++)
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int e = 0; e < 4; e++) acc[u][i][e] = 0.0f;
    for (uint32_t c0 = 0; c0 < T; c0 += ACH) {
        __syncthreads();  // the weights are in; ST is free
        if constexpr (PANELS) {
            // (key j, dimension d) at ((d/16) T + j) 16 + d%16: four dimensions a 16-byte load
            for (uint32_t e = tid; e < ACH * (dk / 4); e += A_THREADS) {
                const uint32_t d4 = e % (dk / 4), jj = e / (dk / 4), j = c0 + jj, d = 4 * d4;
                float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (j < T) v = *reinterpret_cast<const float4*>(vh + (static_cast<size_t>(d / 16) * T + j) * 16 + d % 16);
                *reinterpret_cast<float4*>(&ST[jj * DS + d]) = v;
            }
        } else {
            stage_kp(vh, a.vs, c0, T, T);
        }
        __syncthreads();
        const uint32_t kc = min(static_cast<uint32_t>(ACH), T - c0);
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const uint32_t tile = tid + u * A_THREADS;
            if (tile >= ntiles) break;
            const uint32_t dq = tile % (dk / 4), qg = tile / (dk / 4);
            const float* w0r = S + (4 * qg) * SP + c0;
            uint32_t kk = 0;
            for (; kk + 4 <= kc; kk += 4) {
                float4 p[4];
#pragma unroll
                for (int i = 0; i < 4; i++) p[i] = *reinterpret_cast<const float4*>(w0r + i * SP + kk);
#pragma unroll
                for (int s = 0; s < 4; s++) {
                    const float4 v = *reinterpret_cast<const float4*>(&ST[(kk + s) * DS + 4 * dq]);
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float pk = s == 0 ? p[i].x : s == 1 ? p[i].y : s == 2 ? p[i].z : p[i].w;
                        acc[u][i][0] = fma_r<RM>(v.x, pk, acc[u][i][0]);
                        acc[u][i][1] = fma_r<RM>(v.y, pk, acc[u][i][1]);
                        acc[u][i][2] = fma_r<RM>(v.z, pk, acc[u][i][2]);
                        acc[u][i][3] = fma_r<RM>(v.w, pk, acc[u][i][3]);
                    }
                }
            }
            for (; kk < kc; kk++) {
                const float4 v = *reinterpret_cast<const float4*>(&ST[kk * DS + 4 * dq]);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float pk = w0r[i * SP + kk];
                    acc[u][i][0] = fma_r<RM>(v.x, pk, acc[u][i][0]);
                    acc[u][i][1] = fma_r<RM>(v.y, pk, acc[u][i][1]);
                    acc[u][i][2] = fma_r<RM>(v.z, pk, acc[u][i][2]);
                    acc[u][i][3] = fma_r<RM>(v.w, pk, acc[u][i][3]);
                }
            }
        }
    }
#pragma unroll
    for (int u = 0; u < 2; u++) {
        const uint32_t tile = tid + u * A_THREADS;
        if (tile >= ntiles) break;
        const uint32_t dq = tile % (dk / 4), qg = tile / (dk / 4);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t qi = 4 * qg + i;
            if (qi >= nq) break;
            float* orow = a.o + static_cast<size_t>(sg.f + i0 + qi) * a.os + h * dk + 4 * dq;
#pragma unroll
            for (int e = 0; e < 4; e++) orow[e] = add_r<RM>(acc[u][i][e], 0.0f);
        }
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
    attention_kernel<RM, PANELS><<<a.items, A_THREADS, smem, stream>>>(a);
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
    cudaError_t e = allow_smem(attention_kernel<RM, true>, optin);
    if (e == cudaSuccess) e = allow_smem(attention_kernel<RM, false>, optin);
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

size_t attention_smem(uint32_t dk, uint32_t sp, uint32_t bp) {
    return (static_cast<size_t>(2 * AQ + ACH) * (dk + 4) + static_cast<size_t>(AQ) * (sp + bp)) * sizeof(float);
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
    const size_t smem = attention_smem(a.dk, a.sp, a.bp);
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
