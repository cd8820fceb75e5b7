// TDT's greedy search (core/decoder.c:125-179) over a batch of segments in
// lockstep, on the device, sm_100a: each round every segment still running
// takes one joint step at its own frame, and the segments that emitted a
// token step their prediction network before the next round. Two forms:
// tdt_persist, the whole search as one cooperative launch (below, where the
// batch's inputs fit a CTA's shared memory), and rounds of launches, whose
// int8 products (the LSTM layers' wx and wh, jpred, jout) are the product
// kernel (pkb_gemm.cu) with the batch's segments as its columns and whose
// float steps around them are these kernels:
//
//   tdt_lstm       k_lstm (backend/ref/kernels.c:203-212) with pk_sigmoidf and
//                  pk_tanhf (core/vmath.h:149-165), then h quantized as one
//                  block, the input of the next layer's wx and of the next
//                  step's wh
//   tdt_joint_in   joint's relu(f_t + g) (core/decoder.c:87-91), quantized as
//                  one block for jout
//   tdt_step       joint's two first maxima (:93-100) and the search's step:
//                  skip frames on a blank, emit a token, the max_symbols rule
//
// Every float operation is the reference's, rounded once in the mode RM; the
// quantization is k_quantize's (backend/ref/kernels.c:24-58).

#include <algorithm>

#include "pkb_device.cuh"
#include "pkb_internal.h"
#include "pkb_vmath.cuh"

namespace pkb {

namespace {

constexpr int TD_THREADS = 256;

// pk_sigmoidf (core/vmath.h:149-151): 1 / (1 + pk_expf(-x))
template <int RM>
__device__ __forceinline__ float pk_sigmoid(float x) {
    return div_r<RM>(1.0f, add_r<RM>(1.0f, pk_exp<RM>(-x)));
}

// pk_tanhf (core/vmath.h:153-165) with its constants (:108-116)
template <int RM>
__device__ __forceinline__ float pk_tanh(float x) {
    const float a = fabsf(x);
    if (a < 0.625f) {
        const float x2 = mul_r<RM>(x, x);
        float p = -0x1.75e1cep-8f;
        p = fma_r<RM>(p, x2, 0x1.52269cp-6f);
        p = fma_r<RM>(p, x2, -0x1.b83c5ap-5f);
        p = fma_r<RM>(p, x2, 0x1.110726p-3f);
        p = fma_r<RM>(p, x2, -0x1.555532p-2f);
        return fma_r<RM>(mul_r<RM>(x, x2), p, x);
    }
    const float e = pk_exp<RM>(mul_r<RM>(2.0f, a));
    return copysignf(sub_r<RM>(1.0f, div_r<RM>(2.0f, add_r<RM>(e, 1.0f))), x);
}

// The largest of the block's values (as the bits of |v|, so that a NaN or an
// infinity sorts above every finite value), to every thread.
__device__ __forceinline__ uint32_t block_max_bits(uint32_t m, uint32_t* red) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    __syncthreads();  // red is free
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = 0;
    for (uint32_t w = 0; w < blockDim.x / 32; w++) m = max(m, red[w]);
    return m;
}

// k_quantize's block (backend/ref/kernels.c:24-58) over the n floats of v
// (shared memory), the whole CTA: a block holding a NaN or an infinity, or
// whose largest magnitude is below 2^-121, becomes zeros with scale 0; any
// other is scaled by amax / 127 and rounded in the mode to [-127, 127].
template <int RM>
__device__ void quant_row(int8_t* q, float* d, const float* v, uint32_t n, uint32_t* red) {
    uint32_t m = 0;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) m = max(m, __float_as_uint(v[i]) & 0x7fffffffu);
    m = block_max_bits(m, red);
    const float amax = __uint_as_float(m);
    if (m >= 0x7f800000u || amax < 0x1p-121f) {
        for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) q[i] = 0;
        if (threadIdx.x == 0) *d = 0.0f;
        return;
    }
    const float id = div_r<RM>(127.0f, amax);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) q[i] = static_cast<int8_t>(quant1<RM>(v[i], id) & 0xffu);
    if (threadIdx.x == 0) *d = div_r<RM>(amax, 127.0f);
}

// A segment's search state.
struct TdtSeg {
    uint32_t t, last, lasts, ntok;
    uint32_t active;  // still searching
    uint32_t pred;    // its prediction network steps before its next joint
    uint32_t label;   // the token it steps on
    uint32_t over;    // more tokens than the capacity
    uint32_t steps;   // joint steps taken (rounds in which it was searching)
};
static_assert(offsetof(TdtSeg, active) == 4 * TDT_SEG_ACTIVE && offsetof(TdtSeg, over) == 4 * TDT_SEG_OVER &&
                  offsetof(TdtSeg, steps) == 4 * TDT_SEG_STEPS,
              "the words the host reads back");

// The first layer's quantized input for segment s: the embedding of its
// label, from the table quantized once a call (a row of P, one block).
__device__ __forceinline__ void gather_label(const TdtArgs& a, uint32_t s, uint32_t label) {
    const uint32_t P = a.P;
    const int8_t* src = a.qembed + static_cast<size_t>(label) * P;
    int8_t* dst = a.qx + static_cast<size_t>(s) * P;
    for (uint32_t i = threadIdx.x; i < P; i += blockDim.x) dst[i] = src[i];
    if (threadIdx.x == 0) a.dx[s] = a.dembed[label];
}

// Every segment's state at the start: frame 0, nothing emitted, the blank's
// prediction from a zero state next (core/decoder.c:163-166, :127).
__global__ void __launch_bounds__(TD_THREADS) tdt_init(TdtArgs a) {
    const uint32_t s = blockIdx.x;
    TdtSeg* g = reinterpret_cast<TdtSeg*>(a.seg) + s;
    const bool live = a.T[s] > 0;
    if (threadIdx.x == 0) {
        g->t = 0;
        g->last = 0xffffffffu;
        g->lasts = 0;
        g->ntok = 0;
        g->active = live;
        g->pred = live;
        g->label = a.V;
        g->over = 0;
        g->steps = 0;
        a.ntok[s] = 0;
    }
    if (live) gather_label(a, s, a.V);
}

// The LSTM cell of layer l for every segment whose prediction steps: h and
// c in place from the gates [i f u o] (4P a segment), then h quantized.
template <int RM>
__global__ void __launch_bounds__(TD_THREADS) tdt_lstm(TdtArgs a, uint32_t l) {
    __shared__ uint32_t red[TD_THREADS / 32];
    extern __shared__ __align__(16) float hs[];
    const uint32_t s = blockIdx.x, P = a.P;
    const TdtSeg* g = reinterpret_cast<const TdtSeg*>(a.seg) + s;
    if (!g->pred) return;  // the block's uniform choice
    float* h = a.h + (static_cast<size_t>(l) * a.S + s) * P;
    float* c = a.c + (static_cast<size_t>(l) * a.S + s) * P;
    const float* gt = a.gates + static_cast<size_t>(s) * 4 * P;
    for (uint32_t j = threadIdx.x; j < P; j += blockDim.x) {
        const float i = pk_sigmoid<RM>(gt[j]);
        const float f = pk_sigmoid<RM>(gt[P + j]);
        const float u = pk_tanh<RM>(gt[2 * P + j]);
        const float o = pk_sigmoid<RM>(gt[3 * P + j]);
        const float cj = add_r<RM>(mul_r<RM>(f, c[j]), mul_r<RM>(i, u));
        c[j] = cj;
        const float hj = mul_r<RM>(o, pk_tanh<RM>(cj));
        h[j] = hj;
        hs[j] = hj;
    }
    __syncthreads();
    const size_t row = static_cast<size_t>(l) * a.S + s;
    quant_row<RM>(a.qh + row * P, a.dh + row, hs, P, red);
}

// The joint's input for segment s: relu(f_t + g) (g its prediction's
// jpred, just stepped where it emitted), quantized as one block; the whole
// CTA, zs J floats of shared memory. Reads what other CTAs of a persistent
// grid wrote through L2 (the state volatile, the vectors __ldcg).
template <int RM>
__device__ void joint_in_seg(const TdtArgs& a, uint32_t s, float* zs, uint32_t* red) {
    const uint32_t J = a.J;
    volatile TdtSeg* g = reinterpret_cast<volatile TdtSeg*>(a.seg) + s;
    const bool active = g->active, fresh = g->pred;
    const uint32_t t = active ? g->t : 0;
    float* gp = a.gp + static_cast<size_t>(s) * J;
    const float* gn = a.gpn + static_cast<size_t>(s) * J;
    const float* f = a.f + (static_cast<size_t>(a.f0[s]) + t) * J;
    for (uint32_t j = threadIdx.x; j < J; j += blockDim.x) {
        float gj = __ldcg(gp + j);
        if (fresh) {
            gj = __ldcg(gn + j);
            gp[j] = gj;
        }
        float z = 0.0f;
        if (active) {
            const float v = add_r<RM>(f[j], gj);
            z = v > 0.0f ? v : 0.0f;
        }
        zs[j] = z;
    }
    __syncthreads();  // every thread has read the state
    if (threadIdx.x == 0) g->pred = 0;
    quant_row<RM>(a.qz + static_cast<size_t>(s) * J, a.dz + s, zs, J, red);
}

// The joint's input for every running segment, a CTA each.
template <int RM>
__global__ void __launch_bounds__(TD_THREADS) tdt_joint_in(TdtArgs a) {
    __shared__ uint32_t red[TD_THREADS / 32];
    extern __shared__ __align__(16) float zs[];
    joint_in_seg<RM>(a, blockIdx.x, zs, red);
}

// The joint's choice and the search's step for every running segment
// (core/decoder.c:93-100, :132-148). The logits are finite (a product of
// bounded integers and finite scales plus a finite bias), so the first
// largest is the reduction that keeps the larger value and, of equal ones,
// the lower index.
// The whole CTA, for segment s; reads what other CTAs of a persistent grid
// wrote through L2 (the state volatile, the logits __ldcg).
__device__ void step_seg(const TdtArgs& a, uint32_t s) {
    __shared__ float bv[TD_THREADS / 32];
    __shared__ uint32_t bi[TD_THREADS / 32];
    __shared__ uint32_t s_emit, s_label;
    const uint32_t V = a.V, lane = threadIdx.x % 32, warp = threadIdx.x / 32;
    volatile TdtSeg* g = reinterpret_cast<volatile TdtSeg*>(a.seg) + s;
    if (!g->active) return;  // the block's uniform choice
    const float* lg = a.logits + static_cast<size_t>(s) * a.nout;
    float best = __ldcg(lg);
    uint32_t at = 0;
    auto take = [&](float v, uint32_t i) {
        if (v > best || (v == best && i < at)) {
            best = v;
            at = i;
        }
    };
    // four logits a load where the row is 16-byte aligned (a multiple of 4
    // of them a row), the rest one at a time
    const uint32_t n4 = (a.nout % 4 == 0 && (reinterpret_cast<uintptr_t>(lg) & 15) == 0) ? (V + 1) / 4 : 0;
#pragma unroll 4
    for (uint32_t i = threadIdx.x; i < n4; i += blockDim.x) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(lg) + i);
        take(v.x, 4 * i);
        take(v.y, 4 * i + 1);
        take(v.z, 4 * i + 2);
        take(v.w, 4 * i + 3);
    }
    for (uint32_t i = 4 * n4 + threadIdx.x; i <= V; i += blockDim.x) take(__ldcg(lg + i), i);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, at, o);
        if (ob > best || (ob == best && oi < at)) {
            best = ob;
            at = oi;
        }
    }
    if (lane == 0) {
        bv[warp] = best;
        bi[warp] = at;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float b = bv[0];
        uint32_t k = bi[0];
        for (uint32_t w = 1; w < blockDim.x / 32; w++)
            if (bv[w] > b || (bv[w] == b && bi[w] < k)) {
                b = bv[w];
                k = bi[w];
            }
        // the best duration, the first of equals (a handful: one thread)
        uint32_t di = 0;
        for (uint32_t i = 1; i < a.n_dur; i++)
            if (__ldcg(lg + V + 1 + i) > __ldcg(lg + V + 1 + di)) di = i;
        const uint32_t t0 = g->t;
        uint32_t d = a.dur[di];
        uint32_t emit = 0;
        g->steps++;
        if (k == V) {
            if (d == 0) d = 1;
            g->t = t0 + d;
            if (g->t >= a.T[s]) g->active = 0;  // a blank ran off the end: the search stops
        } else if (g->ntok == a.cap) {
            g->over = 1;  // no room for the token: the call fails
            g->active = 0;
        } else {
            int32_t* tk = a.toks + (static_cast<size_t>(s) * a.cap + g->ntok) * 3;
            tk[0] = static_cast<int32_t>(k);
            tk[1] = static_cast<int32_t>(t0);
            tk[2] = static_cast<int32_t>(a.dur[di]);
            g->ntok++;
            a.ntok[s] = g->ntok;
            g->t = t0 + d;
            g->lasts = g->last == t0 ? g->lasts + 1 : 1;
            g->last = t0;
            if (g->lasts >= a.max_symbols && g->last == g->t) g->t++;
            if (g->t >= a.T[s]) {
                g->active = 0;  // its prediction would change nothing
            } else {
                g->pred = 1;
                g->label = k;
                emit = 1;
            }
        }
        s_emit = emit;
        s_label = k;
    }
    __syncthreads();
    if (s_emit) gather_label(a, s, s_label);
    __syncthreads();  // s_emit and s_label stay until every thread has read them
}

__global__ void __launch_bounds__(TD_THREADS) tdt_step(TdtArgs a) { step_seg(a, blockIdx.x); }

// ------------------------------------------------- the persistent search --
//
// The same rounds as one cooperative launch whose CTAs all stay resident:
// each round's steps are phases separated by grid-wide barriers, so a round
// costs its phases and 2L + 4 barriers instead of 3L + 4 launches, each with
// its own start-up and its own fill of the SMs. The phases:
//
//   gates(l)   for each unit j of P (8 a job), the 4 gate rows i f u o of wx
//              and of wh against every segment's input and last h, the
//              gates, and k_lstm's cell: c, h (segments whose prediction
//              steps)
//   quant(l)   each such segment's h quantized as one block (a CTA a
//              segment), the next layer's input and the next step's wh input
//   jpred      g = jpred h + b (32 rows a job) for those segments
//   joint      relu(f_t + g) quantized (a CTA a segment; tdt_joint_in's)
//   jout       the logits (32 rows a job) of every running segment
//   step       tdt_step's choice and step (a CTA a segment)
//
// Each product is k_gemm_q8 with one block (qb = n): its int32 sums from
// mma.sync.m16n8k32 (16 rows x 8 segments, exact integer sums), then
// acc = fma((float)s, d, +0), v = acc * ws (+ bias) in the mode, as the
// product kernel computes a block of qb = n. At 64 segments a product is
// 64 columns, too few to feed tcgen05's 128-row tiles; the legacy MMA
// reads its operands from registers loaded out of shared memory, where a
// job's weight rows and every segment's input are staged (rows K + 16 bytes
// apart, so the fragment loads of a warp hit 32 distinct banks).
//
// Everything a phase reads that another CTA wrote in an earlier phase is
// read through L2 (__ldcg, or the state through a volatile pointer), and the
// barrier orders it: each CTA's writes, __syncthreads, a fence, then the
// arrival. A barrier wait that runs past the limit sets the error word and
// the abort flag, and every CTA returns at its next barrier.

constexpr uint32_t PS_ROWS = 32;  // weight rows a job: two MMA tiles of 16

__device__ __forceinline__ uint32_t ld_acquire_gpu(const unsigned* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Every CTA of the grid has arrived (true), or a wait gave up (false).
__device__ bool grid_barrier(const TdtPersist& p, uint32_t& epoch) {
    __shared__ int s_ok;
    __syncthreads();
    epoch++;
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(p.bar, 1u);
        const unsigned target = epoch * gridDim.x;
        const long long t0 = clock64();
        int ok = 1;
        while (ld_acquire_gpu(p.bar) < target) {
            if (*reinterpret_cast<volatile int*>(p.abort)) {
                ok = 0;
                break;
            }
            if (clock64() - t0 > p.timeout) {
                atomicExch(p.abort, 1);
                atomicOr(p.err, PKB_DEVERR_TIMEOUT);
                ok = 0;
                break;
            }
            __nanosleep(32);
        }
        __threadfence();
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

// Segments' quantized inputs [S][K] (written by other CTAs: copied through
// L2 by cp.async.cg) into shared memory, KP = K + 16 bytes apart, segments
// S..Spad-1 zeros. The copies are only issued: the caller commits and waits.
__device__ void stage_inputs(int8_t* dst, const int8_t* x, uint32_t S, uint32_t Spad, uint32_t K) {
    const uint32_t per = K / 16, KP = K + 16;
    for (uint32_t i = threadIdx.x; i < Spad * per; i += blockDim.x) {
        const uint32_t s = i / per, u = i % per;
        if (s < S)
            cp_async16(dst + s * KP + u * 16, x + static_cast<size_t>(s) * K + u * 16);
        else
            *reinterpret_cast<int4*>(dst + s * KP + u * 16) = make_int4(0, 0, 0, 0);
    }
}

// PS_ROWS weight rows [K] (read-only) into shared memory, KP apart: row lr
// is row `row(lr)` of w, or zeros where that is past `rows`. Issued only.
template <typename RowOf>
__device__ void stage_weights(int8_t* dst, const int8_t* w, uint32_t K, uint32_t rows, RowOf row) {
    const uint32_t per = K / 16, KP = K + 16;
    for (uint32_t i = threadIdx.x; i < PS_ROWS * per; i += blockDim.x) {
        const uint32_t lr = i / per, u = i % per, r = row(lr);
        if (r < rows)
            cp_async16(dst + lr * KP + u * 16, w + static_cast<size_t>(r) * K + u * 16);
        else
            *reinterpret_cast<int4*>(dst + lr * KP + u * 16) = make_int4(0, 0, 0, 0);
    }
}

// A CTA's scales of every segment [S] (written by other CTAs) into shared memory.
__device__ __forceinline__ void stage_scales(float* dst, const float* d, uint32_t S) {
    for (uint32_t s = threadIdx.x; s < S; s += blockDim.x) dst[s] = __ldcg(d + s);
}

// Everything staged by this thread's copies has landed, for every thread.
__device__ __forceinline__ void staged() {
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
}

// The int32 sums of NT tiles, each weight rows [16 rt, 16 rt + 16) of W[i]
// with the 8 segments of group sg[i] of X[i], over K (all in shared memory,
// KP apart), their MMAs interleaved. Lane (g = lane / 4, t = lane % 4)
// holds row 16 rt + g (c[i][0], c[i][1]) and + 8 (c[i][2], c[i][3]) of
// segments 8 sg + 2t and + 1.
template <int NT>
__device__ __forceinline__ void mma_rows(int (&c)[NT][4], const int8_t* const (&W)[NT], const int8_t* const (&X)[NT],
                                         const uint32_t (&sg)[NT], uint32_t rt, uint32_t K) {
    const uint32_t lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3, KP = K + 16;
    const int8_t* alo[NT];
    const int8_t* b[NT];
#pragma unroll
    for (int i = 0; i < NT; i++) {
        alo[i] = W[i] + (16 * rt + g) * KP + 4 * t;
        b[i] = X[i] + (8 * sg[i] + g) * KP + 4 * t;
        c[i][0] = c[i][1] = c[i][2] = c[i][3] = 0;
    }
    for (uint32_t k = 0; k < K; k += 32) {
#pragma unroll
        for (int i = 0; i < NT; i++) {
            const uint32_t a0 = *reinterpret_cast<const uint32_t*>(alo[i] + k);
            const uint32_t a1 = *reinterpret_cast<const uint32_t*>(alo[i] + 8 * KP + k);
            const uint32_t a2 = *reinterpret_cast<const uint32_t*>(alo[i] + k + 16);
            const uint32_t a3 = *reinterpret_cast<const uint32_t*>(alo[i] + 8 * KP + k + 16);
            const uint32_t b0 = *reinterpret_cast<const uint32_t*>(b[i] + k);
            const uint32_t b1 = *reinterpret_cast<const uint32_t*>(b[i] + k + 16);
            asm volatile(
                "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                "{%0,%1,%2,%3};"
                : "+r"(c[i][0]), "+r"(c[i][1]), "+r"(c[i][2]), "+r"(c[i][3])
                : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
        }
    }
}

// k_gemm_q8's one block (qb = n) of sum s: acc = fma((float)s, d, +0), then
// acc * ws, + b where there is a bias, each rounded in the mode.
template <int RM>
__device__ __forceinline__ float one_block(int s, float d, float ws, bool has_bias, float b) {
    const float acc = fma_r<RM>(i2f_r<RM>(s), d, 0.0f);
    float v = mul_r<RM>(acc, ws);
    if (has_bias) v = add_r<RM>(v, b);
    return v;
}

struct PsShared {
    uint8_t* base;  // the dynamic area
    uint32_t* pred;  // [S] whose prediction steps this round
    uint32_t* act;   // [S] still searching
};

// Layer l's gates and cells for the segments whose prediction steps.
template <int RM>
__device__ void ps_gates(const TdtArgs& a, const TdtPersist& p, uint32_t l, const PsShared& sh) {
    const uint32_t S = a.S, P = a.P, Spad = (S + 7) & ~7u, KP = P + 16, njobs = P / 8;
    if (blockIdx.x >= njobs) return;  // the CTA's uniform choice
    int8_t* x0 = reinterpret_cast<int8_t*>(sh.base);  // [Spad][KP] the layer's input
    int8_t* x1 = x0 + Spad * KP;                       // [Spad][KP] its h of the last step
    int8_t* wxs = x1 + Spad * KP;                      // [32][KP] the job's rows of wx
    int8_t* whs = wxs + PS_ROWS * KP;                  // [32][KP] of wh
    float* gsm = reinterpret_cast<float*>(whs + PS_ROWS * KP);  // [32][Spad] the gates
    float* d0 = gsm + PS_ROWS * Spad;                  // [Spad] the inputs' scales
    float* d1 = d0 + Spad;                             // [Spad] the last h's
    float* vs = d1 + Spad;                             // [3][32] the job's wxs, whs, lb
    const int8_t* qin = l ? a.qh + static_cast<size_t>(l - 1) * S * P : a.qx;
    const float* din = l ? a.dh + static_cast<size_t>(l - 1) * S : a.dx;
    const int8_t* qhl = a.qh + static_cast<size_t>(l) * S * P;
    const float* dhl = a.dh + static_cast<size_t>(l) * S;
    stage_inputs(x0, qin, S, Spad, P);
    stage_inputs(x1, qhl, S, Spad, P);
    stage_scales(d0, din, S);
    stage_scales(d1, dhl, S);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, rt = warp & 1;
    for (uint32_t job = blockIdx.x; job < njobs; job += gridDim.x) {
        const uint32_t j0 = 8 * job;
        // job row lr: gate lr / 8 of unit j0 + lr % 8
        auto row = [=](uint32_t lr) { return (lr >> 3) * P + j0 + (lr & 7); };
        if (job != blockIdx.x) __syncthreads();  // the last job's rows and gates are done with
        stage_weights(wxs, p.wx[l], P, 4 * P, row);
        stage_weights(whs, p.wh[l], P, 4 * P, row);
        if (threadIdx.x < PS_ROWS) {
            const uint32_t r = row(threadIdx.x);
            vs[threadIdx.x] = __ldg(p.wxs[l] + r);
            vs[PS_ROWS + threadIdx.x] = __ldg(p.whs[l] + r);
            vs[2 * PS_ROWS + threadIdx.x] = __ldg(p.lb[l] + r);
        }
        staged();
        const uint32_t sg0 = warp >> 1;
        if (sg0 < Spad / 8) {
            // the warp's two segment groups (the second may be past the last)
            const uint32_t sg1 = sg0 + 4 < Spad / 8 ? sg0 + 4 : sg0;
            int c[4][4];
            mma_rows<4>(c, {wxs, whs, wxs, whs}, {x0, x1, x0, x1}, {sg0, sg0, sg1, sg1}, rt, P);
#pragma unroll
            for (int h = 0; h < 2; h++) {
                if (h == 1 && sg1 == sg0) break;
                const uint32_t sg = h ? sg1 : sg0;
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const uint32_t lr = 16 * rt + (lane >> 2) + 8 * (e >> 1), sgm = 8 * sg + 2 * (lane & 3) + (e & 1);
                    if (sgm < S && sh.pred[sgm]) {
                        // gates = wx x + lb, then + wh h (the reference's two products, the second added)
                        const float gx = one_block<RM>(c[2 * h][e], d0[sgm], vs[lr], true, vs[2 * PS_ROWS + lr]);
                        const float gh = one_block<RM>(c[2 * h + 1][e], d1[sgm], vs[PS_ROWS + lr], false, 0.0f);
                        gsm[lr * Spad + sgm] = add_r<RM>(gx, gh);
                    }
                }
            }
        }
        // the warps' remaining segment groups (more than 64 segments)
        for (uint32_t sg = sg0 + 8; sg < Spad / 8; sg += 4) {
            int c[2][4];
            mma_rows<2>(c, {wxs, whs}, {x0, x1}, {sg, sg}, rt, P);
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const uint32_t lr = 16 * rt + (lane >> 2) + 8 * (e >> 1), sgm = 8 * sg + 2 * (lane & 3) + (e & 1);
                if (sgm < S && sh.pred[sgm]) {
                    const float gx = one_block<RM>(c[0][e], d0[sgm], vs[lr], true, vs[2 * PS_ROWS + lr]);
                    const float gh = one_block<RM>(c[1][e], d1[sgm], vs[PS_ROWS + lr], false, 0.0f);
                    gsm[lr * Spad + sgm] = add_r<RM>(gx, gh);
                }
            }
        }
        __syncthreads();
        // k_lstm's cell for units j0..j0+7
        for (uint32_t i = threadIdx.x; i < 8 * S; i += blockDim.x) {
            const uint32_t u = i & 7, sg = i >> 3;
            if (!sh.pred[sg]) continue;
            const size_t at = (static_cast<size_t>(l) * S + sg) * P + j0 + u;
            const float cold = __ldcg(a.c + at);
            const float ig = pk_sigmoid<RM>(gsm[u * Spad + sg]);
            const float fg = pk_sigmoid<RM>(gsm[(8 + u) * Spad + sg]);
            const float ug = pk_tanh<RM>(gsm[(16 + u) * Spad + sg]);
            const float og = pk_sigmoid<RM>(gsm[(24 + u) * Spad + sg]);
            const float cj = add_r<RM>(mul_r<RM>(fg, cold), mul_r<RM>(ig, ug));
            a.c[at] = cj;
            a.h[at] = mul_r<RM>(og, pk_tanh<RM>(cj));
        }
    }
}

// Layer l's new h quantized as one block, a CTA a segment whose prediction steps.
template <int RM>
__device__ void ps_quant_h(const TdtArgs& a, uint32_t l, const PsShared& sh, uint32_t* red) {
    const uint32_t S = a.S, P = a.P;
    float* hs = reinterpret_cast<float*>(sh.base);
    for (uint32_t s = blockIdx.x; s < S; s += gridDim.x) {
        if (!sh.pred[s]) continue;  // uniform
        const size_t row = static_cast<size_t>(l) * S + s;
        for (uint32_t j = threadIdx.x; j < P; j += blockDim.x) hs[j] = __ldcg(a.h + row * P + j);
        __syncthreads();
        quant_row<RM>(a.qh + row * P, a.dh + row, hs, P, red);
        __syncthreads();
    }
}

// A product of PS_ROWS rows a job against every segment's input x [S][K]
// (scales d), for the segments `want` marks: out[s * os + r] =
// one_block(...). Rows past `rows` are not written. A CTA stages the
// inputs and the weights of two of its jobs at once.
template <int RM>
__device__ void ps_product(const int8_t* w, const float* ws, const float* bias, uint32_t rows, uint32_t K,
                           const int8_t* x, const float* d, uint32_t S, const uint32_t* want, float* out, size_t os,
                           const PsShared& sh) {
    const uint32_t Spad = (S + 7) & ~7u, KP = K + 16, njobs = (rows + PS_ROWS - 1) / PS_ROWS;
    if (blockIdx.x >= njobs) return;  // uniform
    int8_t* xs = reinterpret_cast<int8_t*>(sh.base);  // [Spad][KP]
    int8_t* wsm = xs + Spad * KP;                     // [2][32][KP]
    float* ds = reinterpret_cast<float*>(wsm + 2 * PS_ROWS * KP);  // [Spad]
    float* vs = ds + Spad;                            // [2][2][32] row scales, biases
    stage_inputs(xs, x, S, Spad, K);
    stage_scales(ds, d, S);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, rt = warp & 1;
    for (uint32_t job = blockIdx.x; job < njobs; job += 2 * gridDim.x) {
        const uint32_t job2 = job + gridDim.x, nj = job2 < njobs ? 2 : 1;
        if (job != blockIdx.x) __syncthreads();
        for (uint32_t k = 0; k < nj; k++) {
            const uint32_t r0 = PS_ROWS * (k ? job2 : job);
            stage_weights(wsm + k * PS_ROWS * KP, w, K, rows, [=](uint32_t lr) { return r0 + lr; });
            if (threadIdx.x < PS_ROWS) {
                const uint32_t r = r0 + threadIdx.x;
                vs[k * 2 * PS_ROWS + threadIdx.x] = r < rows ? __ldg(ws + r) : 0.0f;
                vs[k * 2 * PS_ROWS + PS_ROWS + threadIdx.x] = r < rows && bias ? __ldg(bias + r) : 0.0f;
            }
        }
        staged();
        for (uint32_t k = 0; k < nj; k++) {
            const uint32_t r0 = PS_ROWS * (k ? job2 : job);
            const int8_t* W = wsm + k * PS_ROWS * KP;
            const float* v = vs + k * 2 * PS_ROWS;
            for (uint32_t sg = warp >> 1; sg < Spad / 8; sg += 8) {
                const uint32_t sg1 = sg + 4 < Spad / 8 ? sg + 4 : sg;
                int c[2][4];
                mma_rows<2>(c, {W, W}, {xs, xs}, {sg, sg1}, rt, K);
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    if (h == 1 && sg1 == sg) break;
                    const uint32_t g = h ? sg1 : sg;
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const uint32_t lr = 16 * rt + (lane >> 2) + 8 * (e >> 1), r = r0 + lr;
                        const uint32_t sgm = 8 * g + 2 * (lane & 3) + (e & 1);
                        if (r < rows && sgm < S && want[sgm])
                            out[sgm * os + r] = one_block<RM>(c[h][e], ds[sgm], v[lr], bias != nullptr, v[PS_ROWS + lr]);
                    }
                }
            }
        }
    }
}

template <int RM>
__global__ void __launch_bounds__(TD_THREADS, 1) tdt_persist(TdtArgs a, TdtPersist p) {
    extern __shared__ __align__(16) uint8_t ps_smem[];
    __shared__ uint32_t red[TD_THREADS / 32];
    __shared__ uint32_t s_any_act, s_any_pred;
    const uint32_t S = a.S, P = a.P, J = a.J;
    PsShared sh;
    sh.pred = reinterpret_cast<uint32_t*>(ps_smem);
    sh.act = sh.pred + S;
    sh.base = ps_smem + ((8 * static_cast<size_t>(S) + 15) & ~size_t(15));
    uint32_t epoch = 0;
    for (uint32_t round = 0; round < p.max_rounds; round++) {
        // every CTA reads the same states: the last writes to them came
        // before the barrier that ended the last round
        if (threadIdx.x == 0) {
            s_any_act = 0;
            s_any_pred = 0;
        }
        __syncthreads();
        for (uint32_t s = threadIdx.x; s < S; s += blockDim.x) {
            volatile TdtSeg* g = reinterpret_cast<volatile TdtSeg*>(a.seg) + s;
            const uint32_t act = g->active, pred = act && g->pred;
            sh.act[s] = act;
            sh.pred[s] = pred;
            if (act) atomicOr(&s_any_act, 1u);
            if (pred) atomicOr(&s_any_pred, 1u);
        }
        __syncthreads();
        if (!s_any_act) break;  // every search has ended (the grid's uniform choice)
        if (s_any_pred) {
            for (uint32_t l = 0; l < p.L; l++) {
                ps_gates<RM>(a, p, l, sh);
                if (!grid_barrier(p, epoch)) return;
                ps_quant_h<RM>(a, l, sh, red);
                if (!grid_barrier(p, epoch)) return;
            }
            const size_t top = static_cast<size_t>(p.L - 1) * S;
            ps_product<RM>(p.jpred, p.jpreds, p.jpredb, J, P, a.qh + top * P, a.dh + top, S, sh.pred, a.gpn, J, sh);
            if (!grid_barrier(p, epoch)) return;
        }
        for (uint32_t s = blockIdx.x; s < S; s += gridDim.x) {
            joint_in_seg<RM>(a, s, reinterpret_cast<float*>(sh.base), red);
            __syncthreads();
        }
        if (!grid_barrier(p, epoch)) return;
        ps_product<RM>(p.jout, p.jouts, p.joutb, a.nout, J, a.qz, a.dz, S, sh.act, a.logits, a.nout, sh);
        if (!grid_barrier(p, epoch)) return;
        for (uint32_t s = blockIdx.x; s < S; s += gridDim.x) step_seg(a, s);
        if (!grid_barrier(p, epoch)) return;
    }
}

template <int RM>
cudaError_t tdt_round_rm(const TdtArgs& a, int phase, uint32_t l, cudaStream_t stream) {
    switch (phase) {
    case TDT_LSTM:
        tdt_lstm<RM><<<a.S, TD_THREADS, a.P * sizeof(float), stream>>>(a, l);
        break;
    case TDT_JOINT_IN:
        tdt_joint_in<RM><<<a.S, TD_THREADS, a.J * sizeof(float), stream>>>(a);
        break;
    default:
        tdt_step<<<a.S, TD_THREADS, 0, stream>>>(a);
        break;
    }
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_tdt_init(const TdtArgs& a, cudaStream_t stream) {
    tdt_init<<<a.S, TD_THREADS, 0, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_tdt(const TdtArgs& a, int phase, uint32_t l, int rmode, cudaStream_t stream) {
    switch (rmode) {
    case 1: return tdt_round_rm<1>(a, phase, l, stream);
    case 2: return tdt_round_rm<2>(a, phase, l, stream);
    case 3: return tdt_round_rm<3>(a, phase, l, stream);
    default: return tdt_round_rm<0>(a, phase, l, stream);
    }
}

size_t tdt_seg_bytes() { return sizeof(TdtSeg); }

size_t tdt_persist_smem(const TdtArgs& a, size_t smem_max) {
    const size_t S = a.S, Spad = (S + 7) & ~size_t(7), KP = a.P + 16, KJ = a.J + 16;
    // gates: inputs and last h, the job's rows of wx and wh, the gates, two scale vectors, the job's vectors
    size_t need = 2 * Spad * KP + 2 * PS_ROWS * KP + 4 * PS_ROWS * Spad + 8 * Spad + 12 * PS_ROWS;
    // jpred, jout: inputs, two jobs' rows, the scales, the jobs' vectors
    need = std::max(need, Spad * std::max(KP, KJ) + 2 * PS_ROWS * std::max(KP, KJ) + 4 * Spad + 16 * PS_ROWS);
    need = std::max(need, 4 * static_cast<size_t>(std::max(a.P, a.J)));  // quantized rows
    need += (8 * S + 15) & ~size_t(15);                                  // the round's flags
    return need <= smem_max ? need : 0;
}

namespace {
template <int RM>
int persist_grid_rm(int sms, size_t smem) {
    if (cudaFuncSetAttribute(tdt_persist<RM>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
        return 0;
    int per = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, tdt_persist<RM>, TD_THREADS, smem) != cudaSuccess) return 0;
    return sms * std::min(per, 2);
}

template <int RM>
cudaError_t persist_rm(const TdtArgs& a, const TdtPersist& p, int grid, size_t smem, cudaStream_t stream) {
    TdtArgs aa = a;
    TdtPersist pp = p;
    void* args[] = {&aa, &pp};
    return cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(tdt_persist<RM>), dim3(grid), dim3(TD_THREADS),
                                       args, smem, stream);
}
}  // namespace

int tdt_persist_grid(const TdtArgs&, int rmode, int sms, size_t smem) {
    cudaGetLastError();
    int g = 0;
    switch (rmode) {
    case 1: g = persist_grid_rm<1>(sms, smem); break;
    case 2: g = persist_grid_rm<2>(sms, smem); break;
    case 3: g = persist_grid_rm<3>(sms, smem); break;
    default: g = persist_grid_rm<0>(sms, smem); break;
    }
    cudaGetLastError();  // a refusal above leaves no error behind: the rounds take the launches instead
    return g;
}

cudaError_t launch_tdt_persist(const TdtArgs& a, const TdtPersist& p, int rmode, int grid, size_t smem,
                               cudaStream_t stream) {
    switch (rmode) {
    case 1: return persist_rm<1>(a, p, grid, smem, stream);
    case 2: return persist_rm<2>(a, p, grid, smem, stream);
    case 3: return persist_rm<3>(a, p, grid, smem, stream);
    default: return persist_rm<0>(a, p, grid, smem, stream);
    }
}

}  // namespace pkb
