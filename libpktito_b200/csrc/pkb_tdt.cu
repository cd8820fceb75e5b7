// TDT's greedy search (core/decoder.c:125-179) over a batch of segments in
// lockstep, on the device, sm_100a: each round every segment still running
// takes one joint step at its own frame, and the segments that emitted a
// token step their prediction network before the next round. Two forms:
// tdt_persist, the whole search as one cooperative launch (below, where the
// model's rows fit a CTA's shared memory), and rounds of launches, whose
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
constexpr uint32_t TD_MAX_DUR = sizeof(TdtArgs::dur) / sizeof(uint32_t);

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
        // the best duration, the first of equals (a handful: one thread);
        // its logits and the state loaded before any is used, so their
        // round trips to L2 overlap
        float dl[TD_MAX_DUR];
#pragma unroll
        for (uint32_t i = 0; i < TD_MAX_DUR; i++) dl[i] = i < a.n_dur ? __ldcg(lg + V + 1 + i) : 0.0f;
        const uint32_t t0 = g->t, last = g->last, lasts = g->lasts, ntok = g->ntok, steps = g->steps;
        const uint32_t Ts = a.T[s];
        uint32_t di = 0;
        float bd = dl[0];
#pragma unroll
        for (uint32_t i = 1; i < TD_MAX_DUR; i++)
            if (i < a.n_dur && dl[i] > bd) {
                bd = dl[i];
                di = i;
            }
        const uint32_t dur = a.dur[di];
        uint32_t emit = 0;
        g->steps = steps + 1;
        if (k == V) {
            const uint32_t nt = t0 + (dur ? dur : 1);
            g->t = nt;
            if (nt >= Ts) g->active = 0;  // a blank ran off the end: the search stops
        } else if (ntok == a.cap) {
            g->over = 1;  // no room for the token: the call fails
            g->active = 0;
        } else {
            int32_t* tk = a.toks + (static_cast<size_t>(s) * a.cap + ntok) * 3;
            tk[0] = static_cast<int32_t>(k);
            tk[1] = static_cast<int32_t>(t0);
            tk[2] = static_cast<int32_t>(dur);
            g->ntok = ntok + 1;
            a.ntok[s] = ntok + 1;
            uint32_t nt = t0 + dur;
            const uint32_t nlasts = last == t0 ? lasts + 1 : 1;
            g->lasts = nlasts;
            g->last = t0;
            if (nlasts >= a.max_symbols && t0 == nt) nt++;
            g->t = nt;
            if (nt >= Ts) {
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
// job's weight rows and every segment's input are staged (rows ps_pitch(K)
// bytes apart, so the fragment loads of a warp hit distinct banks).
//
// Everything a phase reads that another CTA wrote in an earlier phase is
// read through L2 (__ldcg, or the state through a volatile pointer), and the
// barrier orders it: each CTA's writes, __syncthreads, a fence, then the
// arrival. A barrier wait that runs past the limit sets the error word and
// the abort flag, and every CTA returns at its next barrier.

constexpr uint32_t PS_ROWS = 32;  // weight rows a job: two MMA tiles of 16
constexpr uint32_t PS_COLS = 64;  // segments a chunk of a product's columns: 8 MMA groups of 8

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

// Bytes between rows of K int8 in shared memory: K rounded up so that the
// pitch in 16-byte units is 4 modulo 8, so a quarter-warp's 16-byte loads of
// two rows (lanes 4g + t, bytes 16t of row g) cover 8 distinct bank groups.
__host__ __device__ __forceinline__ uint32_t ps_pitch(uint32_t K) {
    const uint32_t u = K / 16;
    return 16 * (u + ((4u - u % 8u) & 7u));
}

// n rows of K quantized inputs, row c from src(c) (written by other CTAs or
// before the launch: copied through L2 by cp.async.cg), into shared memory
// ps_pitch(K) bytes apart, rows n..npad-1 zeros. The copies are only
// issued: the caller commits and waits.
template <typename Src>
__device__ void stage_inputs(int8_t* dst, Src src, uint32_t n, uint32_t npad, uint32_t K) {
    const uint32_t per = K / 16, KP = ps_pitch(K);
    for (uint32_t i = threadIdx.x; i < npad * per; i += blockDim.x) {
        const uint32_t c = i / per, u = i % per;
        if (c < n)
            cp_async16(dst + c * KP + u * 16, src(c) + u * 16);
        else
            *reinterpret_cast<int4*>(dst + c * KP + u * 16) = make_int4(0, 0, 0, 0);
    }
}

// PS_ROWS weight rows [K] (read-only) into shared memory, KP apart: row lr
// is row `row(lr)` of w, or zeros where that is past `rows`. Issued only.
template <typename RowOf>
__device__ void stage_weights(int8_t* dst, const int8_t* w, uint32_t K, uint32_t rows, RowOf row) {
    const uint32_t per = K / 16, KP = ps_pitch(K);
    for (uint32_t i = threadIdx.x; i < PS_ROWS * per; i += blockDim.x) {
        const uint32_t lr = i / per, u = i % per, r = row(lr);
        if (r < rows)
            cp_async16(dst + lr * KP + u * 16, w + static_cast<size_t>(r) * K + u * 16);
        else
            *reinterpret_cast<int4*>(dst + lr * KP + u * 16) = make_int4(0, 0, 0, 0);
    }
}

// n scales, scale c at *src(c) (written by other CTAs: through L2), into shared memory.
template <typename Src>
__device__ __forceinline__ void stage_scales(float* dst, Src src, uint32_t n) {
    for (uint32_t c = threadIdx.x; c < n; c += blockDim.x) dst[c] = __ldcg(src(c));
}

// Everything staged by this thread's copies has landed, for every thread.
__device__ __forceinline__ void staged() {
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
}

// The int32 sums of NT tiles, each weight rows [16 rt, 16 rt + 16) of W[i]
// with the 8 segments of group sg[i] of X[i], over K (all in shared memory,
// ps_pitch(K) apart), their MMAs interleaved. Lane (g = lane / 4, t = lane
// % 4) holds row 16 rt + g (c[i][0], c[i][1]) and + 8 (c[i][2], c[i][3]) of
// segments 8 sg + 2t and + 1.
//
// A sum of integer products does not depend on the order of its terms, so
// the MMA's k need only pair the same bytes of a weight row and of a
// segment's input: of each 64 bytes of K, lane t takes bytes 16t..16t+15 of
// its rows in one 16-byte load, bytes 0-7 as its k of one MMA (its fragment
// registers 0 and 2, resp. 0 and 1 of B) and 8-15 of the next; a K that is
// an odd multiple of 32 ends with 8-byte loads.
template <int NT>
__device__ __forceinline__ void mma_rows(int (&c)[NT][4], const int8_t* const (&W)[NT], const int8_t* const (&X)[NT],
                                         const uint32_t (&sg)[NT], uint32_t rt, uint32_t K) {
    const uint32_t lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3, KP = ps_pitch(K);
    const int8_t* alo[NT];
    const int8_t* b[NT];
#pragma unroll
    for (int i = 0; i < NT; i++) {
        alo[i] = W[i] + (16 * rt + g) * KP;
        b[i] = X[i] + (8 * sg[i] + g) * KP;
        c[i][0] = c[i][1] = c[i][2] = c[i][3] = 0;
    }
    auto mma = [](int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    };
    uint32_t k = 0;
    for (; k + 64 <= K; k += 64) {
#pragma unroll
        for (int i = 0; i < NT; i++) {
            const uint4 lo = *reinterpret_cast<const uint4*>(alo[i] + k + 16 * t);
            const uint4 hi = *reinterpret_cast<const uint4*>(alo[i] + 8 * KP + k + 16 * t);
            const uint4 bb = *reinterpret_cast<const uint4*>(b[i] + k + 16 * t);
            mma(c[i], lo.x, hi.x, lo.y, hi.y, bb.x, bb.y);
            mma(c[i], lo.z, hi.z, lo.w, hi.w, bb.z, bb.w);
        }
    }
    if (k < K) {  // the last 32 bytes: 8 a lane
#pragma unroll
        for (int i = 0; i < NT; i++) {
            const uint2 lo = *reinterpret_cast<const uint2*>(alo[i] + k + 8 * t);
            const uint2 hi = *reinterpret_cast<const uint2*>(alo[i] + 8 * KP + k + 8 * t);
            const uint2 bb = *reinterpret_cast<const uint2*>(b[i] + k + 8 * t);
            mma(c[i], lo.x, hi.x, lo.y, hi.y, bb.x, bb.y);
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
    uint8_t* base;    // the dynamic area
    uint32_t* plist;  // [np] the segments whose prediction steps this round, in order
    uint32_t* alist;  // [na] the segments still searching, in order
    TdtSeg* st;       // [S] every segment's search state: each CTA's own copy, all updated alike
    uint32_t np, na;
};

// Layer l's gates and cells for the segments whose prediction steps, as
// the columns of its products (column c: segment plist[c]), PS_COLS
// columns at a time (the job's weight rows staged once, each chunk's
// inputs then), so that shared memory does not grow with the batch. Layer
// 0's input is the embedding of the segment's label, quantized a row a
// block once a call.
template <int RM>
__device__ void ps_gates(const TdtArgs& a, const TdtPersist& p, uint32_t l, const PsShared& sh) {
    const uint32_t S = a.S, P = a.P, n = sh.np, KP = ps_pitch(P), njobs = P / 8;
    if (blockIdx.x >= njobs || !n) return;  // the CTA's uniform choice
    int8_t* x0 = reinterpret_cast<int8_t*>(sh.base);  // [PS_COLS][KP] the chunk's inputs
    int8_t* x1 = x0 + PS_COLS * KP;                    // [PS_COLS][KP] their h of the last step
    int8_t* wxs = x1 + PS_COLS * KP;                   // [32][KP] the job's rows of wx
    int8_t* whs = wxs + PS_ROWS * KP;                  // [32][KP] of wh
    float* gsm = reinterpret_cast<float*>(whs + PS_ROWS * KP);  // [32][PS_COLS] the gates
    float* d0 = gsm + PS_ROWS * PS_COLS;               // [PS_COLS] the inputs' scales
    float* d1 = d0 + PS_COLS;                          // [PS_COLS] the last h's
    float* vs = d1 + PS_COLS;                          // [3][32] the job's wxs, whs, lb
    const TdtSeg* st = sh.st;
    const int8_t* qin = l ? a.qh + static_cast<size_t>(l - 1) * S * P : nullptr;
    const float* din = l ? a.dh + static_cast<size_t>(l - 1) * S : nullptr;
    const int8_t* qhl = a.qh + static_cast<size_t>(l) * S * P;
    const float* dhl = a.dh + static_cast<size_t>(l) * S;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, rt = warp & 1;
    for (uint32_t job = blockIdx.x; job < njobs; job += gridDim.x) {
        const uint32_t j0 = 8 * job;
        // job row lr: gate lr / 8 of unit j0 + lr % 8
        auto row = [=](uint32_t lr) { return (lr >> 3) * P + j0 + (lr & 7); };
        __syncthreads();  // the last job's rows and chunk are done with
        stage_weights(wxs, p.wx[l], P, 4 * P, row);
        stage_weights(whs, p.wh[l], P, 4 * P, row);
        if (threadIdx.x < PS_ROWS) {
            const uint32_t r = row(threadIdx.x);
            vs[threadIdx.x] = __ldg(p.wxs[l] + r);
            vs[PS_ROWS + threadIdx.x] = __ldg(p.whs[l] + r);
            vs[2 * PS_ROWS + threadIdx.x] = __ldg(p.lb[l] + r);
        }
        for (uint32_t c0 = 0; c0 < n; c0 += PS_COLS) {
            const uint32_t* pl = sh.plist + c0;
            const uint32_t nc = n - c0 < PS_COLS ? n - c0 : PS_COLS, npad = (nc + 7) & ~7u;
            if (c0) __syncthreads();  // the last chunk's inputs and gates are done with
            if (l == 0) {
                stage_inputs(x0, [&](uint32_t c) { return a.qembed + static_cast<size_t>(st[pl[c]].label) * P; }, nc,
                             npad, P);
                stage_scales(d0, [&](uint32_t c) { return a.dembed + st[pl[c]].label; }, nc);
            } else {
                stage_inputs(x0, [&](uint32_t c) { return qin + static_cast<size_t>(pl[c]) * P; }, nc, npad, P);
                stage_scales(d0, [&](uint32_t c) { return din + pl[c]; }, nc);
            }
            stage_inputs(x1, [&](uint32_t c) { return qhl + static_cast<size_t>(pl[c]) * P; }, nc, npad, P);
            stage_scales(d1, [&](uint32_t c) { return dhl + pl[c]; }, nc);
            // cell i (below) is unit j0 + i % 8 of column i / 8; the old c of
            // this thread's first two, loaded while the copies land
            auto cell_at = [&](uint32_t i) { return (static_cast<size_t>(l) * S + pl[i >> 3]) * P + j0 + (i & 7); };
            float cpre0 = 0.0f, cpre1 = 0.0f;
            if (threadIdx.x < 8 * nc) cpre0 = __ldcg(a.c + cell_at(threadIdx.x));
            if (threadIdx.x + blockDim.x < 8 * nc) cpre1 = __ldcg(a.c + cell_at(threadIdx.x + blockDim.x));
            staged();
            // a warp: one row tile, column groups sg and sg + 4
            const uint32_t sg = warp >> 1;
            if (sg < npad / 8) {
                const uint32_t sg1 = sg + 4 < npad / 8 ? sg + 4 : sg;
                int c[4][4];
                mma_rows<4>(c, {wxs, whs, wxs, whs}, {x0, x1, x0, x1}, {sg, sg, sg1, sg1}, rt, P);
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    if (h == 1 && sg1 == sg) break;
                    const uint32_t g = h ? sg1 : sg;
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const uint32_t lr = 16 * rt + (lane >> 2) + 8 * (e >> 1), col = 8 * g + 2 * (lane & 3) + (e & 1);
                        if (col < nc) {
                            // gates = wx x + lb, then + wh h (the reference's two products, the second added)
                            const float gx = one_block<RM>(c[2 * h][e], d0[col], vs[lr], true, vs[2 * PS_ROWS + lr]);
                            const float gh = one_block<RM>(c[2 * h + 1][e], d1[col], vs[PS_ROWS + lr], false, 0.0f);
                            gsm[lr * PS_COLS + col] = add_r<RM>(gx, gh);
                        }
                    }
                }
            }
            __syncthreads();
            // k_lstm's cell for units j0..j0+7 of the chunk's columns
            for (uint32_t i = threadIdx.x, q = 0; i < 8 * nc; i += blockDim.x, q++) {
                const uint32_t u = i & 7, col = i >> 3;
                const size_t at = cell_at(i);
                const float cold = q == 0 ? cpre0 : q == 1 ? cpre1 : __ldcg(a.c + at);
                const float ig = pk_sigmoid<RM>(gsm[u * PS_COLS + col]);
                const float fg = pk_sigmoid<RM>(gsm[(8 + u) * PS_COLS + col]);
                const float ug = pk_tanh<RM>(gsm[(16 + u) * PS_COLS + col]);
                const float og = pk_sigmoid<RM>(gsm[(24 + u) * PS_COLS + col]);
                const float cj = add_r<RM>(mul_r<RM>(fg, cold), mul_r<RM>(ig, ug));
                a.c[at] = cj;
                a.h[at] = mul_r<RM>(og, pk_tanh<RM>(cj));
            }
        }
    }
}

// Layer l's new h quantized as one block, a CTA a segment whose prediction steps.
template <int RM>
__device__ void ps_quant_h(const TdtArgs& a, uint32_t l, const PsShared& sh, uint32_t* red) {
    const uint32_t S = a.S, P = a.P;
    float* hs = reinterpret_cast<float*>(sh.base);
    for (uint32_t i = blockIdx.x; i < sh.np; i += gridDim.x) {
        const size_t row = static_cast<size_t>(l) * S + sh.plist[i];
        for (uint32_t j = threadIdx.x; j < P; j += blockDim.x) hs[j] = __ldcg(a.h + row * P + j);
        __syncthreads();
        quant_row<RM>(a.qh + row * P, a.dh + row, hs, P, red);
        __syncthreads();
    }
}

// The first largest of values compared as floats as one key that
// atomicMax can combine: the larger value, and of equal ones (-0 and +0
// equal) the lower index. The logits are finite.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t i) {
    uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return (static_cast<unsigned long long>(b) << 32) | (0xFFFFFFFFu - i);
}
__device__ __forceinline__ uint32_t key_index(unsigned long long k) {
    return 0xFFFFFFFFu - static_cast<uint32_t>(k);
}

// A product of PS_ROWS rows a job against the inputs x [S][K] (scales d) of
// the n segments list names, as its columns: one_block(...) of row r and
// column c to out[list[c] * os + r] where out is given, and, where keys
// is, into each column's two keys (keys[2 list[c]]: the first largest
// token logit, rows 0..V; keys[2 list[c] + 1]: the first largest duration
// logit, rows V+1..V+n_dur, its index counted from V+1), reduced across a
// warp and the CTA first. Rows past `rows` are skipped. A CTA stages the
// weights of two of its jobs at once and the columns PS_COLS at a time.
template <int RM>
__device__ void ps_product(const int8_t* w, const float* ws, const float* bias, uint32_t rows, uint32_t K,
                           const int8_t* x, const float* d, const uint32_t* list, uint32_t n, float* out, size_t os,
                           unsigned long long* keys, uint32_t V, uint32_t n_dur, const PsShared& sh) {
    const uint32_t KP = ps_pitch(K), njobs = (rows + PS_ROWS - 1) / PS_ROWS;
    if (blockIdx.x >= njobs || !n) return;  // uniform
    int8_t* xs = reinterpret_cast<int8_t*>(sh.base);  // [PS_COLS][KP] the chunk's inputs
    int8_t* wsm = xs + PS_COLS * KP;                  // [2][32][KP]
    float* ds = reinterpret_cast<float*>(wsm + 2 * PS_ROWS * KP);  // [PS_COLS]
    float* vs = ds + PS_COLS;                         // [2][2][32] row scales, biases
    unsigned long long* sk = reinterpret_cast<unsigned long long*>(vs + 4 * PS_ROWS);  // [PS_COLS][2] the keys
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, rt = warp & 1;
    for (uint32_t job = blockIdx.x; job < njobs; job += 2 * gridDim.x) {
        const uint32_t job2 = job + gridDim.x, nj = job2 < njobs ? 2 : 1;
        __syncthreads();  // the last jobs' rows and chunk are done with
        for (uint32_t k = 0; k < nj; k++) {
            const uint32_t r0 = PS_ROWS * (k ? job2 : job);
            stage_weights(wsm + k * PS_ROWS * KP, w, K, rows, [=](uint32_t lr) { return r0 + lr; });
            if (threadIdx.x < PS_ROWS) {
                const uint32_t r = r0 + threadIdx.x;
                vs[k * 2 * PS_ROWS + threadIdx.x] = r < rows ? __ldg(ws + r) : 0.0f;
                vs[k * 2 * PS_ROWS + PS_ROWS + threadIdx.x] = r < rows && bias ? __ldg(bias + r) : 0.0f;
            }
        }
        for (uint32_t c0 = 0; c0 < n; c0 += PS_COLS) {
            const uint32_t* cl = list + c0;
            const uint32_t nc = n - c0 < PS_COLS ? n - c0 : PS_COLS, npad = (nc + 7) & ~7u;
            if (c0) __syncthreads();  // the last chunk's inputs and keys are done with
            stage_inputs(xs, [&](uint32_t c) { return x + static_cast<size_t>(cl[c]) * K; }, nc, npad, K);
            stage_scales(ds, [&](uint32_t c) { return d + cl[c]; }, nc);
            if (keys)
                for (uint32_t i = threadIdx.x; i < 2 * npad; i += blockDim.x) sk[i] = 0ull;
            staged();
            for (uint32_t k = 0; k < nj; k++) {
                const uint32_t r0 = PS_ROWS * (k ? job2 : job);
                const int8_t* W = wsm + k * PS_ROWS * KP;
                const float* v = vs + k * 2 * PS_ROWS;
                const uint32_t sg = warp >> 1;
                if (sg >= npad / 8) continue;  // warp-uniform
                const uint32_t sg1 = sg + 4 < npad / 8 ? sg + 4 : sg;
                int c[2][4];
                mma_rows<2>(c, {W, W}, {xs, xs}, {sg, sg1}, rt, K);
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    if (h == 1 && sg1 == sg) break;
                    const uint32_t g = h ? sg1 : sg;
                    // the lane's keys of its two columns (token, duration)
                    unsigned long long kt[2] = {0ull, 0ull}, kd[2] = {0ull, 0ull};
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const uint32_t lr = 16 * rt + (lane >> 2) + 8 * (e >> 1), r = r0 + lr;
                        const uint32_t col = 8 * g + 2 * (lane & 3) + (e & 1);
                        if (r < rows && col < nc) {
                            const float y = one_block<RM>(c[h][e], ds[col], v[lr], bias != nullptr, v[PS_ROWS + lr]);
                            if (out) out[cl[col] * os + r] = y;
                            if (keys) {
                                if (r <= V)
                                    kt[e & 1] = max(kt[e & 1], argmax_key(y, r));
                                else if (r <= V + n_dur)
                                    kd[e & 1] = max(kd[e & 1], argmax_key(y, r - V - 1));
                            }
                        }
                    }
                    if (keys) {
                        // the 8 lanes of a column (lane / 4 = the rows) reduced
                        // by shuffles, then one shared atomic a column and key
#pragma unroll
                        for (int o = 4; o <= 16; o <<= 1)
#pragma unroll
                            for (int xx = 0; xx < 2; xx++) {
                                kt[xx] = max(kt[xx], __shfl_xor_sync(0xffffffffu, kt[xx], o));
                                kd[xx] = max(kd[xx], __shfl_xor_sync(0xffffffffu, kd[xx], o));
                            }
                        if (lane < 4)
#pragma unroll
                            for (int xx = 0; xx < 2; xx++) {
                                const uint32_t col = 8 * g + 2 * lane + xx;
                                if (kt[xx]) atomicMax(&sk[2 * col], kt[xx]);
                                if (kd[xx]) atomicMax(&sk[2 * col + 1], kd[xx]);
                            }
                    }
                }
            }
            if (keys) {
                __syncthreads();
                for (uint32_t i = threadIdx.x; i < 2 * nc; i += blockDim.x)
                    if (sk[i]) atomicMax(keys + 2 * cl[i >> 1] + (i & 1), sk[i]);
            }
        }
    }
}

// The joint's input of running segment s (the whole CTA): relu(f_t + g),
// g its prediction's jpred (just stepped where it emitted), quantized as
// one block; zs J floats of shared memory.
template <int RM>
__device__ void ps_joint(const TdtArgs& a, uint32_t s, const TdtSeg& st, float* zs, uint32_t* red) {
    const uint32_t J = a.J;
    const bool fresh = st.pred;
    float* gp = a.gp + static_cast<size_t>(s) * J;
    const float* gn = a.gpn + static_cast<size_t>(s) * J;
    const float* f = a.f + (static_cast<size_t>(a.f0[s]) + st.t) * J;
    for (uint32_t j = threadIdx.x; j < J; j += blockDim.x) {
        float gj;
        if (fresh) {
            gj = __ldcg(gn + j);
            gp[j] = gj;
        } else {
            gj = __ldcg(gp + j);
        }
        const float v = add_r<RM>(f[j], gj);
        zs[j] = v > 0.0f ? v : 0.0f;
    }
    __syncthreads();
    quant_row<RM>(a.qz + static_cast<size_t>(s) * J, a.dz + s, zs, J, red);
}

// The search's step for segment s from its best token k and duration di
// (tdt_step's, core/decoder.c:132-148) on state g; where `owner`, the token
// is written out.
__device__ __forceinline__ void ps_step(const TdtArgs& a, uint32_t s, TdtSeg& g, uint32_t k, uint32_t di, bool owner) {
    const uint32_t t0 = g.t, dur = a.dur[di];
    g.steps++;
    if (k == a.V) {
        g.t = t0 + (dur ? dur : 1);
        if (g.t >= a.T[s]) g.active = 0;  // a blank ran off the end: the search stops
    } else if (g.ntok == a.cap) {
        g.over = 1;  // no room for the token: the call fails
        g.active = 0;
    } else {
        if (owner) {
            int32_t* tk = a.toks + (static_cast<size_t>(s) * a.cap + g.ntok) * 3;
            tk[0] = static_cast<int32_t>(k);
            tk[1] = static_cast<int32_t>(t0);
            tk[2] = static_cast<int32_t>(dur);
            a.ntok[s] = g.ntok + 1;
        }
        g.ntok++;
        g.t = t0 + dur;
        g.lasts = g.last == t0 ? g.lasts + 1 : 1;
        g.last = t0;
        if (g.lasts >= a.max_symbols && g.last == g.t) g.t++;
        if (g.t >= a.T[s]) {
            g.active = 0;  // its prediction would change nothing
        } else {
            g.pred = 1;
            g.label = k;
        }
    }
}

template <int RM>
__global__ void __launch_bounds__(TD_THREADS, 1) tdt_persist(TdtArgs a, TdtPersist p) {
    extern __shared__ __align__(16) uint8_t ps_smem[];
    __shared__ uint32_t red[TD_THREADS / 32];
    __shared__ uint32_t s_np, s_na;
    const uint32_t S = a.S, P = a.P, J = a.J;
    PsShared sh;
    sh.plist = reinterpret_cast<uint32_t*>(ps_smem);
    sh.alist = sh.plist + S;
    sh.st = reinterpret_cast<TdtSeg*>(sh.alist + S);
    sh.base = ps_smem + ((static_cast<size_t>(S) * (8 + sizeof(TdtSeg)) + 15) & ~size_t(15));
    // every CTA's copy of the states, as tdt_init left them
    for (uint32_t i = threadIdx.x; i < S * (sizeof(TdtSeg) / 4); i += blockDim.x)
        reinterpret_cast<uint32_t*>(sh.st)[i] = reinterpret_cast<const uint32_t*>(a.seg)[i];
    sh.na = 0;
    uint32_t epoch = 0;
    for (uint32_t round = 0; round < p.max_rounds; round++) {
        __syncthreads();
        if (round) {
            // the last round's step, from its jout's keys, for each segment
            // it ran: every CTA on its own copy, alike; the token written
            // by the segment's owner CTA
            const unsigned long long* kp = p.keys + ((round - 1) & 1) * 2 * S;
            for (uint32_t i = threadIdx.x; i < sh.na; i += blockDim.x) {
                const uint32_t s = sh.alist[i];
                const uint32_t k = key_index(__ldcg(kp + 2 * s)), di = key_index(__ldcg(kp + 2 * s + 1));
                ps_step(a, s, sh.st[s], k, di, s % gridDim.x == blockIdx.x);
            }
            __syncthreads();
        }
        // this round's jout keys start from zero (the buffer was last read at
        // the start of the last round, two barriers ago at least)
        if (blockIdx.x == 0)
            for (uint32_t i = threadIdx.x; i < 2 * S; i += blockDim.x) p.keys[(round & 1) * 2 * S + i] = 0ull;
        // the segments still searching and those whose prediction steps, in order
        if (threadIdx.x < 32) {
            uint32_t np = 0, na = 0;
            for (uint32_t s0 = 0; s0 < S; s0 += 32) {
                const uint32_t s = s0 + threadIdx.x;
                const uint32_t act = s < S && sh.st[s].active, pred = act && sh.st[s].pred;
                const uint32_t ma = __ballot_sync(0xffffffffu, act), mp = __ballot_sync(0xffffffffu, pred);
                const uint32_t below = (1u << threadIdx.x) - 1;
                if (act) sh.alist[na + __popc(ma & below)] = s;
                if (pred) sh.plist[np + __popc(mp & below)] = s;
                na += __popc(ma);
                np += __popc(mp);
            }
            if (threadIdx.x == 0) {
                s_np = np;
                s_na = na;
            }
        }
        __syncthreads();
        sh.np = s_np;
        sh.na = s_na;
        if (!sh.na) break;  // every search has ended (the grid's uniform choice)
        if (sh.np) {
            for (uint32_t l = 0; l < p.L; l++) {
                ps_gates<RM>(a, p, l, sh);
                if (!grid_barrier(p, epoch)) return;
                ps_quant_h<RM>(a, l, sh, red);
                if (!grid_barrier(p, epoch)) return;
            }
            const size_t top = static_cast<size_t>(p.L - 1) * S;
            ps_product<RM>(p.jpred, p.jpreds, p.jpredb, J, P, a.qh + top * P, a.dh + top, sh.plist, sh.np, a.gpn, J,
                           nullptr, 0, 0, sh);
            if (!grid_barrier(p, epoch)) return;
        }
        // the joint's input of every running segment; then no prediction is fresh
        for (uint32_t i = blockIdx.x; i < sh.na; i += gridDim.x) {
            ps_joint<RM>(a, sh.alist[i], sh.st[sh.alist[i]], reinterpret_cast<float*>(sh.base), red);
            __syncthreads();
        }
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < sh.np; i += blockDim.x) sh.st[sh.plist[i]].pred = 0;
        if (!grid_barrier(p, epoch)) return;
        // the logits of every running segment, reduced to the keys of its step
        ps_product<RM>(p.jout, p.jouts, p.joutb, a.nout, J, a.qz, a.dz, sh.alist, sh.na, nullptr, 0,
                       p.keys + (round & 1) * 2 * S, a.V, a.n_dur, sh);
        if (!grid_barrier(p, epoch)) return;
    }
    // the states for the host: each segment's by its owner
    __syncthreads();
    for (uint32_t s = blockIdx.x; s < S; s += gridDim.x)
        for (uint32_t i = threadIdx.x; i < sizeof(TdtSeg) / 4; i += blockDim.x)
            reinterpret_cast<uint32_t*>(a.seg)[s * (sizeof(TdtSeg) / 4) + i] =
                reinterpret_cast<const uint32_t*>(sh.st + s)[i];
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
    const size_t S = a.S, C = PS_COLS, KP = ps_pitch(a.P), KJ = ps_pitch(a.J);
    // gates: a chunk's inputs and last h, the job's rows of wx and wh, the gates, two scale vectors, the job's vectors
    size_t need = 2 * C * KP + 2 * PS_ROWS * KP + 4 * PS_ROWS * C + 8 * C + 12 * PS_ROWS;
    // jpred, jout: a chunk's inputs, two jobs' rows, the scales, the jobs' vectors, the columns' keys
    need = std::max(need, C * std::max(KP, KJ) + 2 * PS_ROWS * std::max(KP, KJ) + 4 * C + 16 * PS_ROWS + 16 * C);
    need = std::max(need, 4 * static_cast<size_t>(std::max(a.P, a.J)));  // quantized rows
    need += (S * (8 + sizeof(TdtSeg)) + 15) & ~size_t(15);               // the lists, the states
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
