// TDT's greedy search (core/decoder.c:125-179) over a batch of segments in
// lockstep, on the device, sm_100a: each round every segment still running
// takes one joint step at its own frame, and the segments that emitted a
// token step their prediction network before the next round. The int8
// products (the LSTM layers' wx and wh, jpred, jout) are the product kernel
// (pkb_gemm.cu) with the batch's segments as its columns; this file has the
// float steps around them:
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
};
static_assert(offsetof(TdtSeg, active) == 4 * TDT_SEG_ACTIVE && offsetof(TdtSeg, over) == 4 * TDT_SEG_OVER,
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

// The joint's input for every running segment: relu(f_t + g) (g its
// prediction's jpred, just stepped where it emitted), quantized as one block.
template <int RM>
__global__ void __launch_bounds__(TD_THREADS) tdt_joint_in(TdtArgs a) {
    __shared__ uint32_t red[TD_THREADS / 32];
    extern __shared__ __align__(16) float zs[];
    const uint32_t s = blockIdx.x, J = a.J;
    TdtSeg* g = reinterpret_cast<TdtSeg*>(a.seg) + s;
    const bool active = g->active, fresh = g->pred;
    float* gp = a.gp + static_cast<size_t>(s) * J;
    const float* gn = a.gpn + static_cast<size_t>(s) * J;
    const float* f = a.f + (static_cast<size_t>(a.f0[s]) + (active ? g->t : 0)) * J;
    for (uint32_t j = threadIdx.x; j < J; j += blockDim.x) {
        float gj = gp[j];
        if (fresh) {
            gj = gn[j];
            gp[j] = gj;
        }
        float z = 0.0f;
        if (active) {
            const float v = add_r<RM>(f[j], gj);
            z = v > 0.0f ? v : 0.0f;
        }
        zs[j] = z;
    }
    __syncthreads();
    if (threadIdx.x == 0) g->pred = 0;
    quant_row<RM>(a.qz + static_cast<size_t>(s) * J, a.dz + s, zs, J, red);
}

// The joint's choice and the search's step for every running segment
// (core/decoder.c:93-100, :132-148). The logits are finite (a product of
// bounded integers and finite scales plus a finite bias), so the first
// largest is the reduction that keeps the larger value and, of equal ones,
// the lower index.
__global__ void __launch_bounds__(TD_THREADS) tdt_step(TdtArgs a) {
    __shared__ float bv[TD_THREADS / 32];
    __shared__ uint32_t bi[TD_THREADS / 32];
    __shared__ uint32_t s_emit, s_label;
    const uint32_t s = blockIdx.x, V = a.V, lane = threadIdx.x % 32, warp = threadIdx.x / 32;
    TdtSeg* g = reinterpret_cast<TdtSeg*>(a.seg) + s;
    if (!g->active) return;  // the block's uniform choice
    const float* lg = a.logits + static_cast<size_t>(s) * a.nout;
    float best = lg[0];
    uint32_t at = 0;
    for (uint32_t i = threadIdx.x; i <= V; i += blockDim.x)
        if (lg[i] > best || (lg[i] == best && i < at)) {
            best = lg[i];
            at = i;
        }
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
            if (lg[V + 1 + i] > lg[V + 1 + di]) di = i;
        const uint32_t t0 = g->t;
        uint32_t d = a.dur[di];
        uint32_t emit = 0;
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

}  // namespace pkb
