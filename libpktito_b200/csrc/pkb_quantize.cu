// Activation quantization and the weights' one-time repack, sm_100a.
//
// quantize: the reference's k_quantize (backend/ref/kernels.c:24-58,
// contract backend/kernels.h:47-58). For each column t and block b of qb
// inputs:
//
//   a block holding a NaN or an infinity, or whose amax = max |x| is below
//   2^-121:                                    q = 0, d = 0
//   otherwise:  d = amax / 127,  id = 127 / amax,  q = (int8)rint(x * id)
//
// each operation rounded once in the mode RM (rint rounds to an integer in
// that mode). The maximum is exact in any order, so the reduction's shape
// is free. HBM-bound: 4 bytes read and 1 + 4/qb written an input.
//
// Layout of the work: a block of 32 is 4 threads of 8 inputs (two 16-byte
// loads each), a block of 64 8 threads of 8, so a warp takes 8 or 4 blocks
// at once (and two such chunks a pass, their loads in flight together) and
// reduces each within its thread group by shuffles; wider blocks (qb = n, up
// to 16384) take a warp each, in two passes over the block. Warps stride over
// the blocks, the grid one wave of the CTAs an SM holds.
//
// repack: PK_Q8 panels (core/pkf.h:28-41: 16 rows by 4 inputs in 64-byte
// groups) to plain rows of n bytes, which the product's TMA tiles read.

#include "pkb_device.cuh"
#include "pkb_internal.h"
#include "pkb_vmath.cuh"

namespace pkb {

namespace {

__device__ __forceinline__ float4 load4(const float* p, bool vec) {
    if (vec) return __ldg(reinterpret_cast<const float4*>(p));
    return make_float4(__ldg(p), __ldg(p + 1), __ldg(p + 2), __ldg(p + 3));
}

__device__ __forceinline__ bool finite4(float4 v) {
    return isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w);
}

__device__ __forceinline__ float amax4(float4 v) {
    return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
}

// Blocks of QB = 32 or 64 inputs, E inputs (E / 4 16-byte loads) a thread,
// QB / E threads a block. A warp takes 32 / (QB / E) blocks a chunk and U
// chunks a pass, loading all of them before reducing any: several 16-byte
// loads in flight a thread keep HBM busy (measured on B200 at qb 32, grid of
// eight CTAs an SM: one a thread 2.7 TB/s, four 3.6-4.0, eight 4.4-5.1; with
// the grid one resident wave, four loads of two chunks beat eight of four,
// whose registers leave fewer CTAs on an SM). IDX is the index type,
// 32-bit wherever T * n / qb fits. SILU: each input goes through the
// reference's SiLU first (siluq_tile, core/encoder.c:150-158: k_silu on the
// row, then pk_quant_part).
template <int RM, int QB, int E, int U, typename IDX, bool SILU>
__device__ __forceinline__ void quantize_narrow_body(int8_t* __restrict__ q, float* __restrict__ d,
                                                     const float* __restrict__ x, size_t xs, IDX nb, IDX total,
                                                     bool vec) {
    constexpr uint32_t G = QB / E;         // threads a block
    constexpr uint32_t PER_WARP = 32 / G;  // blocks a warp chunk
    constexpr int V = E / 4;               // 16-byte loads a thread and block
    const uint32_t lane = threadIdx.x & 31, lg = lane % G;
    const IDX nwarps = static_cast<IDX>(gridDim.x) * (blockDim.x / 32);
    const IDX warp0 = static_cast<IDX>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
    const IDX chunks = (total + PER_WARP - 1) / PER_WARP;
    for (IDX c0 = warp0; c0 < chunks; c0 += nwarps * U) {  // warp-uniform
        float4 v[U][V];
        IDX t[U], b[U];
        bool valid[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const IDX blk = (c0 + u * nwarps) * PER_WARP + lane / G;
            valid[u] = blk < total;
            t[u] = valid[u] ? blk / nb : 0;
            b[u] = valid[u] ? blk - t[u] * nb : 0;
            const float* xp = x + static_cast<size_t>(t[u]) * xs + static_cast<size_t>(b[u]) * QB + E * lg;
#pragma unroll
            for (int e = 0; e < V; e++) v[u][e] = valid[u] ? load4(xp + 4 * e, vec) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if constexpr (SILU) {
            // the thread's U * V * 4 inputs through SiLU as one batch
            float xs4[U * V * 4];
#pragma unroll
            for (int u = 0; u < U; u++)
#pragma unroll
                for (int e = 0; e < V; e++) {
                    float* o = xs4 + 4 * (u * V + e);
                    o[0] = v[u][e].x;
                    o[1] = v[u][e].y;
                    o[2] = v[u][e].z;
                    o[3] = v[u][e].w;
                }
            silu_batch<RM, U * V * 4>(xs4);
#pragma unroll
            for (int u = 0; u < U; u++)
#pragma unroll
                for (int e = 0; e < V; e++) {
                    const float* o = xs4 + 4 * (u * V + e);
                    v[u][e] = make_float4(o[0], o[1], o[2], o[3]);
                }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            // the block's largest |x| bits: its amax, or a non-finite value
            uint32_t m = 0;
#pragma unroll
            for (int e = 0; e < V; e++)
                m = max(m, max(max(abs_bits(v[u][e].x), abs_bits(v[u][e].y)),
                               max(abs_bits(v[u][e].z), abs_bits(v[u][e].w))));
#pragma unroll
            for (int off = G / 2; off >= 1; off >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, off));
            if (!valid[u]) continue;
            uint32_t packed[V];
#pragma unroll
            for (int e = 0; e < V; e++) packed[e] = 0;
            float scale = 0.0f;
            if (block_scaled(m)) {
                const float amax = __uint_as_float(m);
                scale = div_r<RM>(amax, 127.0f);
                const float id = div_r<RM>(127.0f, amax);
#pragma unroll
                for (int e = 0; e < V; e++) packed[e] = quant4<RM>(v[u][e], id);
            }
            const size_t row = static_cast<size_t>(t[u]);
            int8_t* qo = q + row * (nb * QB) + static_cast<size_t>(b[u]) * QB + E * lg;  // E-byte aligned
#pragma unroll
            for (int e = 0; e + 1 < V; e += 2)
                *reinterpret_cast<uint2*>(qo + 4 * e) = make_uint2(packed[e], packed[e + 1]);
            if constexpr (V & 1) *reinterpret_cast<uint32_t*>(qo + 4 * (V - 1)) = packed[V - 1];
            if (lg == 0) d[row * nb + b[u]] = scale;
        }
    }
}

// chunks a pass for the SiLU form: fewer than the plain form's four, for
// registers (its batch of values is live across the sigmoid)
#ifndef PKB_SILU_U
#define PKB_SILU_U 2
#endif
// chunks a pass for the plain form (measured on B200 at T 11521, qb 32, with
// the grid one wave of resident CTAs: two 11.9 / 40.4 us for n 1024 / 4096,
// four 13.5 / 42.3, eight 20.9 / 82.0 with one CTA an SM)
#ifndef PKB_Q_U
#define PKB_Q_U 2
#endif

template <int RM, int QB, int E, bool SILU>
__global__ void __launch_bounds__(256) quantize_narrow(int8_t* __restrict__ q, float* __restrict__ d,
                                                       const float* __restrict__ x, size_t xs, uint32_t T,
                                                       uint32_t n, bool vec) {
    pdl_trigger();
    pdl_wait();
    constexpr int U = SILU ? PKB_SILU_U : PKB_Q_U;
    const uint32_t nb = n / QB;
    const uint64_t total = static_cast<uint64_t>(T) * nb;
    if (total <= 0xFFFFFFF0ull)
        quantize_narrow_body<RM, QB, E, U, uint32_t, SILU>(q, d, x, xs, nb, static_cast<uint32_t>(total), vec);
    else
        quantize_narrow_body<RM, QB, E, U, uint64_t, SILU>(q, d, x, xs, nb, total, vec);
}

#ifndef PKB_Q64_E
#define PKB_Q64_E 8
#endif

// Blocks of any multiple of 32 inputs, a warp each.
template <int RM>
__global__ void __launch_bounds__(256) quantize_wide(int8_t* __restrict__ q, float* __restrict__ d,
                                                     const float* __restrict__ x, size_t xs, uint32_t T,
                                                     uint32_t n, uint32_t qb, bool vec) {
    pdl_trigger();
    pdl_wait();
    const uint32_t nb = n / qb;
    const size_t total = static_cast<size_t>(T) * nb;
    const uint32_t lane = threadIdx.x & 31;
    const size_t warp0 = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
    const size_t nwarps = static_cast<size_t>(gridDim.x) * blockDim.x / 32;
    for (size_t blk = warp0; blk < total; blk += nwarps) {  // warp-uniform
        const size_t t = blk / nb, b = blk % nb;
        const float* v = x + t * xs + b * qb;
        float amax = 0.0f;
        uint32_t bad = 0;
        for (uint32_t i = 4 * lane; i < qb; i += 128) {
            const float4 f = load4(v + i, vec);
            amax = fmaxf(amax, amax4(f));
            bad |= finite4(f) ? 0u : 1u;
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
            bad |= __shfl_xor_sync(0xffffffffu, bad, off);
        }
        int8_t* qo = q + t * n + b * qb;
        const bool zero = bad || !(amax >= 0x1p-121f);
        const float id = zero ? 0.0f : div_r<RM>(127.0f, amax);
        for (uint32_t i = 4 * lane; i < qb; i += 128)
            *reinterpret_cast<uint32_t*>(qo + i) = zero ? 0u : quant4<RM>(load4(v + i, vec), id);
        if (lane == 0) d[t * nb + b] = zero ? 0.0f : div_r<RM>(amax, 127.0f);
    }
}

// CTAs of a narrow instance resident on an SM at once (its registers decide),
// asked once: the grid is one wave of them, each warp striding over the rest
// of the blocks (measured on B200: a grid of eight 256-thread CTAs an SM ran
// as 2.7 waves of the three that fit, and the partial last wave cost 5-20 %)
template <int RM, int QB, int E, bool SILU>
size_t narrow_resident() {
    static const size_t r = [] {
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, quantize_narrow<RM, QB, E, SILU>, 256, 0) !=
                cudaSuccess ||
            per_sm < 1)
            per_sm = 1;
        return static_cast<size_t>(per_sm);
    }();
    return r;
}

template <int RM, bool SILU>
size_t resident(uint32_t qb, bool q8) {
    // the SiLU form is instruction-bound and keeps eight CTAs an SM (one
    // resident wave measured 71.4 us against 67.8-69.5 on n 4096)
    if constexpr (SILU) return 8;
    if (qb == 32) return q8 ? narrow_resident<RM, 32, 8, SILU>() : narrow_resident<RM, 32, 4, SILU>();
    if (qb == 64) return q8 ? narrow_resident<RM, 64, PKB_Q64_E, SILU>() : narrow_resident<RM, 64, 4, SILU>();
    return 8;  // the wide form: a warp a block, eight CTAs an SM
}

template <int RM, bool SILU>
cudaError_t quantize_rm(int8_t* q, float* d, const float* x, size_t xs, uint32_t T, uint32_t n, uint32_t qb,
                        int num_sms, cudaStream_t stream) {
    const bool vec = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (xs % 4 == 0);
    const size_t blocks = static_cast<size_t>(T) * (n / qb);
    // eight inputs a thread store 8 bytes of q at once: only where q is 8-byte
    // aligned (the interface asks 4), else four inputs and 4-byte stores
    const bool q8 = reinterpret_cast<uintptr_t>(q) % 8 == 0;
    const int e = qb == 32 ? (q8 ? 8 : 4) : qb == 64 ? (q8 ? PKB_Q64_E : 4) : 0;
    // blocks a 256-thread CTA takes a pass: 8 warps x U chunks x blocks a chunk
    const size_t per_cta = e ? 8 * (SILU ? PKB_SILU_U : PKB_Q_U) * (32 / (qb / e)) : 8;
    size_t grid = (blocks + per_cta - 1) / per_cta;
    const size_t cap = static_cast<size_t>(num_sms) * resident<RM, SILU>(qb, q8);
    if (grid > cap) grid = cap;
    if (grid == 0) grid = 1;
    const dim3 g(static_cast<unsigned>(grid)), b(256);
    if (qb == 32)
        return q8 ? launch_pdl(quantize_narrow<RM, 32, 8, SILU>, g, b, 0, stream, q, d, x, xs, T, n, vec)
                  : launch_pdl(quantize_narrow<RM, 32, 4, SILU>, g, b, 0, stream, q, d, x, xs, T, n, vec);
    else if (qb == 64)
        return q8 ? launch_pdl(quantize_narrow<RM, 64, PKB_Q64_E, SILU>, g, b, 0, stream, q, d, x, xs, T, n, vec)
                  : launch_pdl(quantize_narrow<RM, 64, 4, SILU>, g, b, 0, stream, q, d, x, xs, T, n, vec);
    else if constexpr (SILU)
        return cudaErrorInvalidValue;  // the encoder's blocks are 32 or 64 (qb(), core/encoder.c:56)
    else
        return launch_pdl(quantize_wide<RM>, g, b, 0, stream, q, d, x, xs, T, n, qb, vec);
}

__global__ void __launch_bounds__(256) repack_q8(uint32_t* __restrict__ dst, const uint32_t* __restrict__ src,
                                                 uint32_t rows, uint32_t n) {
    pdl_trigger();
    pdl_wait();
    // word (r, k/4) of the plain rows from word ((r/16)*(n/4) + k/4)*16 + r%16
    // of the panels
    const uint32_t n4 = n / 4;
    const size_t total = static_cast<size_t>(rows) * n4;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t r = i / n4, k4 = i % n4;
        dst[i] = __ldg(src + ((r / 16) * n4 + k4) * 16 + (r % 16));
    }
}

}  // namespace

cudaError_t launch_quantize(int8_t* q, float* d, const float* x, size_t xs, uint32_t T, uint32_t n, uint32_t qb,
                            int rmode, int num_sms, cudaStream_t stream) {
    switch (rmode) {
    case 1: return quantize_rm<1, false>(q, d, x, xs, T, n, qb, num_sms, stream);
    case 2: return quantize_rm<2, false>(q, d, x, xs, T, n, qb, num_sms, stream);
    case 3: return quantize_rm<3, false>(q, d, x, xs, T, n, qb, num_sms, stream);
    default: return quantize_rm<0, false>(q, d, x, xs, T, n, qb, num_sms, stream);
    }
}

cudaError_t launch_silu_quantize(int8_t* q, float* d, const float* u, size_t us, uint32_t T, uint32_t n,
                                 uint32_t qb, int rmode, int num_sms, cudaStream_t stream) {
    switch (rmode) {
    case 1: return quantize_rm<1, true>(q, d, u, us, T, n, qb, num_sms, stream);
    case 2: return quantize_rm<2, true>(q, d, u, us, T, n, qb, num_sms, stream);
    case 3: return quantize_rm<3, true>(q, d, u, us, T, n, qb, num_sms, stream);
    default: return quantize_rm<0, true>(q, d, u, us, T, n, qb, num_sms, stream);
    }
}

cudaError_t launch_repack_q8(int8_t* wpack, const int8_t* w_pk, uint32_t rows, uint32_t n, int num_sms,
                             cudaStream_t stream) {
    const size_t words = static_cast<size_t>(rows) * (n / 4);
    size_t grid = (words + 255) / 256;
    const size_t cap = static_cast<size_t>(num_sms) * 16;
    if (grid > cap) grid = cap;
    if (grid == 0) grid = 1;
    return launch_pdl(repack_q8, dim3(static_cast<unsigned>(grid)), dim3(256), 0, stream,
                      reinterpret_cast<uint32_t*>(wpack), reinterpret_cast<const uint32_t*>(w_pk), rows, n);
}

// Every narrow instance's residency asked once, at the device's set-up
// (outside any stream capture, before the first launch needs it).
void prepare_quantize() {
    for (uint32_t qb : {32u, 64u})
        for (bool q8 : {false, true}) {
            resident<0, false>(qb, q8);
            resident<1, false>(qb, q8);
            resident<2, false>(qb, q8);
            resident<3, false>(qb, q8);
        }
}

}  // namespace pkb
