// The reference's own exp and sigmoid (core/vmath.h), on the device,
// operation for operation.
//
// libpktito defines these functions by their code, not by their values: a
// minimax polynomial of its own fit, every step one IEEE operation, so that
// every backend computes the same bits (its tests hold them to that). Here
// each step is the same operation rounded once in the mode RM, the mode the
// caller's arithmetic runs in. These are the reference's definitions, not
// CUDA's math library; the constants below are its constants, which define
// the function and so have to be the same.
#pragma once

#include "pkb_device.cuh"

namespace pkb {

// x = n ln2 + r, ln2 split so that n * ln2 is exact (core/vmath.h:93-97)
constexpr float VM_LOG2E = 0x1.715476p+0f;
constexpr float VM_LN2_HI = 0x1.62e430p-1f;
constexpr float VM_LN2_LO = -0x1.05c610p-29f;
// exp(r) on [-ln2/2, ln2/2] = 1 + r + c2 r^2 + ... + c6 r^6 (core/vmath.h:99-106)
constexpr float VM_EXP_C2 = 0x1.fffffap-2f;
constexpr float VM_EXP_C3 = 0x1.55540ap-3f;
constexpr float VM_EXP_C4 = 0x1.55589ap-5f;
constexpr float VM_EXP_C5 = 0x1.126d0cp-7f;
constexpr float VM_EXP_C6 = 0x1.6ab980p-10f;
// the argument's clamp, keeping 2^n a normal float (core/vmath.h:118-124)
constexpr float VM_EXP_LO = -87.0f;
constexpr float VM_EXP_HI = 88.0f;

// rintf in the mode: the nearest integral float, ties to even under RN,
// else rounded down, up or toward zero
template <int RM> __device__ __forceinline__ float rint_r(float x);
template <> __device__ __forceinline__ float rint_r<0>(float x) { return rintf(x); }
template <> __device__ __forceinline__ float rint_r<1>(float x) { return floorf(x); }
template <> __device__ __forceinline__ float rint_r<2>(float x) { return ceilf(x); }
template <> __device__ __forceinline__ float rint_r<3>(float x) { return truncf(x); }

template <int RM> __device__ __forceinline__ float sqrt_r(float x);
template <> __device__ __forceinline__ float sqrt_r<0>(float x) { return __fsqrt_rn(x); }
template <> __device__ __forceinline__ float sqrt_r<1>(float x) { return __fsqrt_rd(x); }
template <> __device__ __forceinline__ float sqrt_r<2>(float x) { return __fsqrt_ru(x); }
template <> __device__ __forceinline__ float sqrt_r<3>(float x) { return __fsqrt_rz(x); }

// 1 / y rounded once in the mode: the correctly rounded reciprocal is the
// correctly rounded quotient 1 / y, for every y
template <int RM> __device__ __forceinline__ float rcp_r(float y);
template <> __device__ __forceinline__ float rcp_r<0>(float y) { return __frcp_rn(y); }
template <> __device__ __forceinline__ float rcp_r<1>(float y) { return __frcp_rd(y); }
template <> __device__ __forceinline__ float rcp_r<2>(float y) { return __frcp_ru(y); }
template <> __device__ __forceinline__ float rcp_r<3>(float y) { return __frcp_rz(y); }

// 1 / y for y in [1, 2^126) (where the reciprocal is normal), rounded once
// in the mode RM, without a branch: Markstein's method (P. Markstein, "IA-64
// and Elementary Functions", Prentice Hall 2000, ch. 8). From the hardware's
// approximation r = rcp.approx(y), NEWTON steps r + r (1 - y r) in
// round-to-nearest fused operations, then the same step once more with its
// one rounding in the mode: the residual 1 - y r is exact in an FMA, so the
// last step is the exact reciprocal's rounding wherever r is close enough.
// Measured exhaustively (pkb_rcp_selftest): with one Newton step it is the
// correctly rounded reciprocal for every float of [1, 2^126) in all four
// modes; for y of [2^126, 2^128), whose reciprocal is subnormal, the last
// step's error (about y (r - 1/y)^2, near 2^-171) can exceed the distance
// to a rounding midpoint of the subnormal grid, and 5 floats round wrong
// under RN, so those take the correctly rounded division (rcp_batch).
template <int RM, int NEWTON>
__device__ __forceinline__ float rcp_markstein(float y) {
    float r;
    asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(y));
#pragma unroll
    for (int i = 0; i < NEWTON; i++) r = __fmaf_rn(r, __fmaf_rn(-y, r, 1.0f), r);
    return fma_r<RM>(r, __fmaf_rn(-y, r, 1.0f), r);
}

#ifndef PKB_RCP_NEWTON
#define PKB_RCP_NEWTON 1
#endif

// a - b, IEEE's subtraction (a + (-b), rounded once in the mode)
template <int RM> __device__ __forceinline__ float sub_r(float a, float b) { return add_r<RM>(a, -b); }

// pk_pow2i (core/vmath.h:126-132): 2^n for n in [-126, 127], the float whose exponent field is n + 127
__device__ __forceinline__ float pow2i(int n) { return __uint_as_float(static_cast<uint32_t>(n + 127) << 23); }

// pk_expf (core/vmath.h:134-147): clamp (a NaN becomes the low end, as
// fmaxf returns its other operand), n = rint(x log2e), r = x - n ln2 in
// two fused steps, the polynomial by Horner in fused steps, times 2^n.
template <int RM>
__device__ __forceinline__ float pk_exp(float x) {
    x = fminf(fmaxf(x, VM_EXP_LO), VM_EXP_HI);
    const float t = mul_r<RM>(x, VM_LOG2E);  // in [-125.6, 127]
    float n;
    int ni;
    if constexpr (RM == 3) {
        n = rint_r<RM>(t);
        ni = __float2int_rz(n);  // n is integral: the conversion is exact
    } else {
        // rint(t) by the 1.5 * 2^23 addition (pkb_device.cuh): the sum is
        // rint(t) + 1.5 * 2^23, its bits 0x4B400000 + rint(t)
        const float y = add_r<RM>(t, RINT_MAGIC);
        n = y - RINT_MAGIC;  // exact
        ni = static_cast<int>(__float_as_uint(y) - RINT_MAGIC_BITS);
    }
    float r = fma_r<RM>(n, -VM_LN2_HI, x);
    r = fma_r<RM>(n, -VM_LN2_LO, r);
    float p = VM_EXP_C6;
    p = fma_r<RM>(p, r, VM_EXP_C5);
    p = fma_r<RM>(p, r, VM_EXP_C4);
    p = fma_r<RM>(p, r, VM_EXP_C3);
    p = fma_r<RM>(p, r, VM_EXP_C2);
    p = fma_r<RM>(p, r, 1.0f);
    p = fma_r<RM>(p, r, 1.0f);
    return mul_r<RM>(p, pow2i(ni));
}

// The sigmoid's denominators 1 + e^-a and 1 + e^-b, pk_expf's operations on
// two values at once: the fused multiply-adds (the reduction's two, Horner's
// six) and the exact subtraction on pairs (f32x2), the multiplies that an
// add follows one at a time (a packed multiply feeding a packed add would be
// fused, pkb_device.cuh). Bit for bit pk_expf's on each; toward zero each
// goes through pk_exp.
template <int RM>
__device__ __forceinline__ void sigmoid_den2(float a, float b, float& da, float& db) {
    if constexpr (RM == 3) {
        da = add_r<RM>(1.0f, pk_exp<RM>(-a));
        db = add_r<RM>(1.0f, pk_exp<RM>(-b));
    } else {
        const float xa = fminf(fmaxf(-a, VM_EXP_LO), VM_EXP_HI), xb = fminf(fmaxf(-b, VM_EXP_LO), VM_EXP_HI);
        const float ya = add_r<RM>(mul_r<RM>(xa, VM_LOG2E), RINT_MAGIC);
        const float yb = add_r<RM>(mul_r<RM>(xb, VM_LOG2E), RINT_MAGIC);
        const uint64_t n = add2_r<RM>(pack2(ya, yb), pack2(-RINT_MAGIC, -RINT_MAGIC));  // exact
        uint64_t r = fma2_r<RM>(n, pack2(-VM_LN2_HI, -VM_LN2_HI), pack2(xa, xb));
        r = fma2_r<RM>(n, pack2(-VM_LN2_LO, -VM_LN2_LO), r);
        uint64_t p = fma2_r<RM>(pack2(VM_EXP_C6, VM_EXP_C6), r, pack2(VM_EXP_C5, VM_EXP_C5));
        p = fma2_r<RM>(p, r, pack2(VM_EXP_C4, VM_EXP_C4));
        p = fma2_r<RM>(p, r, pack2(VM_EXP_C3, VM_EXP_C3));
        p = fma2_r<RM>(p, r, pack2(VM_EXP_C2, VM_EXP_C2));
        p = fma2_r<RM>(p, r, pack2(1.0f, 1.0f));
        p = fma2_r<RM>(p, r, pack2(1.0f, 1.0f));
        float pa, pb;
        unpack2(p, pa, pb);
        const int na = static_cast<int>(__float_as_uint(ya) - RINT_MAGIC_BITS);
        const int nb = static_cast<int>(__float_as_uint(yb) - RINT_MAGIC_BITS);
        da = add_r<RM>(1.0f, mul_r<RM>(pa, pow2i(na)));
        db = add_r<RM>(1.0f, mul_r<RM>(pb, pow2i(nb)));
    }
}

// 1 / den[i] (each at least 1) for a thread's batch of N (even), each
// rounded once in the mode RM: Markstein's method on pairs (rcp_markstein,
// its steps as f32x2 FMAs) unless a value of the batch on any active lane
// is 2^126 or more (a subnormal reciprocal, from an input below about
// -87.3); then the whole warp takes the correctly rounded division for the
// batch. One vote a batch keeps the branch uniform across the warp and out
// of the batch's arithmetic.
template <int RM, int N>
__device__ __forceinline__ void rcp_batch(const float (&den)[N], float (&rec)[N]) {
    static_assert(N % 2 == 0, "pairs");
    float big = den[0];
#pragma unroll
    for (int i = 1; i < N; i++) big = fmaxf(big, den[i]);
    if (__any_sync(__activemask(), big >= 0x1p126f)) {
#pragma unroll
        for (int i = 0; i < N; i++) rec[i] = rcp_r<RM>(den[i]);
        return;
    }
    // every value below 2^126: every reciprocal normal, so the approximation
    // may flush subnormals (.ftz: none arise), which spares its scaling
#pragma unroll
    for (int i = 0; i < N; i += 2) {
        float xa, xb;
        asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(xa) : "f"(den[i]));
        asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(xb) : "f"(den[i + 1]));
        const uint64_t nd = pack2(-den[i], -den[i + 1]), one = pack2(1.0f, 1.0f);
        uint64_t r = pack2(xa, xb);
#pragma unroll
        for (int k = 0; k < PKB_RCP_NEWTON; k++) r = fma2_r<0>(r, fma2_r<0>(nd, r, one), r);
        r = fma2_r<RM>(r, fma2_r<0>(nd, r, one), r);
        unpack2(r, rec[i], rec[i + 1]);
    }
}

// sigmoid(x[i]) for a batch (pk_sigmoidf, core/vmath.h:149-151)
template <int RM, int N>
__device__ __forceinline__ void sigmoid_batch(const float (&x)[N], float (&s)[N]) {
    float den[N];
#pragma unroll
    for (int i = 0; i < N; i += 2) sigmoid_den2<RM>(x[i], x[i + 1], den[i], den[i + 1]);
    rcp_batch<RM, N>(den, s);
}

// x[i] * sigmoid(x[i]) in place for a batch (k_silu, backend/ref/kernels.c:149-151)
template <int RM, int N>
__device__ __forceinline__ void silu_batch(float (&x)[N]) {
    float s[N];
    sigmoid_batch<RM, N>(x, s);
#pragma unroll
    for (int i = 0; i < N; i++) x[i] = mul_r<RM>(x[i], s[i]);
}

// pk_sigmoidf (core/vmath.h:149-151): 1 / (1 + e^-x)
template <int RM>
__device__ __forceinline__ float pk_sigmoid(float x) {
    const float y = add_r<RM>(1.0f, pk_exp<RM>(-x));
    const float den[2] = {y, y};
    float rec[2];
    rcp_batch<RM, 2>(den, rec);
    return rec[0];
}

// SiLU as the reference's k_silu writes it (backend/ref/kernels.c:149-151)
template <int RM>
__device__ __forceinline__ float pk_silu(float x) {
    return mul_r<RM>(x, pk_sigmoid<RM>(x));
}

}  // namespace pkb
