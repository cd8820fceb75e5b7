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
    const float n = rint_r<RM>(mul_r<RM>(x, VM_LOG2E));
    float r = fma_r<RM>(n, -VM_LN2_HI, x);
    r = fma_r<RM>(n, -VM_LN2_LO, r);
    float p = VM_EXP_C6;
    p = fma_r<RM>(p, r, VM_EXP_C5);
    p = fma_r<RM>(p, r, VM_EXP_C4);
    p = fma_r<RM>(p, r, VM_EXP_C3);
    p = fma_r<RM>(p, r, VM_EXP_C2);
    p = fma_r<RM>(p, r, 1.0f);
    p = fma_r<RM>(p, r, 1.0f);
    return mul_r<RM>(p, pow2i(__float2int_rz(n)));  // n is integral: the conversion is exact
}

// pk_sigmoidf (core/vmath.h:149-151): 1 / (1 + e^-x)
template <int RM>
__device__ __forceinline__ float pk_sigmoid(float x) {
    return div_r<RM>(1.0f, add_r<RM>(1.0f, pk_exp<RM>(-x)));
}

// SiLU as the reference's k_silu writes it (backend/ref/kernels.c:149-151)
template <int RM>
__device__ __forceinline__ float pk_silu(float x) {
    return mul_r<RM>(x, pk_sigmoid<RM>(x));
}

}  // namespace pkb
