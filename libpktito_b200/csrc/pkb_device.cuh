// Device-side building blocks for the sm_100a kernels of libpktito_b200:
// IEEE operations in a rounding mode chosen at compile time, mbarrier waits
// that give up after a bounded time, TMA tile loads, and the tcgen05
// (5th-generation tensor core) instructions, as inline PTX.
//
// Nothing here uses a cluster multicast form: every TMA load names this
// CTA's own shared memory and this GPU's own global memory.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace pkb {

// ---------------------------------------------------------------- rounding --
//
// The reference's arithmetic runs in the caller's rounding mode
// (fesetround); each kernel is instantiated for the four modes, RM being
// PKB_RN/RD/RU/RZ. Every operation below is one correctly rounded IEEE
// operation with subnormals kept (the library is built with -ftz=false).

template <int RM> __device__ __forceinline__ float fma_r(float a, float b, float c);
template <> __device__ __forceinline__ float fma_r<0>(float a, float b, float c) { return __fmaf_rn(a, b, c); }
template <> __device__ __forceinline__ float fma_r<1>(float a, float b, float c) { return __fmaf_rd(a, b, c); }
template <> __device__ __forceinline__ float fma_r<2>(float a, float b, float c) { return __fmaf_ru(a, b, c); }
template <> __device__ __forceinline__ float fma_r<3>(float a, float b, float c) { return __fmaf_rz(a, b, c); }

template <int RM> __device__ __forceinline__ float mul_r(float a, float b);
template <> __device__ __forceinline__ float mul_r<0>(float a, float b) { return __fmul_rn(a, b); }
template <> __device__ __forceinline__ float mul_r<1>(float a, float b) { return __fmul_rd(a, b); }
template <> __device__ __forceinline__ float mul_r<2>(float a, float b) { return __fmul_ru(a, b); }
template <> __device__ __forceinline__ float mul_r<3>(float a, float b) { return __fmul_rz(a, b); }

template <int RM> __device__ __forceinline__ float add_r(float a, float b);
template <> __device__ __forceinline__ float add_r<0>(float a, float b) { return __fadd_rn(a, b); }
template <> __device__ __forceinline__ float add_r<1>(float a, float b) { return __fadd_rd(a, b); }
template <> __device__ __forceinline__ float add_r<2>(float a, float b) { return __fadd_ru(a, b); }
template <> __device__ __forceinline__ float add_r<3>(float a, float b) { return __fadd_rz(a, b); }

template <int RM> __device__ __forceinline__ float div_r(float a, float b);
template <> __device__ __forceinline__ float div_r<0>(float a, float b) { return __fdiv_rn(a, b); }
template <> __device__ __forceinline__ float div_r<1>(float a, float b) { return __fdiv_rd(a, b); }
template <> __device__ __forceinline__ float div_r<2>(float a, float b) { return __fdiv_ru(a, b); }
template <> __device__ __forceinline__ float div_r<3>(float a, float b) { return __fdiv_rz(a, b); }

// int -> float, rounded in the mode (exact below 2^24)
template <int RM> __device__ __forceinline__ float i2f_r(int a);
template <> __device__ __forceinline__ float i2f_r<0>(int a) { return __int2float_rn(a); }
template <> __device__ __forceinline__ float i2f_r<1>(int a) { return __int2float_rd(a); }
template <> __device__ __forceinline__ float i2f_r<2>(int a) { return __int2float_ru(a); }
template <> __device__ __forceinline__ float i2f_r<3>(int a) { return __int2float_rz(a); }

// float -> int, rounded to an integer in the mode: rintf's rounding in
// that mode, then C's conversion to int
template <int RM> __device__ __forceinline__ int f2i_r(float a);
template <> __device__ __forceinline__ int f2i_r<0>(float a) { return __float2int_rn(a); }
template <> __device__ __forceinline__ int f2i_r<1>(float a) { return __float2int_rd(a); }
template <> __device__ __forceinline__ int f2i_r<2>(float a) { return __float2int_ru(a); }
template <> __device__ __forceinline__ int f2i_r<3>(float a) { return __float2int_rz(a); }

// An int32 block sum as a float, exactly, for |s| < 2^22: the integer plus
// 0x4B400000 is the float 1.5 * 2^23 + s, and subtracting 1.5 * 2^23 is
// exact. The subtraction is rounded to nearest whatever the mode, so that a
// zero sum is +0 as (float)0 is (x - x is -0 rounding downward).
__device__ __forceinline__ float sum_to_float_exact(uint32_t s) {
    return __fsub_rn(__uint_as_float(s + 0x4B400000u), 12582912.0f);
}

// Rounding to an integer by adding 1.5 * 2^23 (RN, RD, RU): for |p| < 2^22
// the sum lies in [2^23, 2^24), where floats are the integers, so the one
// rounding of the addition is rint(p) in the mode (ties to even under RN:
// 1.5 * 2^23 is even), and the sum's bits are 0x4B400000 + rint(p). Exact
// and on the FP32 pipe, where a float-to-int conversion takes the
// quarter-rate conversion pipe. Toward zero the sum would round a negative
// p down, so RZ converts instead.
constexpr float RINT_MAGIC = 12582912.0f;  // 1.5 * 2^23
constexpr uint32_t RINT_MAGIC_BITS = 0x4B400000u;

// One quantized byte, as the low byte of a word: (int8)rint(v * id), rint
// in the mode RM, through int as the reference's (int8_t)rintf(...)
// (backend/ref/kernels.c:24-58); |v * id| <= 127 rounded.
template <int RM>
__device__ __forceinline__ uint32_t quant1(float v, float id) {
    const float p = mul_r<RM>(v, id);
    if constexpr (RM == 3) return static_cast<uint8_t>(static_cast<int8_t>(f2i_r<RM>(p)));
    return __float_as_uint(add_r<RM>(p, RINT_MAGIC));  // low byte: 0x00 + rint(p), two's complement
}

// The low bytes of four words, packed little-endian in that order.
__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// Four quantized bytes, packed little-endian in the inputs' order.
template <int RM>
__device__ __forceinline__ uint32_t quant4(float4 v, float id) {
    return pack_low_bytes(quant1<RM>(v.x, id), quant1<RM>(v.y, id), quant1<RM>(v.z, id), quant1<RM>(v.w, id));
}

// |v|'s bits. For floats of one sign the bits order as the values, and
// every infinity or NaN is above every finite value, so the largest of a
// block's |v| bits is its amax, or at least 0x7F800000 where it holds a
// non-finite value.
__device__ __forceinline__ uint32_t abs_bits(float v) { return __float_as_uint(v) & 0x7FFFFFFFu; }

// Whether a block whose largest |v| bits are m is quantized (finite, amax
// at least 2^-121) or becomes zeros with scale 0.
__device__ __forceinline__ bool block_scaled(uint32_t m) {
    return m < 0x7F800000u && __uint_as_float(m) >= 0x1p-121f;
}

// Two floats in one 64-bit register, for the packed f32x2 instructions of
// sm_100 (one instruction, two independent IEEE operations).
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

// a * b + c on both halves, each rounded once in the mode
template <int RM> __device__ __forceinline__ uint64_t fma2_r(uint64_t a, uint64_t b, uint64_t c);
template <> __device__ __forceinline__ uint64_t fma2_r<0>(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
template <> __device__ __forceinline__ uint64_t fma2_r<1>(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rm.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
template <> __device__ __forceinline__ uint64_t fma2_r<2>(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rp.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
template <> __device__ __forceinline__ uint64_t fma2_r<3>(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rz.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// a + b on both halves, rounded to nearest
__device__ __forceinline__ uint64_t add2_rn(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// a * b and a + b on both halves, each rounded once in the mode RM.
// Measured on B200 (ptxas 12.9): a packed multiply whose result feeds a
// packed add is fused into one packed FMA, explicit rounding and -fmad=false
// notwithstanding, which rounds once where the reference rounds twice. So a
// mul2_r result never goes into an add2_r (or fma2_r's addend); a multiply
// that an add follows is the scalar mul_r (__fmul_rn and its kind are never
// fused).
template <int RM> __device__ __forceinline__ uint64_t mul2_r(uint64_t a, uint64_t b);
template <int RM> __device__ __forceinline__ uint64_t add2_r(uint64_t a, uint64_t b);
#define PKB_F32X2_OP(NAME, OP, RM, RND)                                                 \
    template <> __device__ __forceinline__ uint64_t NAME<RM>(uint64_t a, uint64_t b) { \
        uint64_t r;                                                                       \
        asm(OP "." RND ".f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));                  \
        return r;                                                                         \
    }
PKB_F32X2_OP(mul2_r, "mul", 0, "rn")
PKB_F32X2_OP(mul2_r, "mul", 1, "rm")
PKB_F32X2_OP(mul2_r, "mul", 2, "rp")
PKB_F32X2_OP(mul2_r, "mul", 3, "rz")
PKB_F32X2_OP(add2_r, "add", 0, "rn")
PKB_F32X2_OP(add2_r, "add", 1, "rm")
PKB_F32X2_OP(add2_r, "add", 2, "rp")
PKB_F32X2_OP(add2_r, "add", 3, "rz")
#undef PKB_F32X2_OP

// --------------------------------------------------------------- smem / sync --

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// One try: true once the phase with this parity has completed. The thread
// may be suspended meanwhile, up to the time hint, and resumes when the
// phase completes (measured on B200: a hint lets the waiting threads sleep
// without slowing the barriers' other traffic as a bare try_wait does).
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(0x989680)
        : "memory");
    return ok != 0;
}

// Waits for the phase of `bar` with this parity to complete. Gives up after
// `limit` SM clock cycles, or as soon as another role of the CTA has given
// up (*abort set), and returns false: no wait can hang the GPU.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          long long limit) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (clock64() - t0 > limit) return false;
    }
}

__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// mbar_wait by polling: test_wait never suspends the thread, and the abort
// flag and the clock are read once every 256 tries; the same bounds.
__device__ __forceinline__ bool mbar_poll(uint64_t* bar, uint32_t parity, volatile int* abort, long long limit) {
    if (mbar_test_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (uint32_t i = 0;; i++) {
        if (mbar_test_wait(bar, parity)) return true;
        if ((i & 255) == 255) {
            if (*abort) return false;
            if (clock64() - t0 > limit) return false;
        }
    }
}

// The same wait without the abort flag, still bounded: for a role that has
// given up and must let its own copies or MMAs in flight land before the CTA
// frees its shared memory and TMEM.
__device__ __forceinline__ bool mbar_drain(uint64_t* bar, uint32_t parity, long long limit) {
    const long long t0 = clock64();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (clock64() - t0 > limit) return false;
    }
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// ----------------------------------------------------------------------- TMA --

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// A 2-D tile of `map` at element coordinates (x inner, y outer) into this
// CTA's shared memory, completing as bytes on `bar`. x * element size is a
// multiple of 16 bytes at every call site (x is a multiple of 128 bytes).
__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, void* dst, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// `bytes` (a multiple of 16) from global `src` into this CTA's shared memory
// `dst` (both 16-byte aligned), completing as bytes on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// A 2-D tile of this CTA's shared memory into `map` at element coordinates
// (x inner, y outer), asynchronously, in the thread's current bulk group;
// elements outside the tensor are not written. x * element size is a
// multiple of 16 bytes and both coordinates are non-negative at every call
// site.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
}

// The same for 3-D and 4-D maps (the attention's panels): x is 0 at every
// call site, the other coordinates non-negative.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int x, int y, int z) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
                 : "memory");
}

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int x, int y, int z, int w) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z), "r"(w)
                 : "memory");
}

// Closes the thread's current bulk group of TMA stores.
// Per-thread asynchronous copies into shared memory (LDGSTS): 16 or 4
// bytes, tracked in groups that the copying thread waits for itself (a
// hardware wait, not a poll).
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// all but the newest N groups of this thread's copies have landed
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Waits until the thread's bulk groups have finished reading their shared
// memory (the source may be written again).
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// Waits until the thread's bulk groups have completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA, tensor core) reads of them.
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ----------------------------------------------- programmatic dependent launch --
//
// Kernels of this library are launched with programmatic stream
// serialization: the next kernel in the stream may start as soon as every
// CTA of the current one has called pdl_trigger(), and its CTAs take SMs as
// the current kernel's last CTAs leave. Before it touches global memory a
// kernel calls pdl_wait(), which returns once the preceding kernel has
// completed and its memory operations are visible (at once where there is
// no preceding kernel or the launch did not allow the overlap).

__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ------------------------------------------------------------------- tcgen05 --

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with the 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes
// apart (stride byte offset), version 1 (sm_100), layout SWIZZLE_128B. The
// tile starts 1024-byte aligned; a K step inside the 128-byte row moves the
// start address by its bytes.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);   // start address >> 4, bits 0-13
    d |= static_cast<uint64_t>(1) << 16;                    // leading byte offset (unused when swizzled)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;            // stride byte offset: 8 rows x 128 B
    d |= static_cast<uint64_t>(1) << 46;                    // descriptor version for sm_100
    d |= static_cast<uint64_t>(2) << 61;                    // SWIZZLE_128B
    return d;
}

// Shared-memory matrix descriptor for a K-major operand tile without
// swizzle: 8-row x 16-byte core matrices, `lbo` bytes apart along K and
// `sbo` bytes apart along the rows, version 1 (sm_100), layout SWIZZLE_NONE.
__device__ __forceinline__ uint64_t plain_kmajor_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);   // start address >> 4, bits 0-13
    d |= static_cast<uint64_t>(lbo >> 4) << 16;             // leading byte offset: K neighbours
    d |= static_cast<uint64_t>(sbo >> 4) << 32;             // stride byte offset: 8-row groups
    d |= static_cast<uint64_t>(1) << 46;                    // descriptor version for sm_100
    return d;                                               // layout bits 61-63 = 0: no swizzle
}

// Instruction descriptor of tcgen05.mma.kind::f16 with bf16 A and B and a
// float32 accumulator, both operands K-major, M x N.
__host__ __device__ constexpr uint32_t bf16_instr_desc(uint32_t M, uint32_t N) {
    return (1u << 4)            // D format: F32
           | (1u << 7)          // A: bf16
           | (1u << 10)         // B: bf16
           | ((N >> 3) << 17)   // N / 8
           | ((M >> 4) << 24);  // M / 16
}

// Instruction descriptor of tcgen05.mma.kind::i8: signed A and B, int32
// accumulator, both operands K-major, M x N.
__host__ __device__ constexpr uint32_t i8_instr_desc(uint32_t M, uint32_t N) {
    return (2u << 4)            // D format: S32
           | (1u << 7)          // A: signed 8-bit
           | (1u << 10)         // B: signed 8-bit
           | ((N >> 3) << 17)   // N / 8
           | ((M >> 4) << 24);  // M / 16
}

// D[tmem] (+)= A[smem] * B[smem]^T, one K=32 step, issued by one thread.
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T for bf16 A and B, one K=16 step, float32
// accumulator, issued by one thread.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued before has
// completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 TMEM lanes (this warp's quarter) x 32 consecutive 32-bit columns into
// 32 registers per thread: thread i gets lane (base lane + i).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

// The same for 16 consecutive columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// 32 lanes x 16 columns of TMEM set to the same 32-bit value v.
__device__ __forceinline__ void tmem_st_32x32b_x16_fill(uint32_t taddr, uint32_t v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr),
        "r"(v)
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// The wait, naming the registers a tcgen05.ld filled as read-written here:
// the compiler sees the load's outputs as defined when the load is issued,
// so without this it could move their first use above the wait.
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
}

// No instruction: names 32 registers a tcgen05.ld filled as read-written
// here, after a wait that covered that load (tcgen05.wait::ld waits for all
// of the thread's loads), so the compiler keeps their first use below it.
__device__ __forceinline__ void tmem_ld_settled(uint32_t (&r)[32]) {
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

// The same for the 32 registers two x16 loads filled.
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

// Bits of the device-side error word (include/pktito_b200.h, pkb_device_errors)
enum : uint32_t { PKB_DEVERR_TIMEOUT = 1u, PKB_DEVERR_ARGS = 2u };

}  // namespace pkb
