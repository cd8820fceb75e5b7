/* The libpktito backend table, declared for building the cuda-b200 backend
 * outside the reference's tree.
 *
 * A backend of libpktito exports one `const pk_kernels` whose layout the
 * reference fixes in backend/kernels.h:41-45 (pk_act), :195-199 (pk_fft)
 * and :242-278 (pk_kernels). This header declares the same three types,
 * member for member in the same order, so that the table libpktito_b200
 * exports can be linked into the reference unchanged. oracle/abi_offsets.c,
 * compiled once against this header and once against the reference's,
 * checks that every size and member offset agrees (tests/test_abi.py).
 *
 * Built inside the reference's tree (backend/cuda-b200/, with
 * -DPK_CUDA_B200_IN_TREE), the backend includes the reference's own
 * kernels.h instead and this file is not used.
 */
#ifndef PK_KERNELS_ABI_H
#define PK_KERNELS_ABI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* T columns of int8 activations: column t is q + t*n, with n/qb block
 * scales at d + t*(n/qb). */
typedef struct {
    int8_t *q;
    float *d;
    uint32_t n, qb, T;
} pk_act;

/* What an STFT kernel is given of a model's FFT (off the int8 path; here
 * only so the table's stft member has its type). */
typedef struct {
    uint32_t n;
    const float *window, *fcos, *fsin;
    const uint16_t *rev;
} pk_fft;

/* One backend: its name as PKTITO_KERNELS spells it, a description, the
 * CPU features it needs (NULL-ended), whether the reference's picker times
 * it against the next backend, then one function per kernel. */
typedef struct {
    const char *id;
    const char *name;
    const char *const *needs;
    int competes;
    void (*quantize)(pk_act *a, const float *x, size_t xs);
    void (*gemm_q8)(float *out, size_t os, const int8_t *w, const float *ws, const float *bias,
                    uint32_t rows, const pk_act *a, int add);
    void (*gemm_f32)(float *out, size_t os, const float *w, uint32_t ld, uint32_t rows,
                     uint32_t n, const float *x, size_t xs, uint32_t T,
                     const float *bias, size_t bs, int relu);
    void (*layernorm)(float *out, size_t os, const float *x, size_t xs, uint32_t T, uint32_t n,
                      const float *w, const float *b, float eps);
    void (*softmax)(float *x, uint32_t n, float scale);
    void (*silu)(float *x, size_t n);
    void (*gelu)(float *x, size_t n);
    void (*glu)(float *out, size_t os, const float *x, size_t xs, uint32_t T, uint32_t n);
    void (*dwconv)(float *out, size_t os, const float *x, size_t xs, uint32_t T, uint32_t C,
                   const float *w, const float *b, uint32_t K);
    void (*conv3x3s2)(float *out, const float *in, uint32_t r0, uint32_t Ti, uint32_t Fi,
                      uint32_t C, int depthwise, const float *w, const float *b, int relu,
                      uint32_t t0, uint32_t t1);
    void (*lstm)(float *h, float *c, const float *g, uint32_t H);
    void (*stft)(float *out, size_t os, const float *const *x, uint32_t count,
                 const pk_fft *f, float *scratch);
    void (*resample)(float *y, const float *x, uint32_t nb, uint32_t orig, uint32_t nw,
                     const float *k, const size_t *at, const uint32_t *first, const uint32_t *len);
} pk_kernels;

#ifdef __cplusplus
}
#endif

#endif /* PK_KERNELS_ABI_H */
