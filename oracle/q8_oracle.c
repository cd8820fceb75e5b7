/* CPU restatement of libpktito's int8 path: TEST INFRASTRUCTURE ONLY.
 *
 * This file is the checker the parity tests hold the CUDA path to. Only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load it;
 * the product (libpktito_b200) never links, calls or falls back to it.
 *
 * It restates two functions of the reference, in this file's own code:
 *
 *   oracle_quantize  backend/ref/kernels.c:24-58 (contract backend/kernels.h:47-58)
 *   oracle_gemm_q8   backend/ref/kernels.c:60-86 (contract backend/kernels.h:60-78),
 *                    with the PK_Q8 panel index of core/pkf.h:28-41
 *
 * Both take the rounding mode as an argument (PKB_RN/RD/RU/RZ, the codes of
 * include/pktito_b200.h) and run their float arithmetic under it, since the
 * reference's arithmetic follows the caller's fesetround() and its
 * q8check runs the product under all four modes (tests/q8check.c:146-155).
 * The fused multiply-add is C's fmaf, IEEE fusedMultiplyAdd, which is what
 * the reference's pk_fmaf defines (core/vmath.h:41-91).
 *
 * Pinned: tests/test_oracle.py holds this file to the reference's own ref
 * backend (oracle/_ref/libpkref.so, built from the reference's sources by
 * oracle/Makefile) and to the committed golden vectors in tests/golden/,
 * which that backend produced.
 *
 * Built with -ffp-contract=off -frounding-math so the compiler neither fuses
 * a multiply and an add nor assumes round-to-nearest.
 */
#include <fenv.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#pragma STDC FENV_ACCESS ON

enum { OR_RN = 0, OR_RD = 1, OR_RU = 2, OR_RZ = 3 };

static int fe_of(int rmode) {
    switch (rmode) {
    case OR_RD: return FE_DOWNWARD;
    case OR_RU: return FE_UPWARD;
    case OR_RZ: return FE_TOWARDZERO;
    default: return FE_TONEAREST;
    }
}

/* One block of qb floats: its scale, and its qb bytes. A block holding a
 * NaN or an infinity, or whose largest magnitude is below 2^-121, becomes
 * zeros with scale 0; any other block is scaled by amax/127 and rounded
 * (in the current mode) to [-127, 127]. */
static void quant_block(int8_t *q, float *d, const float *v, uint32_t qb) {
    float amax = 0.0f;
    int finite = 1;
    for (uint32_t i = 0; i < qb; i++) {
        if (!isfinite(v[i])) {
            finite = 0;
            break;
        }
        const float a = fabsf(v[i]);
        if (a > amax)
            amax = a;
    }
    if (!finite || amax < 0x1p-121f) {
        *d = 0.0f;
        memset(q, 0, qb);
        return;
    }
    *d = amax / 127.0f;
    const float inv = 127.0f / amax;
    for (uint32_t i = 0; i < qb; i++) {
        /* rintf rounds in the current mode; the conversion to int8 goes
         * through int, as the reference's (int8_t)rintf(...) does */
        const float r = rintf(v[i] * inv);
        q[i] = (int8_t)(int32_t)r;
    }
}

/* T columns of n floats (column t at x + t*xs) into q [T][n] and d [T][n/qb] */
void oracle_quantize(int8_t *q, float *d, const float *x, size_t xs, uint32_t T, uint32_t n,
                     uint32_t qb, int rmode) {
    const int was = fegetround();
    fesetround(fe_of(rmode));
    const uint32_t nb = n / qb;
    for (uint32_t t = 0; t < T; t++)
        for (uint32_t b = 0; b < nb; b++)
            quant_block(q + (size_t)t * n + (size_t)b * qb, d + (size_t)t * nb + b,
                        x + (size_t)t * xs + (size_t)b * qb, qb);
    fesetround(was);
}

/* Byte offset of weight (r, k) of a PK_Q8 matrix with n inputs: panels of
 * 16 rows, each a run of 64-byte groups holding 4 inputs of its 16 rows. */
static size_t pk_q8_at(uint32_t n, uint32_t r, uint32_t k) {
    const size_t panel = r / 16, group = k / 4;
    return (panel * (n / 4) + group) * 64 + (size_t)(r % 16) * 4 + k % 4;
}

/* PK_Q8 panels [rows][n] to plain rows, w_rm[r*n + k] */
void oracle_unpack_q8(int8_t *w_rm, const int8_t *w, uint32_t rows, uint32_t n) {
    for (uint32_t r = 0; r < rows; r++)
        for (uint32_t k = 0; k < n; k++)
            w_rm[(size_t)r * n + k] = w[pk_q8_at(n, r, k)];
}

/* plain rows to PK_Q8 panels (the inverse, for building test matrices) */
void oracle_pack_q8(int8_t *w, const int8_t *w_rm, uint32_t rows, uint32_t n) {
    for (uint32_t r = 0; r < rows; r++)
        for (uint32_t k = 0; k < n; k++)
            w[pk_q8_at(n, r, k)] = w_rm[(size_t)r * n + k];
}

/* The exact integer sum of one block: |each product| <= 128*127, so at qb <=
 * 16384 the sum stays inside int32 (the reference's bound, n < 133,000). */
static int32_t block_sum(const int8_t *wr, const int8_t *qt, uint32_t len) {
    int32_t s = 0;
    for (uint32_t k = 0; k < len; k++)
        s += (int32_t)wr[k] * (int32_t)qt[k];
    return s;
}

/* out[t*os + r] for t < T, r < rows, of the PK_Q8 matrix w (its first row at
 * w), activations q [T][n] with scales d [T][n/qb]:
 *
 *   acc = +0; for each block b in order: acc = fmaf((float)s_b, d_b, acc)
 *   v = acc * ws[r]; v = v + bias[r] if bias; out = add ? out + v : v
 *
 * every operation rounded once in the given mode. */
void oracle_gemm_q8(float *out, size_t os, const int8_t *w, const float *ws, const float *bias,
                    uint32_t rows, const int8_t *q, const float *d, uint32_t n, uint32_t qb,
                    uint32_t T, int add, int rmode) {
    if (!T || !rows)
        return;
    const uint32_t nb = n / qb;
    int8_t *w_rm = malloc((size_t)rows * n);
    if (!w_rm)
        abort();
    oracle_unpack_q8(w_rm, w, rows, n);
    const int was = fegetround();
    fesetround(fe_of(rmode));
    for (uint32_t t = 0; t < T; t++) {
        const int8_t *qt = q + (size_t)t * n;
        const float *dt = d + (size_t)t * nb;
        for (uint32_t r = 0; r < rows; r++) {
            const int8_t *wr = w_rm + (size_t)r * n;
            float acc = 0.0f;
            for (uint32_t b = 0; b < nb; b++) {
                const int32_t s = block_sum(wr + (size_t)b * qb, qt + (size_t)b * qb, qb);
                acc = fmaf((float)s, dt[b], acc);
            }
            float v = acc * ws[r];
            if (bias)
                v = v + bias[r];
            float *o = out + (size_t)t * os + r;
            *o = add ? *o + v : v;
        }
    }
    fesetround(was);
    free(w_rm);
}

/* The integer block sums alone, s[t][r][b], for tests that check the tensor
 * core's sums separately from the float chain. */
void oracle_block_sums(int32_t *s, const int8_t *w, uint32_t rows, const int8_t *q, uint32_t n,
                       uint32_t qb, uint32_t T) {
    const uint32_t nb = n / qb;
    int8_t *w_rm = malloc((size_t)rows * n);
    if (!w_rm)
        abort();
    oracle_unpack_q8(w_rm, w, rows, n);
    for (uint32_t t = 0; t < T; t++)
        for (uint32_t r = 0; r < rows; r++)
            for (uint32_t b = 0; b < nb; b++)
                s[((size_t)t * rows + r) * nb + b] =
                    block_sum(w_rm + (size_t)r * n + (size_t)b * qb, q + (size_t)t * n + (size_t)b * qb, qb);
    free(w_rm);
}
