/* CPU restatement of libpktito's int8 path: TEST INFRASTRUCTURE ONLY.
 *
 * This file is the checker the parity tests hold the CUDA path to. Only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load it;
 * the product (libpktito_b200) never links, calls or falls back to it.
 *
 * It restates these functions of the reference, in this file's own code:
 *
 *   oracle_quantize  backend/ref/kernels.c:24-58 (contract backend/kernels.h:47-58)
 *   oracle_gemm_q8   backend/ref/kernels.c:60-86 (contract backend/kernels.h:60-78),
 *                    with the PK_Q8 panel index of core/pkf.h:28-41
 *   and the producers of the product's inputs in the encoder, with the float
 *   kernels and the mathematics they use:
 *   oracle_layernorm_quantize  normq, core/encoder.c:112-130 (k_layernorm,
 *                    backend/ref/kernels.c:109-131, then pk_quant_part,
 *                    core/passes.c:114-118)
 *   oracle_silu_quantize       siluq_tile, core/encoder.c:150-158 (k_silu,
 *                    backend/ref/kernels.c:149-151)
 *   oracle_dwconv_quantize     glu_item + dw_item, core/encoder.c:160-183
 *                    (k_glu :157-161, k_dwconv :163-177)
 *   oracle_expf, oracle_sigmoidf  pk_expf, pk_sigmoidf, core/vmath.h:93-151
 *   and the attention's float work that reads the products' K, P and V panels:
 *   oracle_gemm_f32   k_gemm_f32, backend/ref/kernels.c:90-105 (contract
 *                    backend/kernels.h:88-103)
 *   oracle_softmax    k_softmax, backend/ref/kernels.c:134-147
 *   oracle_attention  att_item, core/encoder.c:280-326, every head and query
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

/* How rintf rounds. 0: IEEE's roundToIntegral in the current mode, the
 * contract's rint (backend/kernels.h:52). 1: as gcc compiles rintf for
 * baseline x86-64 (the reference's own ref build): |x| rounded in the mode,
 * the sign put back, so that under FE_DOWNWARD a negative value rounds
 * toward zero and under FE_UPWARD away from it. The tests use 1 to hold this
 * file to that compiled ref in every mode, and 0 for the CUDA path. */
static int g_rint_style = 0;

void oracle_set_rint_style(int style) { g_rint_style = style; }

static float or_rintf(float x) {
    if (!g_rint_style)
        return rintf(x);
    const float a = fabsf(x);
    if (!(a < 0x1p23f))
        return x;
    return copysignf((a + 0x1p23f) - 0x1p23f, x);
}

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
        const float r = or_rintf(v[i] * inv);
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

/* ------------------------------------------- the producers' float steps -- */

/* pk_expf (core/vmath.h:134-147) with its constants (core/vmath.h:93-124):
 * n = rint(x log2e) on the clamped x, r = x - n ln2 in two fused steps, a
 * degree-6 polynomial by Horner in fused steps, times 2^n. */
static float or_expf(float x) {
    x = fminf(fmaxf(x, -87.0f), 88.0f);
    const float n = or_rintf(x * 0x1.715476p+0f);
    float r = fmaf(n, -0x1.62e430p-1f, x);
    r = fmaf(n, 0x1.05c610p-29f, r);
    float p = 0x1.6ab980p-10f;
    p = fmaf(p, r, 0x1.126d0cp-7f);
    p = fmaf(p, r, 0x1.55589ap-5f);
    p = fmaf(p, r, 0x1.55540ap-3f);
    p = fmaf(p, r, 0x1.fffffap-2f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const uint32_t u = (uint32_t)((int32_t)n + 127) << 23;
    float two_n;
    memcpy(&two_n, &u, sizeof two_n);
    return p * two_n;
}

/* pk_sigmoidf (core/vmath.h:149-151) */
static float or_sigmoidf(float x) { return 1.0f / (1.0f + or_expf(-x)); }

void oracle_expf(float *y, const float *x, size_t n, int rmode) {
    const int was = fegetround();
    fesetround(fe_of(rmode));
    for (size_t i = 0; i < n; i++)
        y[i] = or_expf(x[i]);
    fesetround(was);
}

void oracle_sigmoidf(float *y, const float *x, size_t n, int rmode) {
    const int was = fegetround();
    fesetround(fe_of(rmode));
    for (size_t i = 0; i < n; i++)
        y[i] = or_sigmoidf(x[i]);
    fesetround(was);
}

/* lanes_sum (backend/ref/kernels.c:109-113): 16 partial sums folded 8, 4, 2, 1 */
static float or_fold16(float *acc) {
    for (int h = 8; h > 0; h /= 2)
        for (int i = 0; i < h; i++)
            acc[i] = acc[i] + acc[i + h];
    return acc[0];
}

/* k_layernorm (backend/ref/kernels.c:115-131) on one row: the sums in 16
 * lanes, input i into lane i % 16, in order */
static void or_layernorm_row(float *o, const float *v, uint32_t n, const float *w, const float *b, float eps) {
    float acc[16] = { 0 };
    for (uint32_t i = 0; i < n; i++)
        acc[i % 16] = acc[i % 16] + v[i];
    const float mean = or_fold16(acc) / (float)n;
    memset(acc, 0, sizeof acc);
    for (uint32_t i = 0; i < n; i++) {
        const float c = v[i] - mean;
        acc[i % 16] = acc[i % 16] + c * c;
    }
    const float var = or_fold16(acc) / (float)n;
    const float r = 1.0f / sqrtf(var + eps);
    for (uint32_t i = 0; i < n; i++)
        o[i] = (v[i] - mean) * r * w[i] + b[i];
}

void oracle_layernorm(float *out, size_t os, const float *x, size_t xs, uint32_t T, uint32_t n, const float *w,
                      const float *b, float eps, int rmode) {
    const int was = fegetround();
    fesetround(fe_of(rmode));
    for (uint32_t t = 0; t < T; t++)
        or_layernorm_row(out + (size_t)t * os, x + (size_t)t * xs, n, w, b, eps);
    fesetround(was);
}

/* normq (core/encoder.c:112-130): each row normalized into scratch, then
 * quantized whole (pk_quant_part with k0 = 0, core/passes.c:114-118) */
void oracle_layernorm_quantize(int8_t *q, float *d, const float *x, size_t xs, uint32_t T, uint32_t n, uint32_t qb,
                               const float *w, const float *b, float eps, int rmode) {
    float *row = malloc((size_t)n * sizeof *row);
    if (!row)
        abort();
    const int was = fegetround();
    fesetround(fe_of(rmode));
    const uint32_t nb = n / qb;
    for (uint32_t t = 0; t < T; t++) {
        or_layernorm_row(row, x + (size_t)t * xs, n, w, b, eps);
        for (uint32_t k = 0; k < nb; k++)
            quant_block(q + (size_t)t * n + (size_t)k * qb, d + (size_t)t * nb + k, row + (size_t)k * qb, qb);
    }
    fesetround(was);
    free(row);
}

/* siluq_tile (core/encoder.c:150-158): a row copied to scratch, k_silu
 * (backend/ref/kernels.c:149-151) on it, quantized */
void oracle_silu_quantize(int8_t *q, float *d, const float *u, size_t us, uint32_t T, uint32_t n, uint32_t qb,
                          int rmode) {
    float *row = malloc((size_t)n * sizeof *row);
    if (!row)
        abort();
    const int was = fegetround();
    fesetround(fe_of(rmode));
    const uint32_t nb = n / qb;
    for (uint32_t t = 0; t < T; t++) {
        for (uint32_t i = 0; i < n; i++) {
            const float v = u[(size_t)t * us + i];
            row[i] = v * or_sigmoidf(v);
        }
        for (uint32_t k = 0; k < nb; k++)
            quant_block(q + (size_t)t * n + (size_t)k * qb, d + (size_t)t * nb + k, row + (size_t)k * qb, qb);
    }
    fesetround(was);
    free(row);
}

/* k_glu (backend/ref/kernels.c:157-161): out[t][i] = a[i] * sigmoid(a[n + i]) */
static void or_glu(float *out, size_t os, const float *x, size_t xs, uint32_t T, uint32_t n) {
    for (uint32_t t = 0; t < T; t++)
        for (uint32_t i = 0; i < n; i++)
            out[(size_t)t * os + i] = x[(size_t)t * xs + i] * or_sigmoidf(x[(size_t)t * xs + n + i]);
}

/* k_dwconv (backend/ref/kernels.c:163-177): K taps centred, those reading
 * past either end skipped, + bias, SiLU */
static void or_dwconv(float *out, size_t os, const float *x, size_t xs, uint32_t T, uint32_t C, const float *w,
                      const float *b, uint32_t K) {
    for (uint32_t t = 0; t < T; t++)
        for (uint32_t c = 0; c < C; c++) {
            float acc = 0.0f;
            for (uint32_t j = 0; j < K; j++) {
                const int64_t s = (int64_t)t + j - K / 2;
                if (s >= 0 && s < T)
                    acc = fmaf(w[(size_t)c * K + j], x[(size_t)s * xs + c], acc);
            }
            const float v = acc + b[c];
            out[(size_t)t * os + c] = v * or_sigmoidf(v);
        }
}

/* glu_item + dw_item (core/encoder.c:160-183): with glu, x is pw1's output
 * (2C a frame) made into k_glu's C first; the convolution into out (scratch
 * when out is NULL), then each frame quantized (its chunks of 64 channels
 * are whole blocks, so a frame's blocks are the same as the row's) */
void oracle_dwconv_quantize(int8_t *q, float *d, float *out, size_t os, const float *x, size_t xs, uint32_t T,
                            uint32_t C, const float *w, const float *b, uint32_t K, int glu, uint32_t qb, int rmode) {
    float *h = NULL, *o = out;
    if (glu && !(h = malloc((size_t)T * C * sizeof *h)))
        abort();
    if (!o) {
        if (!(o = malloc((size_t)T * C * sizeof *o)))
            abort();
        os = C;
    }
    const int was = fegetround();
    fesetround(fe_of(rmode));
    if (glu) {
        or_glu(h, C, x, xs, T, C);
        or_dwconv(o, os, h, C, T, C, w, b, K);
    } else {
        or_dwconv(o, os, x, xs, T, C, w, b, K);
    }
    const uint32_t nb = C / qb;
    for (uint32_t t = 0; t < T; t++)
        for (uint32_t k = 0; k < nb; k++)
            quant_block(q + (size_t)t * C + (size_t)k * qb, d + (size_t)t * nb + k, o + (size_t)t * os + (size_t)k * qb,
                        qb);
    fesetround(was);
    if (o != out)
        free(o);
    free(h);
}

/* ------------------------------------------------- the attention's panels -- */

/* pk_panels_tile (core/passes.c:169-196) over a whole matrix: src's n rows
 * of D floats (frame j of row r at src[j*D + r]) into K/P panels,
 * (dimension d of head h, frame j) at dst[((h*np + j/16)*dk + d)*16 + j%16],
 * frames n .. np-1 zeros. */
void oracle_panels_kp(float *dst, const float *src, uint32_t n, uint32_t np, uint32_t D, uint32_t dk) {
    for (uint32_t r = 0; r < D; r++) {
        const uint32_t h = r / dk, d = r % dk;
        for (uint32_t j = 0; j < np; j++)
            dst[(((size_t)h * np + (j / 16) * 16) * dk) + (size_t)d * 16 + j % 16] =
                j < n ? src[(size_t)j * D + r] : 0.0f;
    }
}

/* ---------------------------------------- the attention's float products -- */

/* k_gemm_f32 (backend/ref/kernels.c:90-105; contract backend/kernels.h:88-103)
 * in the current mode: w in panels of 16 rows, ld k to a panel, w at the
 * first k of the run; each of a panel's 16 outputs for column t is one fused
 * chain over k from +0, then + the bias (bias[t*bs + r], or + 0.0f without
 * one), then the ReLU (v > 0 ? v : 0). out may be bias itself (os == bs). */
static void or_gemm_f32(float *out, size_t os, const float *w, uint32_t ld, uint32_t rows, uint32_t n,
                        const float *x, size_t xs, uint32_t T, const float *bias, size_t bs, int relu) {
    for (uint32_t t = 0; t < T; t++)
        for (uint32_t p = 0; p < rows / 16; p++) {
            const float *wp = w + (size_t)p * ld * 16, *xt = x + (size_t)t * xs;
            float acc[16] = { 0 };
            for (uint32_t k = 0; k < n; k++)
                for (int i = 0; i < 16; i++)
                    acc[i] = fmaf(wp[16 * (size_t)k + i], xt[k], acc[i]);
            for (int i = 0; i < 16; i++) {
                const float v = acc[i] + (bias ? bias[(size_t)t * bs + 16 * p + i] : 0.0f);
                out[(size_t)t * os + 16 * p + i] = relu ? (v > 0 ? v : 0) : v;
            }
        }
}

void oracle_gemm_f32(float *out, size_t os, const float *w, uint32_t ld, uint32_t rows, uint32_t n, const float *x,
                     size_t xs, uint32_t T, const float *bias, size_t bs, int relu, int rmode) {
    const int was = fegetround();
    fesetround(fe_of(rmode));
    or_gemm_f32(out, os, w, ld, rows, n, x, xs, T, bias, bs, relu);
    fesetround(was);
}

/* k_softmax (backend/ref/kernels.c:134-147) on one row, in place: y = x *
 * scale and its maximum (fmaxf, so a NaN is passed over), e = pk_expf(y -
 * m), the sum of the e in 16 lanes folded 8, 4, 2, 1, then e * (1 / sum). */
static void or_softmax(float *x, uint32_t n, float scale) {
    float m = -INFINITY;
    for (uint32_t i = 0; i < n; i++) {
        x[i] = x[i] * scale;
        m = fmaxf(m, x[i]);
    }
    float acc[16] = { 0 };
    for (uint32_t i = 0; i < n; i++) {
        x[i] = or_expf(x[i] - m);
        acc[i % 16] = acc[i % 16] + x[i];
    }
    const float inv = 1.0f / or_fold16(acc);
    for (uint32_t i = 0; i < n; i++)
        x[i] = x[i] * inv;
}

/* T rows of n scores, row t at x + t*xs, each softmaxed in place */
void oracle_softmax(float *x, size_t xs, uint32_t T, uint32_t n, float scale, int rmode) {
    const int was = fegetround();
    fesetround(fe_of(rmode));
    for (uint32_t t = 0; t < T; t++)
        or_softmax(x + (size_t)t * xs, n, scale);
    fesetround(was);
}

/* att_item (core/encoder.c:280-326) for every head and every query of one
 * segment of T frames, in the current mode. q: rows of D floats at stride
 * qs; kp, pp: the K and P panels (head h at kp + h*Tp*dk and pp + h*Pp*dk,
 * Tp = T rounded up to 16, Pp = 2T-1 rounded up to 16, plus 16); vp: the V
 * panels (head h at vp + h*(dk/16)*T*16). Query i of head h:
 *
 *   qu = q_i + bias_u, qv = q_i + bias_v                  (per dimension)
 *   s_k = (qu . K_k + 0) + (qv . P_{T-1-i+k} + 0)         each dot one fused chain over d
 *   softmax(s, T, 1 / sqrtf(dk))
 *   o_i = V^T s + 0                                       one fused chain over k
 *
 * The reference takes the position products over a window of rows per
 * block of 16 queries, and its queries in blocks: neither changes a value,
 * so this takes them query by query. */
void oracle_attention(float *o, size_t os, const float *q, size_t qs, const float *kp, const float *pp,
                      const float *vp, const float *bias_u, const float *bias_v, uint32_t T, uint32_t D, uint32_t H,
                      int rmode) {
    const int was = fegetround();
    fesetround(fe_of(rmode));
    const uint32_t dk = D / H, Tp = (T + 15) & ~15u, Pp = ((2 * T - 1 + 15) & ~15u) + 16;
    float *qu = malloc(dk * sizeof *qu), *qv = malloc(dk * sizeof *qv), *s = malloc((size_t)T * sizeof *s);
    const float scale = 1.0f / sqrtf((float)dk);
    for (uint32_t h = 0; h < H; h++) {
        const float *kh = kp + (size_t)h * Tp * dk, *ph = pp + (size_t)h * Pp * dk;
        const float *vh = vp + (size_t)h * (dk / 16) * T * 16;
        for (uint32_t i = 0; i < T; i++) {
            for (uint32_t d = 0; d < dk; d++) {
                qu[d] = q[(size_t)i * qs + h * dk + d] + bias_u[h * dk + d];
                qv[d] = q[(size_t)i * qs + h * dk + d] + bias_v[h * dk + d];
            }
            for (uint32_t k = 0; k < T; k++) {
                const uint32_t r = T - 1 - i + k;
                float a = 0.0f, b = 0.0f;
                for (uint32_t d = 0; d < dk; d++) {
                    a = fmaf(kh[((size_t)(k / 16) * dk + d) * 16 + k % 16], qu[d], a);
                    b = fmaf(ph[((size_t)(r / 16) * dk + d) * 16 + r % 16], qv[d], b);
                }
                s[k] = (a + 0.0f) + (b + 0.0f);
            }
            or_softmax(s, T, scale);
            for (uint32_t d = 0; d < dk; d++) {
                float acc = 0.0f;
                for (uint32_t k = 0; k < T; k++)
                    acc = fmaf(vh[((size_t)(d / 16) * T + k) * 16 + d % 16], s[k], acc);
                o[(size_t)i * os + h * dk + d] = acc + 0.0f;
            }
        }
    }
    free(qu);
    free(qv);
    free(s);
    fesetround(was);
}

/* --------------------------------------------- the TDT decoder's search -- */

/* pk_tanhf (core/vmath.h:153-165) with its constants (:108-116): below
 * |x| = 0.625 x + x^3 p(x^2) by Horner in fused steps, else
 * copysign(1 - 2 / (e^2|x| + 1), x) */
static float or_tanhf(float x) {
    const float a = fabsf(x);
    if (a < 0.625f) {
        const float x2 = x * x;
        float p = -0x1.75e1cep-8f;
        p = fmaf(p, x2, 0x1.52269cp-6f);
        p = fmaf(p, x2, -0x1.b83c5ap-5f);
        p = fmaf(p, x2, 0x1.110726p-3f);
        p = fmaf(p, x2, -0x1.555532p-2f);
        return fmaf(x * x2, p, x);
    }
    const float e = or_expf(2.0f * a);
    return copysignf(1.0f - 2.0f / (e + 1.0f), x);
}

void oracle_tanhf(float *y, const float *x, size_t n, int rmode) {
    const int was = fegetround();
    fesetround(fe_of(rmode));
    for (size_t i = 0; i < n; i++)
        y[i] = or_tanhf(x[i]);
    fesetround(was);
}

/* k_lstm (backend/ref/kernels.c:203-212): gates g = [i f u o] of H each */
static void or_lstm(float *h, float *c, const float *g, uint32_t H) {
    for (uint32_t j = 0; j < H; j++) {
        const float i = or_sigmoidf(g[j]);
        const float f = or_sigmoidf(g[H + j]);
        const float u = or_tanhf(g[2 * H + j]);
        const float o = or_sigmoidf(g[3 * H + j]);
        c[j] = f * c[j] + i * u;
        h[j] = o * or_tanhf(c[j]);
    }
}

void oracle_lstm(float *h, float *c, const float *g, uint32_t H, int rmode) {
    const int was = fegetround();
    fesetround(fe_of(rmode));
    or_lstm(h, c, g, H);
    fesetround(was);
}

/* The decoder's weights, as core/model.c holds them: int8 matrices in PK_Q8
 * panels with their row scales. */
typedef struct {
    uint32_t P, L, J, V, n_dur, max_symbols, n_out_pad;
    const uint32_t *dur;          /* [n_dur] */
    const float *embed;           /* [V + 1][P] */
    const int8_t *wx, *wh;        /* [L][4P x P] */
    const float *wxs, *whs, *lb;  /* [L][4P] */
    const int8_t *jpred;          /* J x P */
    const float *jpreds, *jpredb; /* [J] */
    const int8_t *jout;           /* n_out_pad x J */
    const float *jouts, *joutb;   /* [n_out_pad] */
} oracle_tdt;

typedef struct {
    const oracle_tdt *m;
    float *h, *c, *gates, *gp, *z, *logit, *d;
    int8_t *q;
    int rmode;
} or_dec;

/* gemv (core/decoder.c:53-63): x quantized as one block of cols, then the
 * product of one column */
static void or_gemv(or_dec *s, float *out, const int8_t *w, const float *ws, uint32_t rows, uint32_t cols,
                    const float *bias, const float *x, int add) {
    oracle_quantize(s->q, s->d, x, cols, 1, cols, cols, s->rmode);
    oracle_gemm_q8(out, rows, w, ws, bias, rows, s->q, s->d, cols, cols, 1, add, s->rmode);
}

/* predict (core/decoder.c:67-79) */
static void or_predict(or_dec *s, uint32_t label) {
    const oracle_tdt *m = s->m;
    const uint32_t P = m->P;
    const float *x = m->embed + (size_t)label * P;
    for (uint32_t l = 0; l < m->L; l++) {
        float *h = s->h + (size_t)l * P, *c = s->c + (size_t)l * P;
        const size_t wo = (size_t)l * 4 * P * P, so = (size_t)l * 4 * P;
        or_gemv(s, s->gates, m->wx + wo, m->wxs + so, 4 * P, P, m->lb + so, x, 0);
        or_gemv(s, s->gates, m->wh + wo, m->whs + so, 4 * P, P, NULL, h, 1);
        oracle_lstm(h, c, s->gates, P, s->rmode);
        x = h;
    }
    or_gemv(s, s->gp, m->jpred, m->jpreds, m->J, P, m->jpredb, x, 0);
}

/* joint (core/decoder.c:83-103): the best token and duration index */
static void or_joint(or_dec *s, const float *f, uint32_t *k, uint32_t *di) {
    const oracle_tdt *m = s->m;
    const int was = fegetround();
    fesetround(fe_of(s->rmode));
    for (uint32_t j = 0; j < m->J; j++) {
        const float v = f[j] + s->gp[j];
        s->z[j] = v > 0 ? v : 0;
    }
    fesetround(was);
    or_gemv(s, s->logit, m->jout, m->jouts, m->n_out_pad, m->J, m->joutb, s->z, 0);
    uint32_t best = 0;
    for (uint32_t i = 1; i <= m->V; i++)
        if (s->logit[i] > s->logit[best])
            best = i;
    uint32_t bd = 0;
    for (uint32_t i = 1; i < m->n_dur; i++)
        if (s->logit[m->V + 1 + i] > s->logit[m->V + 1 + bd])
            bd = i;
    *k = best;
    *di = bd;
}

/* pk_decode + search (core/decoder.c:125-179): TDT's greedy search over T
 * frames of the joint's encoder half (f: [T][J]), from the blank's
 * prediction of a zero state. Writes up to cap tokens (id, frame, duration)
 * and returns their count (-1 past cap). */
long oracle_tdt_search(int32_t *id, int32_t *frame, int32_t *durs, long cap, const float *f, uint32_t T,
                       const oracle_tdt *m, int rmode) {
    or_dec s = { m };
    const uint32_t P = m->P;
    s.rmode = rmode;
    s.h = calloc((size_t)m->L * P, sizeof(float));
    s.c = calloc((size_t)m->L * P, sizeof(float));
    s.gates = malloc((size_t)4 * P * sizeof(float));
    s.gp = malloc((size_t)m->J * sizeof(float));
    s.z = malloc((size_t)m->J * sizeof(float));
    s.logit = malloc((size_t)m->n_out_pad * sizeof(float));
    const uint32_t big = (P > m->J ? P : m->J);
    s.q = malloc(big);
    s.d = malloc(sizeof(float));
    long n = 0;
    const uint32_t blank = m->V;
    if (T) {
        or_predict(&s, blank);
        uint32_t t = 0, last = UINT32_MAX, lasts = 0;
        while (t < T) {
            uint32_t k, di, d, at;
            do {
                at = t;
                or_joint(&s, f + (size_t)t * m->J, &k, &di);
                d = m->dur[di];
                if (k == blank && d == 0)
                    d = 1;
                t += d;
            } while (k == blank && t < T);
            if (k == blank)
                break;
            if (n >= cap) {
                n = -1;
                break;
            }
            id[n] = (int32_t)k;
            frame[n] = (int32_t)at;
            durs[n] = (int32_t)m->dur[di];
            n++;
            lasts = last == at ? lasts + 1 : 1;
            last = at;
            or_predict(&s, k);
            if (lasts >= m->max_symbols && last == t)
                t++;
        }
    }
    free(s.h);
    free(s.c);
    free(s.gates);
    free(s.gp);
    free(s.z);
    free(s.logit);
    free(s.q);
    free(s.d);
    return n;
}
