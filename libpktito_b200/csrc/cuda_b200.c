/* backend/cuda-b200: libpktito's int8 path on an NVIDIA B200 (sm_100a).
 *
 * The reference's backends each export one table of kernels
 * (backend/kernels.h:242-282); this is the table of a GPU one. Its two
 * kernels on the int8 path run on the GPU through libpktito_b200's C ABI
 * (include/pktito_b200.h):
 *
 *   quantize  pk_k_quantize's contract (backend/kernels.h:47-58)  -> pkb_quantize_host
 *   gemm_q8   pk_k_gemm_q8's contract (backend/kernels.h:60-78)   -> pkb_gemm_q8_host
 *
 * and compute ref's bits (backend/ref/kernels.c:24-86) in the rounding mode
 * the calling thread has set, which they read with fegetround() on every
 * call, as the reference's own arithmetic follows it (tests/q8check.c
 * holds a backend to ref under all four modes).
 *
 * The table has no error channel (its functions return void) and a wrong
 * bit would break the reference's contract silently, so a failure of the
 * GPU path prints the reason and aborts; there is no CPU fallback.
 *
 * The other eleven kernels (float products, norms, activations, the
 * convolutions, LSTM, STFT, resampling) are off the int8 path; they forward
 * to the reference's own ref backend, which defines their bits, when the
 * program that loads this table has it (pk_kernels_ref, declared weak here
 * so that the table also loads where only the int8 path is used).
 *
 * A second table, pk_kernels_cuda_b200_f32 ("cuda-b200-f32"), also runs the
 * attention's float kernels on the GPU:
 *
 *   gemm_f32  pk_k_gemm_f32's contract (backend/kernels.h:88-103)  -> pkb_gemm_f32_host
 *   softmax   pk_k_softmax's contract (backend/kernels.h:124-130)  -> pkb_softmax_host
 *
 * (ref's bits, backend/ref/kernels.c:90-105 and 134-147). Every such call
 * crosses PCIe: the engine calls them per head, block of 16 queries and
 * score row (core/encoder.c:291-325), and the decoder and the VAD call
 * gemm_f32 for small products, so cuda-b200 keeps them on the host and this
 * table is the one to pick where the float products should run on the GPU
 * (the attention over whole segments on device buffers is
 * pkb_attention_dev / pkb_attention_rows_dev).
 *
 * Built inside the reference's tree (backend/cuda-b200/kernels.c with
 * -DPK_CUDA_B200_IN_TREE) it takes the reference's own kernels.h; built
 * here it takes include/pk_kernels_abi.h, the same layout.
 */
#ifdef PK_CUDA_B200_IN_TREE
#include "kernels.h"
#else
#include "../../include/pk_kernels_abi.h"
#endif
#include "../../include/pktito_b200.h"

#include <fenv.h>
#include <stdio.h>
#include <stdlib.h>

#pragma STDC FENV_ACCESS ON

static int rounding_now(void) {
    switch (fegetround()) {
    case FE_DOWNWARD: return PKB_RD;
    case FE_UPWARD: return PKB_RU;
    case FE_TOWARDZERO: return PKB_RZ;
    default: return PKB_RN;
    }
}

static void die(const char *kernel, int rc) {
    fprintf(stderr, "cuda-b200: %s failed (%d): %s\n", kernel, rc, pkb_last_error());
    abort();
}

static void k_quantize(pk_act *a, const float *x, size_t xs) {
    const int rc = pkb_quantize_host(a->q, a->d, a->n, a->qb, a->T, x, xs, rounding_now());
    if (rc)
        die("quantize", rc);
}

static void k_gemm_q8(float *out, size_t os, const int8_t *w, const float *ws, const float *bias,
                      uint32_t rows, const pk_act *a, int add) {
    const int rc = pkb_gemm_q8_host(out, os, w, ws, bias, rows, a->q, a->d, a->n, a->qb, a->T, add,
                                    rounding_now());
    if (rc)
        die("gemm_q8", rc);
}

/* ----------------------------------------- off the int8 path: ref's own -- */

extern const pk_kernels pk_kernels_ref __attribute__((weak));

static const pk_kernels *ref(const char *kernel) {
    if (!&pk_kernels_ref) {
        fprintf(stderr, "cuda-b200: %s is off the GPU path and this program has no ref backend\n", kernel);
        abort();
    }
    return &pk_kernels_ref;
}

static void k_gemm_f32(float *out, size_t os, const float *w, uint32_t ld, uint32_t rows, uint32_t n,
                       const float *x, size_t xs, uint32_t T, const float *bias, size_t bs, int relu) {
    ref("gemm_f32")->gemm_f32(out, os, w, ld, rows, n, x, xs, T, bias, bs, relu);
}

static void k_gemm_f32_gpu(float *out, size_t os, const float *w, uint32_t ld, uint32_t rows, uint32_t n,
                           const float *x, size_t xs, uint32_t T, const float *bias, size_t bs, int relu) {
    const int rc = pkb_gemm_f32_host(out, os, w, ld, rows, n, x, xs, T, bias, bs, relu, rounding_now());
    if (rc)
        die("gemm_f32", rc);
}

static void k_softmax_gpu(float *x, uint32_t n, float scale) {
    const int rc = pkb_softmax_host(x, n, scale, rounding_now());
    if (rc)
        die("softmax", rc);
}

static void k_layernorm(float *out, size_t os, const float *x, size_t xs, uint32_t T, uint32_t n,
                        const float *w, const float *b, float eps) {
    ref("layernorm")->layernorm(out, os, x, xs, T, n, w, b, eps);
}

static void k_softmax(float *x, uint32_t n, float scale) { ref("softmax")->softmax(x, n, scale); }

static void k_silu(float *x, size_t n) { ref("silu")->silu(x, n); }

static void k_gelu(float *x, size_t n) { ref("gelu")->gelu(x, n); }

static void k_glu(float *out, size_t os, const float *x, size_t xs, uint32_t T, uint32_t n) {
    ref("glu")->glu(out, os, x, xs, T, n);
}

static void k_dwconv(float *out, size_t os, const float *x, size_t xs, uint32_t T, uint32_t C,
                     const float *w, const float *b, uint32_t K) {
    ref("dwconv")->dwconv(out, os, x, xs, T, C, w, b, K);
}

static void k_conv3x3s2(float *out, const float *in, uint32_t r0, uint32_t Ti, uint32_t Fi, uint32_t C,
                        int depthwise, const float *w, const float *b, int relu, uint32_t t0,
                        uint32_t t1) {
    ref("conv3x3s2")->conv3x3s2(out, in, r0, Ti, Fi, C, depthwise, w, b, relu, t0, t1);
}

static void k_lstm(float *h, float *c, const float *g, uint32_t H) { ref("lstm")->lstm(h, c, g, H); }

static void k_stft(float *out, size_t os, const float *const *x, uint32_t count, const pk_fft *f,
                   float *scratch) {
    ref("stft")->stft(out, os, x, count, f, scratch);
}

static void k_resample(float *y, const float *x, uint32_t nb, uint32_t orig, uint32_t nw, const float *k,
                       const size_t *at, const uint32_t *first, const uint32_t *len) {
    ref("resample")->resample(y, x, nb, orig, nw, k, at, first, len);
}

/* The CPU features it needs. The reference's picker (backend/kernels.c:
 * 227-236) takes the first backend whose needs the CPU meets, so inside
 * the reference's tree this names "cuda", which core/os.c's cpu_has answers
 * from pkb_device_count() (a one-line addition there); built alone, nothing, and a
 * caller selects it by name (PKTITO_KERNELS=cuda-b200) or by its place in
 * a list. */
#ifdef PK_CUDA_B200_NEEDS_CUDA
static const char *const needs[] = { "cuda", NULL };
#else
static const char *const needs[] = { NULL };
#endif

const pk_kernels pk_kernels_cuda_b200 = {
    "cuda-b200",
    "cuda-b200 (B200 sm_100a: tcgen05 int8 MMA, TMEM int32 sums)",
    needs,
    0,
    k_quantize,
    k_gemm_q8,
    k_gemm_f32,
    k_layernorm,
    k_softmax,
    k_silu,
    k_gelu,
    k_glu,
    k_dwconv,
    k_conv3x3s2,
    k_lstm,
    k_stft,
    k_resample,
};

const pk_kernels pk_kernels_cuda_b200_f32 = {
    "cuda-b200-f32",
    "cuda-b200-f32 (cuda-b200, with gemm_f32 and softmax on the GPU too)",
    needs,
    0,
    k_quantize,
    k_gemm_q8,
    k_gemm_f32_gpu,
    k_layernorm,
    k_softmax_gpu,
    k_silu,
    k_gelu,
    k_glu,
    k_dwconv,
    k_conv3x3s2,
    k_lstm,
    k_stft,
    k_resample,
};
