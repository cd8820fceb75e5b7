/* The reference's own CPU int8 path, timed on this host's cores: the
 * baseline bench.py reports beside the GPU. TEST INFRASTRUCTURE ONLY.
 *
 * Links the reference's backends (_ref/libpkref.so, built by oracle/Makefile
 * from its sources) and lets its own picker choose among them
 * (pk_kernels_pick, backend/kernels.c:277-305: the fastest backend this CPU
 * runs, amx-int8 on an AMX Xeon). A product is run the way the reference's
 * passes run one: the activations quantized in items of 16 columns
 * (pk_quantize_on, core/passes.c:39-46), then the matrix in slices of 64
 * rows dealt to the threads from an atomic counter (pk_gemm_on's items,
 * core/passes.c:60-109; tests/gemmbench.c:73-94 times it the same way).
 */
#include "kernels.h"
#include "os.h"
#include "pkf.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + ts.tv_nsec * 1e-9;
}

/* xorshift64*, the generator the reference's tests use (tests/kcheck.c:40-47) */
static uint32_t next32(uint64_t *s) {
    *s ^= *s >> 12;
    *s ^= *s << 25;
    *s ^= *s >> 27;
    return (uint32_t)((*s * 0x2545F4914F6CDD1Dull) >> 32);
}

static float gauss(uint64_t *s) {
    const double u1 = ((next32(s) >> 8) + 1) / 16777217.0, u2 = (next32(s) >> 8) / 16777216.0;
    return (float)(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
}

/* The backend the reference's picker chooses here; what its probe timed
 * goes to picks. */
const char *cpub_backend(char *picks, size_t len) {
    char why[256];
    const pk_kernels *k = pk_kernels_pick(why, sizeof why);
    if (picks && len)
        pk_k_picks(picks, len);
    return k ? k->id : "none";
}

int cpub_cores(void) { return pk_os_cores(); }

typedef struct {
    float *out;
    size_t os;
    const int8_t *w;
    const float *ws;
    const float *bias;
    const float *x;
    size_t xs;
    pk_act a;
    uint32_t rows;
    int add;
    _Atomic uint32_t next;
    int phase; /* 0 quantize, 1 product */
} job;

static void *worker(void *arg) {
    job *j = arg;
    const uint32_t n = j->a.n, nb = n / j->a.qb;
    if (j->phase == 0) {
        const uint32_t items = (j->a.T + 15) / 16;
        for (;;) {
            const uint32_t i = atomic_fetch_add(&j->next, 1);
            if (i >= items)
                return NULL;
            pk_act sub = j->a;
            const uint32_t t0 = i * 16;
            sub.q += (size_t)t0 * n;
            sub.d += (size_t)t0 * nb;
            sub.T = j->a.T - t0 < 16 ? j->a.T - t0 : 16;
            pk_k_quantize(&sub, j->x + (size_t)t0 * j->xs, j->xs);
        }
    }
    const uint32_t slices = (j->rows + 63) / 64;
    for (;;) {
        const uint32_t i = atomic_fetch_add(&j->next, 1);
        if (i >= slices)
            return NULL;
        const uint32_t r0 = i * 64, nr = j->rows - r0 < 64 ? j->rows - r0 : 64;
        pk_k_gemm_q8(j->out + r0, j->os, j->w + (size_t)r0 * n, j->ws + r0, j->bias ? j->bias + r0 : NULL, nr,
                     &j->a, j->add);
    }
}

static void run_phase(job *j, int phase, int threads) {
    pthread_t th[512];
    if (threads > 512)
        threads = 512;
    if (threads < 1)
        threads = 1;
    j->phase = phase;
    atomic_store(&j->next, 0);
    for (int k = 1; k < threads; k++)
        pthread_create(&th[k], NULL, worker, j);
    worker(j);
    for (int k = 1; k < threads; k++)
        pthread_join(th[k], NULL);
}

/* The picked backend's quantize of T columns of n floats (column t at
 * x + t*xs) in blocks of qb, in items of 16 columns over `threads` threads,
 * as pk_quantize_on deals them (core/passes.c:39-46). */
void cpub_quantize(int8_t *q, float *d, const float *x, size_t xs, uint32_t n, uint32_t qb, uint32_t T,
                   int threads) {
    job j = { NULL, 0, NULL, NULL, NULL, x, xs, { q, d, n, qb, T }, 0, 0, 0, 0 };
    run_phase(&j, 0, threads);
}

/* The picked backend's product (pk_k_gemm_q8's contract, backend/kernels.h:
 * 60-78) with rows x n PK_Q8 weights w, in slices of 64 rows dealt to
 * `threads` threads from an atomic counter, as pk_gemm_on deals them
 * (core/passes.c:60-109); every output is one call's, so the bits do not
 * depend on the split. */
void cpub_gemm(float *out, size_t os, const int8_t *w, const float *ws, const float *bias, uint32_t rows,
               const int8_t *q, const float *d, uint32_t n, uint32_t qb, uint32_t T, int add, int threads) {
    job j = { out, os, w, ws, bias, NULL, 0, { (int8_t *)q, (float *)d, n, qb, T }, rows, add, 0, 1 };
    run_phase(&j, 1, threads);
}

/* Quantize T columns of n floats ~N(0,1) in blocks of qb, then the product
 * with a rows x n matrix (weights uniform in [-127, 127], row scales in
 * [1e-3, 1e-2]), on `threads` threads; the best of `reps` runs of the pair,
 * in seconds, after one untimed run. quant_s gets the quantize's share. */
double cpub_time(uint32_t rows, uint32_t n, uint32_t T, uint32_t qb, int add, int threads, int reps,
                 uint64_t seed, double *quant_s) {
    uint64_t s = seed ? seed : 0x9E3779B97F4A7C15ull;
    int8_t *w = malloc((size_t)rows * n);
    float *ws = malloc((size_t)rows * 4), *x = malloc((size_t)T * n * 4);
    float *out = calloc((size_t)T * rows, 4);
    int8_t *q = malloc((size_t)T * n);
    float *d = malloc((size_t)T * (n / qb) * 4);
    if (!w || !ws || !x || !out || !q || !d)
        return -1.0;
    for (size_t i = 0; i < (size_t)rows * n; i++)
        w[i] = (int8_t)((int)(next32(&s) % 255) - 127);
    for (uint32_t r = 0; r < rows; r++)
        ws[r] = 1e-3f + 9e-3f * (float)(next32(&s) >> 8) / 16777216.0f;
    for (size_t i = 0; i < (size_t)T * n; i++)
        x[i] = gauss(&s);
    job j = { out, rows, w, ws, NULL, x, n, { q, d, n, qb, T }, rows, add, 0, 0 };
    double best = 1e30, bestq = 0;
    for (int rep = 0; rep <= reps; rep++) {
        const double t0 = now_s();
        run_phase(&j, 0, threads);
        const double t1 = now_s();
        run_phase(&j, 1, threads);
        const double t2 = now_s();
        if (rep > 0 && t2 - t0 < best) {
            best = t2 - t0;
            bestq = t1 - t0;
        }
    }
    if (quant_s)
        *quant_s = bestq;
    free(w), free(ws), free(x), free(out), free(q), free(d);
    return best;
}
