/* The reference's TDT greedy search on its own model, for pinning the
 * oracle's restatement: TEST INFRASTRUCTURE ONLY (oracle/Makefile links it
 * against the reference's engine core, oracle/_ref/libpkcore.so).
 *
 *   tdt_ref <model.pkf> <frames> <seed> <scale> <out.bin>
 *
 * Loads the model with the reference's pk_model_load, makes a transcriber
 * with pk_asr_new, draws <frames> frames of the joint's encoder half
 * (J floats each, xorshift64* uniform in [-scale, scale)), runs the
 * reference's pk_decode over them (core/decoder.c:158-179) and writes to
 * <out.bin>, little-endian:
 *
 *   u32 P, L, J, V, n_dur, max_symbols, n_out_pad, T, ntok
 *   u32 dur[n_dur]
 *   f32 embed[(V + 1) P]
 *   per layer: i8 wx[4P P], f32 wxs[4P], i8 wh[4P P], f32 whs[4P], f32 b[4P]
 *   i8 jpred[J P], f32 jpreds[J], f32 jpredb[J]
 *   i8 jout[n_out_pad J], f32 jouts[n_out_pad], f32 joutb[n_out_pad]
 *   f32 f[T J]
 *   i32 (id, frame, dur) for each token
 *
 * Reads the model's fields through the reference's own headers; changes
 * nothing of its sources. */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "asr.h"

static uint64_t g_s;

static uint32_t rnd(void) {
    g_s ^= g_s >> 12;
    g_s ^= g_s << 25;
    g_s ^= g_s >> 27;
    return (uint32_t)((g_s * 0x2545F4914F6CDD1Dull) >> 32);
}

static void put(FILE *o, const void *p, size_t bytes) {
    if (bytes && fwrite(p, 1, bytes, o) != bytes) {
        perror("write");
        exit(1);
    }
}

static void u32(FILE *o, uint32_t v) { put(o, &v, 4); }

int main(int argc, char **argv) {
    if (argc != 6) {
        fprintf(stderr, "usage: %s model.pkf frames seed scale out.bin\n", argv[0]);
        return 2;
    }
    char err[256];
    pk_model *m = pk_model_load(argv[1], err, sizeof err);
    if (!m) {
        fprintf(stderr, "%s\n", err);
        return 1;
    }
    pk_asr *a = pk_asr_new(m, 1);
    if (!a)
        return 1;
    const uint32_t T = (uint32_t)atoi(argv[2]);
    g_s = (uint64_t)strtoull(argv[3], NULL, 10) | 1;
    const float scale = (float)atof(argv[4]);
    const uint32_t P = m->pred_hidden, L = m->pred_layers, J = m->joint_hidden, V = m->vocab;
    float *f = malloc((size_t)T * J * sizeof *f);
    for (size_t i = 0; i < (size_t)T * J; i++)
        f[i] = scale * ((float)(rnd() >> 8) / 8388608.0f - 1.0f);
    const long n = pk_decode(a, T, f, 0);
    if (n < 0)
        return 1;
    FILE *o = fopen(argv[5], "wb");
    if (!o)
        return 1;
    u32(o, P), u32(o, L), u32(o, J), u32(o, V), u32(o, m->n_dur), u32(o, m->max_symbols), u32(o, m->n_out_pad);
    u32(o, T), u32(o, (uint32_t)n);
    put(o, m->dur, m->n_dur * 4);
    put(o, m->embed, (size_t)(V + 1) * P * 4);
    for (uint32_t l = 0; l < L; l++) {
        const pk_lstmw *w = &m->lstm[l];
        put(o, w->wx.q, (size_t)4 * P * P);
        put(o, w->wx.s, (size_t)4 * P * 4);
        put(o, w->wh.q, (size_t)4 * P * P);
        put(o, w->wh.s, (size_t)4 * P * 4);
        put(o, w->b, (size_t)4 * P * 4);
    }
    put(o, m->jpred.q, (size_t)J * P);
    put(o, m->jpred.s, (size_t)J * 4);
    put(o, m->jpred_b, (size_t)J * 4);
    put(o, m->jout.q, (size_t)m->n_out_pad * J);
    put(o, m->jout.s, (size_t)m->n_out_pad * 4);
    put(o, m->jout_b, (size_t)m->n_out_pad * 4);
    put(o, f, (size_t)T * J * 4);
    for (long i = 0; i < n; i++) {
        const int32_t t3[3] = { a->toks[i].id, a->toks[i].frame, a->toks[i].dur };
        put(o, t3, sizeof t3);
    }
    fclose(o);
    pk_asr_free(a);
    pk_model_free(m);
    free(f);
    return 0;
}
