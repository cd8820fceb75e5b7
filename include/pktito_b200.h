/* libpktito_b200: libpktito's int8 path (activation quantization, the
 * int8 x int8 -> int32 block sums, the float32 scale epilogue) on B200
 * (sm_100a), behind a C ABI.
 *
 * Two layers of entry points:
 *
 *  - pkb_*_host: the reference's backend contract, host pointers in and out,
 *    synchronous. These are what the cuda-b200 entry of the reference's
 *    backend table calls (libpktito_b200/csrc/cuda_b200.c exports
 *    `pk_kernels_cuda_b200`, the table of backend/kernels.h:242-278, and
 *    `pk_kernels_cuda_b200_f32`, the same with the attention's float
 *    kernels gemm_f32 and softmax on the GPU too).
 *
 *  - pkb_*_dev: the same arithmetic on device-resident buffers, enqueued on a
 *    caller's CUDA stream and returning at once; for callers that keep a
 *    batch of segments on the GPU. The first call on a device sets the
 *    device up (the kernels' shared-memory limits, their grid sizes); make it
 *    before capturing a stream into a CUDA graph.
 *
 * Every function returns PKB_OK (0) or a nonzero pkb_status; the message of
 * the calling thread's last failure is pkb_last_error(). Nothing falls back
 * to the CPU: without a usable sm_100 device every compute entry fails with
 * PKB_ENODEV.
 *
 * Results are the reference `ref` backend's bits (backend/ref/kernels.c), in
 * whichever of the four IEEE rounding modes the caller names: rmode is one
 * of PKB_RN, PKB_RD, PKB_RU, PKB_RZ, and the table entry passes the mode its
 * caller's fegetround() reports, as the reference's own arithmetic follows it.
 */
#ifndef PKTITO_B200_H
#define PKTITO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    PKB_OK = 0,
    PKB_EINVAL = 1,   /* a shape, stride, alignment or pointer the contract rules out */
    PKB_ECUDA = 2,    /* a CUDA runtime or driver call failed */
    PKB_ENOMEM = 3,   /* device or pinned host memory could not be had */
    PKB_ETIMEOUT = 4, /* a kernel's bounded wait ran out; its results are not to be used */
    PKB_ENODEV = 5    /* no sm_100 device */
} pkb_status;

enum { PKB_RN = 0, PKB_RD = 1, PKB_RU = 2, PKB_RZ = 3 };

/* The widest input a product may have, in blocks of 32: the reference's
 * PK_MAX_BLOCKS (backend/kernels.h:83) times 32. */
#define PKB_MAX_N 16384u

/* ------------------------------------------------------------ library -- */

/* The calling thread's last failure, "" if none. */
const char *pkb_last_error(void);

/* sm_100 devices this process can use (0 without a GPU or a driver). */
int pkb_device_count(void);

/* The device this thread's host-pointer calls run on (default 0). A pool
 * spread over several GPUs binds each of its threads to one. */
int pkb_set_thread_device(int device);

/* Reads and clears the device-side error word of `device`: nonzero after a
 * kernel's bounded wait ran out (bit 0) or it met an argument it refused
 * (bit 1). pkb_*_host check it on every call; pkb_*_dev callers check it
 * after synchronising. */
int pkb_device_errors(int device, uint32_t *word);

/* A self-test of that failure path (no counterpart in the reference): on the
 * calling thread's current device, one small kernel waits on a barrier that
 * nothing completes, gives up after limit_cycles SM clock cycles (1000 to
 * 2^31), sets the error word's timeout bit and returns. *gave_up is 1 when
 * it did; the device stays usable. For tests and health checks. */
int pkb_wait_selftest(uint64_t limit_cycles, int *gave_up);

/* Checks the sigmoid's branch-free reciprocal (Markstein's method, used by
 * the fused producers) against CUDA's correctly rounded reciprocal in the
 * rounding mode rmode for every float whose bits lie in [lo_bits, hi_bits),
 * within [1, 2^128): *mismatches = how many differ, *first_bad = the
 * smallest such bits (0xFFFFFFFF if none). A test of this library's own
 * arithmetic; no counterpart in the reference. */
int pkb_rcp_selftest(int rmode, uint32_t lo_bits, uint32_t hi_bits, uint64_t *mismatches, uint32_t *first_bad);

/* ---------------------------------------------- host-pointer contract -- */

/* pk_k_quantize (backend/kernels.h:47-58; ref backend/ref/kernels.c:24-58):
 * T columns of n floats, column t at x + t*xs, quantized in blocks of qb
 * (qb a multiple of 32 dividing n, n <= PKB_MAX_N) into q [T][n] and
 * d [T][n/qb]. T == 0 touches nothing. */
int pkb_quantize_host(int8_t *q, float *d, uint32_t n, uint32_t qb, uint32_t T, const float *x,
                      size_t xs, int rmode);

/* pk_k_gemm_q8 (backend/kernels.h:60-78; ref backend/ref/kernels.c:60-86):
 * out[t*os + r] for r < rows, t < T, from the PK_Q8 matrix w (core/pkf.h:28-41;
 * rows a multiple of 16, w at its first row), scales ws, optional bias, and
 * the activations q/d of n inputs in blocks of qb. The floats of out between
 * rows and os are left as they were. The matrix is uploaded once and kept on
 * the device, indexed by its host address range (calls on slices of one
 * matrix share one device copy); each call compares sampled lines of its
 * weights with the bytes uploaded (the whole range up to 256 KiB) and
 * uploads them again where they differ. A caller that rewrites or unmaps
 * weights calls pkb_forget first, as the reference's read-only mapping of
 * the model never changes while the model is loaded. */
int pkb_gemm_q8_host(float *out, size_t os, const int8_t *w, const float *ws, const float *bias,
                     uint32_t rows, const int8_t *q, const float *d, uint32_t n, uint32_t qb,
                     uint32_t T, int add, int rmode);

/* Drops every cached matrix whose host bytes overlap [p, p + bytes), on
 * every device; for a caller about to unmap or rewrite weights. A product
 * running on those weights meanwhile finishes on the copy it holds, whose
 * device memory is freed when it returns. */
int pkb_forget(const void *p, size_t bytes);

/* ------------------------------------------------ device-resident path -- */

/* Bytes of the device layout pkb_repack_q8_dev writes for a rows x n matrix:
 * rows of n int8, row r at r*n (rows a multiple of 16, n of 32). */
size_t pkb_wpack_bytes(uint32_t rows, uint32_t n);

/* PK_Q8 panels (device copy of the reference's bytes, core/pkf.h:28-41) to
 * the row-major layout the product's TMA tiles read; once per matrix. */
int pkb_repack_q8_dev(void *stream, int8_t *wpack, const int8_t *w_pk, uint32_t rows, uint32_t n);

/* pkb_quantize_host's arithmetic on device buffers, enqueued on stream. */
int pkb_quantize_dev(void *stream, int8_t *q, float *d, const float *x, size_t xs, uint32_t T,
                     uint32_t n, uint32_t qb, int rmode);

/* pkb_gemm_q8_host's arithmetic on device buffers, enqueued on stream, with
 * the weights repacked by pkb_repack_q8_dev (wpack at its first row). q and
 * wpack must be 16-byte aligned; out may have any stride os >= rows. */
int pkb_gemm_q8_dev(void *stream, float *out, size_t os, const int8_t *wpack, const float *ws,
                    const float *bias, uint32_t rows, const int8_t *q, const float *d, uint32_t n,
                    uint32_t qb, uint32_t T, int add, int rmode);

/* The product straight into the attention's panels (pk_k_gemm_f32's
 * layout), as the reference's encoder makes them (core/passes.c:119-196),
 * on device buffers, for an attention that stays on the GPU. No bias and
 * nothing added, as the reference's V, K and P products.
 *   PKB_PANELS_V:  result (frame t, row r) at panels + (r/16) ps + 16 t + r%16
 *                  (pk_gemm_panels_on: one product a 16-row panel, os 16;
 *                  the reference's ps is 16 T)
 *   PKB_PANELS_KP: result (frame t, row r = h dk + d) at
 *                  panels + h tpad dk + (t/16) 16 dk + 16 d + t%16, frames T to
 *                  tpad - 1 written as zeros (pk_panels_tile: K with tpad the
 *                  frames rounded up to 16, P with its positions rounded up
 *                  to 16 plus 16); dk a multiple of 16 dividing rows.
 * Fastest where n / qb is a multiple of 4 and panels, d and ws are 16-byte
 * aligned (and, for V, ps a multiple of 4): the results then leave by TMA
 * stores of panel-shaped boxes; otherwise by plain stores, same bytes. */
#define PKB_PANELS_V 1
#define PKB_PANELS_KP 2
int pkb_gemm_q8_panels_dev(void *stream, float *panels, int kind, size_t ps, uint32_t dk, uint32_t tpad,
                           const int8_t *wpack, const float *ws, uint32_t rows, const int8_t *q, const float *d,
                           uint32_t n, uint32_t qb, uint32_t T, int rmode);

/* ---------------------------------------- fused producers (device) -- */

/* The producers of the product's int8 inputs in the reference's encoder,
 * each one kernel on device buffers, enqueued on stream: the float step and
 * the quantization of its result, bit for bit the reference's (each float
 * operation its own, in its order, rounded in rmode; the quantization
 * k_quantize's). Blocks qb of 32 or 64, the encoder's qb()
 * (core/encoder.c:56). No counterpart in the backend table: the reference
 * makes these in core/encoder.c from the table's float kernels and
 * pk_quant_part (core/passes.c:114-118) on the host. */

/* The largest row pkb_layernorm_quantize_dev takes. */
#define PKB_LN_MAX_N 8192u

/* normq (core/encoder.c:112-130): each of T rows of n floats (row t at
 * x + t*xs) normalized by k_layernorm (backend/ref/kernels.c:115-131: its
 * two sums in 16 lanes, folded 8, 4, 2, 1; w and b of n; eps) and quantized
 * into q [T][n], d [T][n/qb]. n a multiple of qb, at most PKB_LN_MAX_N. */
int pkb_layernorm_quantize_dev(void *stream, int8_t *q, float *d, const float *x, size_t xs, uint32_t T,
                               uint32_t n, uint32_t qb, const float *w, const float *b, float eps, int rmode);

/* k_layernorm alone (backend/ref/kernels.c:115-131), the floats out: the
 * encoder's out norm (core/encoder.c:367, `norm`), which the next layer's
 * residual reads. out rows at stride os; out may be x itself (in place,
 * os == xs), as the reference runs it. n a multiple of 32, at most
 * PKB_LN_MAX_N. */
int pkb_layernorm_dev(void *stream, float *out, size_t os, const float *x, size_t xs, uint32_t T, uint32_t n,
                      const float *w, const float *b, float eps, int rmode);

/* siluq_tile (core/encoder.c:150-158): T rows of n floats (row t at
 * u + t*us) through k_silu (backend/ref/kernels.c:149-151: x * pk_sigmoidf(x),
 * core/vmath.h:134-151) and quantized into q [T][n], d [T][n/qb]. */
int pkb_silu_quantize_dev(void *stream, int8_t *q, float *d, const float *u, size_t us, uint32_t T,
                          uint32_t n, uint32_t qb, int rmode);

/* glu_item + dw_item (core/encoder.c:160-183): the convolution module's
 * depthwise convolution k_dwconv (backend/ref/kernels.c:163-177: C channels,
 * K taps centred, the taps past either end skipped, + b, SiLU) over T
 * frames, quantized a frame at a time into q [T][C], d [T][C/qb]. Its input:
 * with glu 0, frame t's C floats at x + t*xs; with glu 1, pw1's output, 2C
 * floats a frame at x + t*xs, made into k_glu's x[i] * pk_sigmoidf(x[C + i])
 * (backend/ref/kernels.c:157-161) on the way in. w holds C rows of K taps.
 * out, if not NULL, also receives the convolution's floats (frame t at
 * out + t*os, os >= C), as k_dwconv writes them; it must not overlap x. C a
 * multiple of qb, at most PKB_MAX_N; K odd, at most 63 (the model's bounds,
 * core/model.c:480,500). */
int pkb_dwconv_quantize_dev(void *stream, int8_t *q, float *d, float *out, size_t os, const float *x, size_t xs,
                            uint32_t T, uint32_t C, const float *w, const float *b, uint32_t K, int glu,
                            uint32_t qb, int rmode);

/* --------------------------------- the attention's float work (device) -- */

/* pk_k_gemm_f32 (backend/kernels.h:88-103; backend/ref/kernels.c:90-105) on
 * device buffers, enqueued on stream, bit for bit the reference's ref: w in
 * panels of 16 rows, ld k to a panel, w at the first k of the run this call
 * takes; out[t*os + r] = chain over k of fmaf(w(r, k), x[t*xs + k]) from +0,
 * plus bias[t*bs + r] (bs 0: one bias for every column) or plus 0.0f without
 * one, then max(v, 0) if relu. rows a multiple of 16; out may be bias
 * itself (os == bs), no other argument may overlap out. The reference's
 * table entry on host pointers is pkb_gemm_f32_host. */
int pkb_gemm_f32_dev(void *stream, float *out, size_t os, const float *w, uint32_t ld, uint32_t rows, uint32_t n,
                     const float *x, size_t xs, uint32_t T, const float *bias, size_t bs, int relu, int rmode);

/* The table's gemm_f32 on host memory (what pk_kernels_cuda_b200_f32 calls):
 * the run of panels, the columns and the biases go up, the results' rows
 * come back at their stride (only out[t*os + r] for r < rows is written, as
 * the contract says). Synchronous; the calling thread's device. */
int pkb_gemm_f32_host(float *out, size_t os, const float *w, uint32_t ld, uint32_t rows, uint32_t n,
                      const float *x, size_t xs, uint32_t T, const float *bias, size_t bs, int relu, int rmode);

/* The table's softmax on one row of n floats of host memory, in place. */
int pkb_softmax_host(float *x, uint32_t n, float scale, int rmode);

/* pk_k_softmax (backend/kernels.h:124-130; backend/ref/kernels.c:134-147)
 * on T rows of n scores (row t at x + t*xs), each in place, on device
 * buffers: y = x * scale, m = max(y), e = pk_expf(y - m), x = e * (1 / sum(e))
 * with the sum in the reference's 16 lanes. One row is the table's call;
 * pkb_softmax_host takes it on host memory. */
int pkb_softmax_dev(void *stream, float *x, size_t xs, uint32_t T, uint32_t n, float scale, int rmode);

/* att_item (core/encoder.c:280-326) over every head and query of one
 * segment of T frames, on device buffers, bit for bit the reference's:
 * query i of head h against key k scores
 *   ((q_i + bias_u) . K_k + 0) + ((q_i + bias_v) . P_{T-1-i+k} + 0),
 * each dot one chain of fmaf over the head's dk dimensions; those T scores
 * through pk_k_softmax with scale 1 / sqrtf(dk); o_i = the chain over k of
 * fmaf(V_k, weight_k) + 0, into o + i*os + h*dk. q: rows of D floats at
 * stride qs. kp, pp and vp as the reference lays them out (and
 * pkb_gemm_q8_panels_dev writes them): K panels of Tp = T rounded up to 16
 * frames a head, P panels of Pp = (2T - 1 rounded up to 16) + 16 positions
 * a head (PKB_PANELS_KP layout), V panels of ps = 16 T (PKB_PANELS_V).
 * D = H * dk, dk a multiple of 16 up to 256; kp, pp, vp 16-byte aligned.
 * T is bounded by shared memory (PKB_EINVAL beyond it; about 1,400 frames
 * at dk 128). No counterpart in the backend table: the reference runs this
 * in core/encoder.c from the table's gemm_f32 and softmax. */
int pkb_attention_dev(void *stream, float *o, size_t os, const float *q, size_t qs, const float *kp,
                      const float *pp, const float *vp, const float *bias_u, const float *bias_v, uint32_t T,
                      uint32_t D, uint32_t H, int rmode);

/* A segment of a batch for pkb_attention_rows_dev: T frames, its rows of
 * q, K, V and o from frame f, its 2T - 1 rows of P from row p. */
typedef struct {
    uint32_t T, f, p;
} pkb_att_segment;

/* The same attention over a batch of segments in one launch, with q, K, V
 * and P as plain rows of D floats (the products' own output, the batch's
 * frames one after another): segment s's frame j at q + (f + j)*qs, K at
 * k + (f + j)*ks, V at v + (f + j)*vs, o at o + (f + j)*os; its position row
 * r at p + (p + r)*ps. k, p, v 16-byte aligned, ks, ps, vs multiples of 4.
 * segs is host memory, read before the call returns. No counterpart in the
 * backend table. */
int pkb_attention_rows_dev(void *stream, float *o, size_t os, const float *q, size_t qs, const float *k, size_t ks,
                           const float *v, size_t vs, const float *p, size_t ps, const float *bias_u,
                           const float *bias_v, uint32_t D, uint32_t H, const pkb_att_segment *segs, uint32_t nseg,
                           int rmode);

/* ------------------------------------------ the TDT decoder (device) -- */

#define PKB_TDT_MAX_LAYERS 4
#define PKB_TDT_MAX_DUR 16

/* The TDT decoder's weights on the device: the prediction network's
 * embedding [(V + 1)][P] (row V the blank's) and L LSTM layers (wx, wh:
 * 4P x P, gates i f u o; lb the two biases summed), the joint's jpred (J x P
 * + jpredb) and jout (n_out_pad x J + joutb: V + 1 token logits then n_dur
 * duration logits, rounded up to 16 rows). The int8 matrices are rows as
 * pkb_repack_q8_dev makes them from PK_Q8 panels, with their row scales (the
 * reference's core/model.h:120-128). P and J multiples of 32. */
typedef struct {
    uint32_t P, L, J, V, n_dur, max_symbols, n_out_pad;
    uint32_t dur[PKB_TDT_MAX_DUR];
    const float *embed;
    const int8_t *wx[PKB_TDT_MAX_LAYERS], *wh[PKB_TDT_MAX_LAYERS];
    const float *wxs[PKB_TDT_MAX_LAYERS], *whs[PKB_TDT_MAX_LAYERS], *lb[PKB_TDT_MAX_LAYERS];
    const int8_t *jpred;
    const float *jpreds, *jpredb;
    const int8_t *jout;
    const float *jouts, *joutb;
} pkb_tdt_model;

/* Device bytes pkb_tdt_search_dev's work area takes for S segments. */
size_t pkb_tdt_work_bytes(const pkb_tdt_model *m, uint32_t S);

/* TDT's greedy search (core/decoder.c:125-179, pk_decode) over S segments
 * at once, bit for bit the reference's: segment s's T[s] frames of the
 * joint's encoder half are rows of J floats at f + (f0[s] + t)*J (what the
 * jenc product writes, the batch's segments one after another). Each round
 * every segment still searching takes one joint step at its own frame (the
 * rounds' products have the segments as their columns), and those that
 * emitted a token step their prediction network before the next. Tokens go
 * to toks + (s*cap + i)*3 as (id, frame, duration), their count to ntok[s].
 * f, toks, ntok and work are device memory (work: pkb_tdt_work_bytes of it,
 * 256-byte aligned); f0 and T host memory. Waits for the work already on
 * stream, runs the search on a stream of its own and returns
 * when every search has ended; PKB_EINVAL if a segment found more than cap
 * tokens. No counterpart in the backend table:
 * the reference runs the search in core/decoder.c over the table's
 * quantize, gemm_q8 and lstm, one segment at a time. */
int pkb_tdt_search_dev(void *stream, const pkb_tdt_model *m, const float *f, const uint32_t *f0, const uint32_t *T,
                       uint32_t S, int32_t *toks, uint32_t *ntok, uint32_t cap, void *work, size_t work_bytes,
                       int rmode);

/* Rounds the calling thread's last pkb_tdt_search_dev ran: the joint steps
 * of its longest-running segment. No counterpart in the reference. */
uint64_t pkb_tdt_last_rounds(void);

/* Launches of libpktito_b200 kernels since the process started, on every
 * device: the evidence a benchmark reports for its own kernels' work. */
uint64_t pkb_launch_count(void);

/* Bytes the host-pointer calls (pkb_*_host, the cuda-b200 table) copied
 * from host to device (*up: inputs, row scales, weights when uploaded) and
 * back (*down: results, the device error word), since the process started,
 * on every device. Activations a product reads from the device copy of a
 * quantize result count nothing. No counterpart in the reference. Either
 * pointer may be null. */
void pkb_host_bytes(uint64_t* up, uint64_t* down);

/* ------------------------------------------------- without allocating -- */

/* Bytes of the fixed device staging pkb_quantize_host_noalloc works in. */
#define PKB_NOALLOC_BYTES (8u << 20)

/* pkb_quantize_host's result, for callers that cannot allocate memory when
 * they quantize: an application that gives all of a GPU's memory to its own
 * pool at start-up, or a real-time audio callback in which an allocation (it
 * can synchronize the whole device) is not allowed. It calls no cudaMalloc,
 * cudaMallocHost or cudaFree: the device staging is one array of
 * PKB_NOALLOC_BYTES compiled into the library, which every GPU that loads the
 * library holds until the process exits; the columns are copied straight from
 * the caller's memory. T * n * (5 + 4/qb) bytes (each of the three parts
 * rounded up to 256) must fit in it, or the call fails with PKB_EINVAL and
 * does nothing. It runs on the device pkb_set_thread_device bound the calling
 * thread to (device 0 by default), as the other host-pointer calls do, and
 * reads the device's error word as they do. The first call on a device asks
 * the runtime for the array's address on that device; make it before
 * starting any stream capture. Calls share the array: calls in one process
 * are serialized and each waits for its GPU work before returning, on every
 * path, because two calls whose GPU work overlapped would race on it.
 * No counterpart in the reference: its backends never allocate per call. */
int pkb_quantize_host_noalloc(int8_t *q, float *d, uint32_t n, uint32_t qb, uint32_t T, const float *x,
                              size_t xs, int rmode);

#ifdef __cplusplus
}
#endif

#endif /* PKTITO_B200_H */
