// Declarations shared by the CUDA sources of libpktito_b200 (not installed).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace pkb {

// Records the calling thread's error message (what pkb_last_error returns)
// and returns code.
int set_error(int code, const char* fmt, ...);

// The current device, checked to be an sm_100 one and set up: its SM count
// and the device address of its error word.
int current_device_info(int* sms, uint32_t** err_word);

// One more kernel launched (pkb_launch_count).
void count_launch();

// Bytes a host-pointer call copied host to device and back (pkb_host_bytes).
void count_host_bytes(size_t up, size_t down);

// The device the calling thread's host-pointer calls run on
// (pkb_set_thread_device; 0 until set).
int thread_device();

// Arguments of the product kernel (pkb_gemm.cu) besides its two tensor maps.
struct GemmArgs {
    float* out;            // out[t*os + r]
    const float* ws;       // [rows] row scales
    const float* bias;     // [rows] or null
    const float* d;        // [T][n/qb] block scales
    uint32_t* err;         // device-side error word
    unsigned long long os;
    uint32_t rows, n, qb, T, add;
    uint32_t tiles_m, tiles_n;
    long long timeout;     // SM clock cycles a wait may last
    // where the results go (the attention's panels, core/passes.c:119-196):
    // 0 out[t*os + r]; 1 V panels, (t, r) at (r/16) ps + 16 t + r%16;
    // 2 K/P panels, (t, r = h dk + d) at h tpad dk + (t/16) 16 dk + 16 d + t%16,
    // frames T .. tpad-1 written as zeros
    uint32_t pmode, dk, tpad;
    unsigned long long ps;
};

int gemm_tile_rows();   // frames a tile (TMA box of the activations)
int gemm_tile_cols();   // output rows a tile (TMA box of the weights)
int gemm_box_k();       // inputs of K a TMA box

// Sets the product kernels' launch attributes on the current device (once,
// at the device's set-up, outside any stream capture).
cudaError_t prepare_gemm_q8();

// map_d: a tensor map of the block scales d [T][n/qb] (float32, boxes of
// gemm_scale_box() blocks by gemm_tile_rows() frames); map_o: one of the
// results out [T][rows] (float32, row stride os, boxes of gemm_out_box() by
// gemm_out_box(), 128-byte swizzle), or for pmode 1 and 2 one of the panels
// (3-D for V, 4-D for K/P, laid out as the kernel stages them). map_o is
// given only where out, ws and bias are 16-byte aligned and os (V: ps) a
// multiple of 4: the kernel then moves row scales, biases and results with
// TMA; and with it map_d, where n / qb is a multiple of 4 and d 16-byte
// aligned, except for blocks of whole TMA boxes (gemm_wide_blocks), whose
// few scales a tile are plain loads. Null: plain loads and stores.
cudaError_t launch_gemm_q8(const CUtensorMap& map_a, const CUtensorMap& map_b, const CUtensorMap* map_d,
                           const CUtensorMap* map_o, const GemmArgs& g, int num_sms, int rmode, cudaStream_t stream);
int gemm_out_box();     // frames and output rows of a TMA box of the results
// Whether the product runs blocks of whole TMA boxes along K (qb a multiple
// of gemm_box_k(), at least twice it, n a multiple of it): its block scales
// are then not moved by TMA.
bool gemm_wide_blocks(uint32_t n, uint32_t qb);
int gemm_scale_box();   // blocks of scales a TMA box of them carries

// Launches `kern` on `stream` with programmatic stream serialization allowed
// (the kernel calls pdl_trigger / pdl_wait, pkb_device.cuh).
template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kern)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<Params>(args)...);
}

cudaError_t launch_quantize(int8_t* q, float* d, const float* x, size_t xs, uint32_t T, uint32_t n, uint32_t qb,
                            int rmode, int num_sms, cudaStream_t stream);
// The plain quantizer's grid sizes (CTAs resident an SM), once at the
// device's set-up.
void prepare_quantize();

// k_layernorm alone, the floats out (out may be x with os == xs)
cudaError_t launch_layernorm(float* out, size_t os, const float* x, size_t xs, uint32_t T, uint32_t n, const float* w,
                             const float* b, float eps, int rmode, int num_sms, cudaStream_t stream);

cudaError_t launch_silu_quantize(int8_t* q, float* d, const float* u, size_t us, uint32_t T, uint32_t n,
                                 uint32_t qb, int rmode, int num_sms, cudaStream_t stream);

cudaError_t launch_layernorm_quantize(int8_t* q, float* d, const float* x, size_t xs, uint32_t T, uint32_t n,
                                      uint32_t qb, const float* w, const float* b, float eps, int rmode,
                                      int num_sms, cudaStream_t stream);

cudaError_t launch_dwconv_quantize(int8_t* q, float* d, float* out, size_t os, const float* x, size_t xs, uint32_t T,
                                   uint32_t C, const float* w, const float* bias, uint32_t K, bool glu, uint32_t qb,
                                   int rmode, cudaStream_t stream);

// ----------------------------------------- the attention's float work --
// (pkb_attn.cu)

cudaError_t launch_gemm_f32(float* out, size_t os, const float* w, uint32_t ld, uint32_t rows, uint32_t n,
                            const float* x, size_t xs, uint32_t T, const float* bias, size_t bs, int relu, int rmode,
                            cudaStream_t stream);
cudaError_t launch_softmax(float* x, size_t xs, uint32_t T, uint32_t n, float scale, int rmode, int num_sms,
                           cudaStream_t stream);

constexpr int ATT_MAX_SEG = 128;  // segments one attention launch takes

// One segment of an attention launch: T frames; its q, o (and, laid out as
// rows, K and V) rows from frame f; its P rows from row p; its CTAs from
// item0 (H blocks of queries a head).
struct AttSeg {
    uint32_t T, f, p, item0;
};

struct AttArgs {
    float* o;
    const float *q, *k, *p, *v, *bu, *bv;
    unsigned long long os, qs, ks, ps, vs;  // row strides, in floats (rows layout)
    uint32_t dk, nseg, items;
    uint32_t sp;  // the scores' shared-memory row length (T rounded up to 16)
    AttSeg seg[ATT_MAX_SEG];
};

// Shared memory a CTA takes for heads of dk and score rows of sp floats.
size_t attention_smem(uint32_t dk, uint32_t sp);
uint32_t attention_block();  // queries a CTA
// panels: K, P, V as the reference's panels (one segment); else as rows.
cudaError_t launch_attention(const AttArgs& a, bool panels, int rmode, cudaStream_t stream);
// Lets the attention kernels take the device's largest shared memory (once,
// at the device's set-up).
cudaError_t prepare_attention();
// The dynamic shared memory an attention CTA may take (set by prepare_attention).
size_t attention_smem_max();

// ------------------------------------------------ the TDT search (pkb_tdt.cu) --

enum { TDT_LSTM = 0, TDT_JOINT_IN = 1, TDT_STEP = 2 };

// A lockstep search's buffers (device) and shapes; pkb_tdt.cu's kernels
// take it by value.
struct TdtArgs {
    uint32_t S, P, J, V, n_dur, max_symbols, nout, cap;
    uint32_t dur[16];
    const uint32_t *T, *f0;  // [S] frames, first frame row
    const float* f;          // the joint's encoder half, rows of J
    void* seg;               // [S] search states
    uint32_t* ntok;          // [S] tokens emitted
    int32_t* toks;           // [S][cap][3] id, frame, duration
    const int8_t* qembed;    // [V + 1][P] the embedding quantized a row a block
    const float* dembed;     // [V + 1]
    int8_t* qx;              // [S][P] the first layer's input
    float* dx;               // [S]
    float *h, *c;            // [L][S][P]
    int8_t* qh;              // [L][S][P] h quantized
    float* dh;               // [L][S]
    float* gates;            // [S][4P]
    float *gp, *gpn;         // [S][J] jpred of the prediction, and its next value
    int8_t* qz;              // [S][J] the joint's input quantized
    float* dz;               // [S]
    float* logits;           // [S][nout]
};

cudaError_t launch_tdt_init(const TdtArgs& a, cudaStream_t stream);
cudaError_t launch_tdt(const TdtArgs& a, int phase, uint32_t l, int rmode, cudaStream_t stream);

// The whole search as one cooperative launch (pkb_tdt.cu): the weights, the
// grid barrier's words and the bound on rounds, beside TdtArgs.
constexpr int TDT_MAX_L = 4;
struct TdtPersist {
    uint32_t L;
    const int8_t *wx[TDT_MAX_L], *wh[TDT_MAX_L];  // [4P][P] rows
    const float *wxs[TDT_MAX_L], *whs[TDT_MAX_L], *lb[TDT_MAX_L];
    const int8_t* jpred;  // [J][P]
    const float *jpreds, *jpredb;
    const int8_t* jout;   // [nout][J]
    const float *jouts, *joutb;
    unsigned long long* keys;  // [2][S][2] each running segment's best token and duration (jout's, by round parity)
    unsigned* bar;        // arrivals at the grid's barriers (zero at launch)
    int* abort;           // set by a CTA whose wait gave up (zero at launch)
    uint32_t* err;        // the device error word
    long long timeout;    // SM clock cycles a barrier wait may last
    uint32_t max_rounds;
};
// Shared memory a CTA of the persistent search takes (0: the shapes do not fit).
size_t tdt_persist_smem(const TdtArgs& a, size_t smem_max);
// CTAs the search may run (all resident at once) on a device of `sms` SMs; 0 where none fits.
int tdt_persist_grid(const TdtArgs& a, int rmode, int sms, size_t smem);
cudaError_t launch_tdt_persist(const TdtArgs& a, const TdtPersist& p, int rmode, int grid, size_t smem,
                               cudaStream_t stream);
size_t tdt_seg_bytes();  // one segment's search state
// the 32-bit words of a search state the host reads back: still searching,
// out of token room, joint steps taken
constexpr int TDT_SEG_ACTIVE = 4, TDT_SEG_OVER = 7, TDT_SEG_STEPS = 8;

cudaError_t launch_repack_q8(int8_t* wpack, const int8_t* w_pk, uint32_t rows, uint32_t n, int num_sms,
                             cudaStream_t stream);

}  // namespace pkb
