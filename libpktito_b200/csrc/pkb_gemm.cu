// The int8 product of libpktito on B200's tensor cores (sm_100a).
//
// Computes, for frames t < T and output rows r < rows (the reference's
// k_gemm_q8, backend/ref/kernels.c:66-86, contract backend/kernels.h:60-78):
//
//   acc = +0
//   for each block b of qb inputs, in order:
//       s   = sum of w(r, k) * q(t, k) over the block   (exact int32)
//       acc = fma((float)s, d(t, b), acc)
//   v = acc * ws[r];  v = v + bias[r] if bias;  out[t*os + r] = add ? out + v : v
//
// every float operation rounded once in the rounding mode RM.
//
// Mapping onto the hardware. The block sums are what a tcgen05.mma of
// kind::i8 computes: one MMA of K = 32 is exactly one block of 32 inputs,
// two accumulating MMAs one block of 64, and so on. Each block's int32 sums
// land in a fresh accumulator of a ring of four in tensor memory (TMEM,
// 4 x 128 columns of its 512), so the float chain, which must see every
// block's sum on its own and in order, reads them one block at a time. The
// tile is 128 frames (TMEM lanes, the MMA's M) by 128 output rows (TMEM
// columns, the MMA's N).
//
// The int -> float conversion of a sum costs the chain no extra pass: before
// a block's i8 MMAs, one kind::f16 MMA of constant bf16 tiles (16 products
// 1536 x 512 a cell, all exact) writes the float 1.5 * 2^23 = 12582912,
// bits 0x4B400000, into every cell of the block's accumulator; the i8 MMAs
// add the integer sum to those bits, so each word read back is the float
// 1.5 * 2^23 + s, and one exact subtraction gives (float)s (|s| < 2^22,
// i.e. qb <= 256; wider blocks start from zero and convert in the mode).
//
// Warp roles in a 608-thread CTA, one CTA per SM (its 219 KB of shared
// memory keeps a second off), persistent over the tiles:
//   warp 16    TMA producer: 128-byte-swizzled 128x128 tiles of activations
//              and weights into a 4-stage shared-memory ring, and the
//              activation scales into their own ring
//   warps 17, 18  one thread each issues the MMAs and commits of alternate
//              blocks (warp 17 alone where a stage does not hold whole
//              blocks); warp 17 allocates TMEM
//   warps 0-15 the epilogue: warp w reads TMEM lanes 32*(w%4).. (the
//              quarter its hardware warp slot may access) and columns
//              32*(w/4)..+31 of each block's accumulator, hands the slot back
//              as soon as its loads have landed, and runs the float chain of
//              its frame's 32 output rows in registers, two rows a packed
//              f32x2 instruction; after the tile's last block it scales,
//              biases, adds and stores them.
//
// The fp32 chain is the bound at 32-input blocks, not the tensor core: per
// block and output it is one subtraction and one FMA on the CUDA cores
// (128 lanes a cycle per SM), against 64 tensor-core cycles for the whole
// 128 x 128 x 32 block.
//
// Every wait is bounded: a role that waits past the limit sets the device
// error word and an abort flag the other roles see, waits (bounded) for its
// own copies and MMAs in flight, and the CTA frees its TMEM and returns.

#include "pkb_device.cuh"
#include "pkb_internal.h"

namespace pkb {

namespace gemm {

constexpr int BM = 128;           // frames per tile: TMEM lanes, the MMA's M
constexpr int BN = 128;           // output rows per tile: the MMA's N
constexpr int BK = 128;           // bytes (= int8 inputs) of K per stage: one swizzle row
constexpr int KSTEP = 32;         // K of one kind::i8 MMA
constexpr int NSTAGE = 4;         // shared-memory pipeline depth (16 blocks of 32 ahead)
constexpr int NTMEM = 4;          // block accumulators in TMEM
constexpr int TMEM_COLS = NTMEM * BN;  // 512
#ifndef PKB_EPI_COLS
#define PKB_EPI_COLS 32
#endif
constexpr int EPI_COLS = PKB_EPI_COLS;   // output rows a thread of the epilogue holds (32 or 64)
constexpr int EPI_HALVES = EPI_COLS / 32;  // its groups of 32: TMEM loads a block, staging boxes a tile
constexpr int EPI_WARPS = 4 * (BN / EPI_COLS);  // a warp per lane quarter and column group
constexpr int TMA_WARP = EPI_WARPS;
constexpr int MMA_WARP = EPI_WARPS + 1;   // allocates TMEM; its lane 0 issues the even blocks' MMAs
constexpr int MMA_WARP2 = EPI_WARPS + 2;  // lane 0 issues the odd blocks' MMAs (the staged paths)
constexpr int THREADS = (EPI_WARPS + 3) * 32;
static_assert(EPI_COLS == 32 || EPI_COLS == 64, "a thread's output rows");
constexpr int A_BYTES = BM * BK;
constexpr int B_BYTES = BN * BK;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_PITCH = 33;      // floats a row of an epilogue warp's transpose tile (plain stores)
constexpr int STG_BYTES = 32 * 32 * 4;  // a 128-byte-swizzled staging box of 32 x 32 results (TMA stores)
// the epilogue's area: each warp's transpose tile (plain stores, a group of
// 32 at a time) or its EPI_HALVES staging boxes (TMA stores)
constexpr int EPI_BYTES = EPI_WARPS * 32 * EPI_PITCH * 4 > EPI_WARPS * EPI_HALVES * STG_BYTES
                              ? EPI_WARPS * 32 * EPI_PITCH * 4
                              : EPI_WARPS * EPI_HALVES * STG_BYTES;
constexpr int CHUNK = 4;           // blocks a turn of the TMEM ring
constexpr int DBLK = 16;           // blocks of scales a TMA box of d carries (64 bytes a frame)
constexpr int NDS = 2;             // slots of the scales ring (16 blocks ahead)
constexpr int DS_BYTES = BM * DBLK * 4;
constexpr int WS_BYTES = 2 * BN * 4;  // a tile's row scales, then its biases
constexpr int NWS = 2;             // slots of their ring (a tile each)
constexpr int SEED_K = 16;         // K of the bf16 MMA that writes the accumulator's start value
constexpr int WIDE = 8;            // SPB of the staged path for blocks of whole stages (qb = 256, 384, ...)
constexpr int SEED_BYTES = 128 * SEED_K * 2;  // one 128-row bf16 operand tile of it
constexpr int BAR_BYTES = 512;
constexpr int SMEM_BYTES =
    NSTAGE * STAGE_BYTES + EPI_BYTES + NDS * DS_BYTES + NWS * WS_BYTES + 2 * SEED_BYTES + BAR_BYTES +
    1024;  // + alignment slack

static_assert(TMEM_COLS == 512, "TMEM ring must fit the SM's 512 columns");
static_assert((2 * NSTAGE + 4 + NTMEM + 2 + EPI_WARPS + 2 * NDS + 2 * NWS) * 8 + 8 <= BAR_BYTES, "barrier area");
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory of one CTA");

// The float 1.5 * 2^23, whose bits 0x4B400000 plus an int32 |s| < 2^22 are
// the float 1.5 * 2^23 + s. The start-value MMA writes it as the sum of
// SEED_K products SEED_A * SEED_B, every partial sum an exact integer.
constexpr float SUM_BIAS_F = 12582912.0f;
constexpr uint16_t SEED_A = 0x44C0;  // bf16 1536
constexpr uint16_t SEED_B = 0x4400;  // bf16 512
static_assert(1536.0 * 512.0 * SEED_K == 12582912.0, "start value");

// The EPI_COLS running sums of a thread (its frame x the warp's output
// rows), two rows a 64-bit register, for the f32x2 instructions.
using Acc = uint64_t[EPI_COLS / 2];

// acc[16 h + i] = fma(float(s), d, acc[16 h + i]) for the 32 block sums of
// the warp's column group h, two an instruction, each rounded once in the
// mode RM.
template <int RM, bool EXACT_SUM>
__device__ __forceinline__ void chain32(Acc& acc, const uint32_t (&s)[32], float dv, int h) {
    const uint64_t d2 = pack2(dv, dv);
    const uint64_t bias2 = pack2(-SUM_BIAS_F, -SUM_BIAS_F);
#pragma unroll
    for (int i = 0; i < 16; i++) {
        uint64_t f;
        if constexpr (EXACT_SUM)
            // each word is the float 1.5 * 2^23 + s; less 1.5 * 2^23, rounded
            // to nearest, it is exactly s (+0 for a zero sum)
            f = add2_rn(pack2(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1])), bias2);
        else
            f = pack2(i2f_r<RM>(static_cast<int>(s[2 * i])), i2f_r<RM>(static_cast<int>(s[2 * i + 1])));
        acc[16 * h + i] = fma2_r<RM>(f, d2, acc[16 * h + i]);
    }
}

__device__ __forceinline__ float acc_at(const Acc& acc, int j) {
    float lo, hi;
    unpack2(acc[j / 2], lo, hi);
    return (j & 1) ? hi : lo;
}

// The whole warp waits for `bar`'s phase: every lane polls the barrier, so
// the warp stays converged for the whole-warp TMEM loads that follow, with
// no branch around one lane's wait and no shuffle (measured on B200: a
// lane-0 wait and a shuffle cost the epilogue a third of its time at
// 32-input blocks). Every lane runs the same polls on the same barrier, abort
// flag and clock, so all take the loop's exit together and no further
// warp-wide synchronisation is needed (one cost 2-3 %). False if the wait
// gave up. POLL: test_wait in a loop instead of try_wait's suspended wait
// (measured on B200: 1.7 % faster on blocks of 32 and 64, 5 % slower on
// blocks of whole stages, whose waits are longer).
template <bool POLL>
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, long long limit) {
    if constexpr (POLL)
        return mbar_poll(bar, parity, abort, limit);
    else
        return mbar_wait(bar, parity, abort, limit);
}

// Block accumulators are handed over one at a time: block B (counted over
// all of a CTA's tiles) lives in TMEM slot B % 4 and is announced by its
// own commit on tfull[B % 4]. The epilogue waits for each block and releases
// each slot as soon as it has been loaded. (A commit a pair of blocks, one
// wait fewer a pair, held the pair's first block back until the second was
// done: measured on B200 the one commit a block is 1.4 % faster on FF-up and
// 8 % on the joint's blocks of whole stages; waiting for whole turns of the
// ring leaves the MMAs of a turn's last blocks too little time.)
//
// One block's accumulator (the warp's 32 columns at ta) out of TMEM, after
// its wait: loads, hands the slot back to the MMA threads and runs the
// chain.
template <int RM, bool EXACT_SUM>
__device__ __forceinline__ void epi_block(Acc& acc, uint32_t ta, float dv, uint64_t* tempty) {
    uint32_t sv[EPI_HALVES][32];
    // one load of each 32 columns (two of 16 cost 2 % more), all in flight
    // before the one wait
#pragma unroll
    for (int h = 0; h < EPI_HALVES; h++) tmem_ld_32x32b_x32(ta + 32 * h, sv[h]);
    tmem_ld_wait(sv[0]);
#pragma unroll
    for (int h = 1; h < EPI_HALVES; h++) tmem_ld_settled(sv[h]);
    // every thread orders its own loads before its own arrival (the slot's
    // barrier counts all the epilogue's threads): no warp-wide step between
    tc_fence_before();
    mbar_arrive(tempty);
#pragma unroll
    for (int h = 0; h < EPI_HALVES; h++) chain32<RM, EXACT_SUM>(acc, sv[h], dv, h);
}

// Where result (frame t, output row r) goes on the plain-store path: the
// rows of out, or V's panels (pk_gemm_panels_on, core/passes.c:119-141:
// panel r/16 at (r/16) ps, its frames 16 floats apart).
__device__ __forceinline__ size_t out_at(const GemmArgs& g, uint32_t t, uint32_t r) {
    if (g.pmode == 1) return static_cast<size_t>(r >> 4) * g.ps + 16 * static_cast<size_t>(t) + (r & 15);
    return static_cast<size_t>(t) * g.os + r;
}

// SPB: K steps a block (1, 2 or 4, with n a multiple of BK: every stage
// starts a block and holds four K steps), WIDE (qb a multiple of BK, at least
// 2 BK, with n a multiple of BK: a block spans whole stages, as qb = n does
// for the decoder's and the joint's products), or 0 for any qb and n.
// OM, where the results go: 0 plain loads and stores (rows or panels by
// g.pmode, through out_at); otherwise (the results' rows and the row scales
// and biases whole 16-byte units) the row scales and biases come through a
// bulk-copy ring and the results leave through TMA stores of map_o: 1 rows,
// 2 V panels, 3 K/P panels; and, except on the WIDE path (a few blocks a
// tile, each hundreds of tensor-core cycles long), the block scales come
// through a TMA ring (map_d; a multiple of four blocks a tile, the scales'
// rows whole 16-byte units). The epilogue's loop
// then holds no global load (on B200 a global load in flight there costs the
// chain as much as one waited for at once). The panel layouts are separate
// instances: a run-time choice in the store code cost the rows' instance 9 %
// on B200.
template <int RM, bool EXACT_SUM, int OM, int SPB>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_q8_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const __grid_constant__ CUtensorMap map_d, const __grid_constant__ CUtensorMap map_o,
                   const GemmArgs g) {
    constexpr bool TIO = OM != 0;
    constexpr bool DRING = TIO && SPB != WIDE;  // block scales through the TMA ring
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* epi = reinterpret_cast<float*>(smem + NSTAGE * STAGE_BYTES);
    float* dring = reinterpret_cast<float*>(smem + NSTAGE * STAGE_BYTES + EPI_BYTES);
    float* wsring = reinterpret_cast<float*>(smem + NSTAGE * STAGE_BYTES + EPI_BYTES + NDS * DS_BYTES);
    uint8_t* seed = smem + NSTAGE * STAGE_BYTES + EPI_BYTES + NDS * DS_BYTES + NWS * WS_BYTES;  // A tile, B tile
    uint64_t* full = reinterpret_cast<uint64_t*>(seed + 2 * SEED_BYTES);
    uint64_t* empty = full + NSTAGE;
    uint64_t* tfull = empty + NSTAGE;  // [4]: a block's accumulator done, a slot each
    uint64_t* tempty = tfull + 4;
    uint64_t* drain = tempty + NTMEM;  // one for each MMA thread
    uint64_t* obar = drain + 2;      // an epilogue warp's load of the results it adds to
    uint64_t* dfull = obar + EPI_WARPS;
    uint64_t* dempty = dfull + NDS;
    uint64_t* wsfull = dempty + NDS;
    uint64_t* wsempty = wsfull + NWS;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(wsempty + NWS);
    volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NSTAGE; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], SPB ? 2 : 1);  // both MMA threads release a stage on the staged paths
        }
        for (int i = 0; i < 4; i++) mbar_init(&tfull[i], 1);
        for (int i = 0; i < NTMEM; i++) mbar_init(&tempty[i], EPI_WARPS * 32);
        mbar_init(&drain[0], 1);
        mbar_init(&drain[1], 1);
        for (int i = 0; i < EPI_WARPS; i++) mbar_init(&obar[i], 1);
        for (int i = 0; i < NDS; i++) {
            mbar_init(&dfull[i], 1);
            mbar_init(&dempty[i], EPI_WARPS);
        }
        for (int i = 0; i < NWS; i++) {
            mbar_init(&wsfull[i], 1);
            mbar_init(&wsempty[i], EPI_WARPS);
        }
        *abort = 0;
        fence_mbar_init();
    }
    if (EXACT_SUM && warp < EPI_WARPS) {
        // the start-value MMA's operand tiles: every bf16 of A 1536, of B 512
        uint32_t* sw = reinterpret_cast<uint32_t*>(seed);
        for (int i = threadIdx.x; i < SEED_BYTES / 4; i += EPI_WARPS * 32) {
            sw[i] = (uint32_t(SEED_A) << 16) | SEED_A;
            sw[SEED_BYTES / 4 + i] = (uint32_t(SEED_B) << 16) | SEED_B;
        }
        // written through the generic proxy, read by the tensor core
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == MMA_WARP) {
        tmem_alloc(tslot, TMEM_COLS);
        tmem_relinquish();
    }
    if (warp == TMA_WARP && lane == 0) {
        tma_prefetch_map(&map_a);
        tma_prefetch_map(&map_b);
        if constexpr (DRING) tma_prefetch_map(&map_d);
        if constexpr (TIO) tma_prefetch_map(&map_o);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;
    // set up: the next kernel may launch now; this one reads and writes
    // global memory only once the one before has completed
    pdl_trigger();
    pdl_wait();

    const uint32_t nk = g.n / KSTEP;            // K steps of a tile
    const uint32_t nc = (g.n + BK - 1) / BK;     // shared-memory stages of a tile
    const uint32_t spb = g.qb / KSTEP;          // K steps a block
    const uint32_t nb = g.n / g.qb;             // blocks
    const uint32_t ntiles = g.tiles_m * g.tiles_n;
    const long long limit = g.timeout;

    if (warp == TMA_WARP) {
        if (lane == 0) {
            uint32_t it = 0, dcnt = 0, wcnt = 0;
            const uint32_t nchunks = (nb + DBLK - 1) / DBLK;
            bool ok = true;
            for (uint32_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
                const int m0 = static_cast<int>((tile / g.tiles_n) * BM);
                const int n0 = static_cast<int>((tile % g.tiles_n) * BN);
                if constexpr (TIO) {
                    // the tile's row scales and biases (rows a multiple of 16,
                    // so every copy is whole 64-byte units)
                    const uint32_t wsl = wcnt % NWS;
                    if (!mbar_wait(&wsempty[wsl], ((wcnt / NWS) & 1) ^ 1, abort, limit)) {
                        ok = false;
                        break;
                    }
                    const uint32_t ncol = g.rows - n0 < static_cast<uint32_t>(BN) ? g.rows - n0 : BN;
                    mbar_arrive_expect_tx(&wsfull[wsl], (g.bias ? 2 : 1) * ncol * 4);
                    float* wd = wsring + wsl * (WS_BYTES / 4);
                    bulk_load(wd, g.ws + n0, ncol * 4, &wsfull[wsl]);
                    if (g.bias) bulk_load(wd + BN, g.bias + n0, ncol * 4, &wsfull[wsl]);
                    wcnt++;
                }
                uint32_t dk = 0;  // the tile's next chunk of scales
                for (uint32_t c = 0; ok && c < nc; c++, it++) {
                    if constexpr (DRING) {
                        // the scales of every chunk of blocks starting in this
                        // stage's K range, into the scales ring (the box's x,
                        // a multiple of 8 floats, is 16-byte aligned; blocks
                        // past n / qb read as zeros)
                        while (dk < nchunks && DBLK * dk * g.qb < (c + 1) * BK) {
                            const uint32_t ds = dcnt % NDS;
                            if (!mbar_wait(&dempty[ds], ((dcnt / NDS) & 1) ^ 1, abort, limit)) {
                                ok = false;
                                break;
                            }
                            mbar_arrive_expect_tx(&dfull[ds], DS_BYTES);
                            tma_load_2d(&map_d, reinterpret_cast<uint8_t*>(dring) + ds * DS_BYTES, &dfull[ds],
                                        static_cast<int>(DBLK * dk), m0);
                            dk++;
                            dcnt++;
                        }
                        if (!ok) break;
                    }
                    const uint32_t s = it % NSTAGE, ph = (it / NSTAGE) & 1;
                    if (!mbar_wait(&empty[s], ph ^ 1, abort, limit)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
                    uint8_t* sa = smem + s * STAGE_BYTES;
                    tma_load_2d(&map_a, sa, &full[s], static_cast<int>(c * BK), m0);
                    tma_load_2d(&map_b, sa + A_BYTES, &full[s], static_cast<int>(c * BK), n0);
                }
            }
            if (!ok) {
                *abort = 1;
                atomicOr(g.err, PKB_DEVERR_TIMEOUT);
                // the copies this role issued and nobody consumed: let them land
                const uint32_t back = it < NSTAGE ? it : NSTAGE;
                for (uint32_t i = it - back; i < it; i++)
                    mbar_drain(&full[i % NSTAGE], (i / NSTAGE) & 1, limit);
                const uint32_t dback = dcnt < NDS ? dcnt : NDS;
                for (uint32_t i = dcnt - dback; i < dcnt; i++)
                    mbar_drain(&dfull[i % NDS], (i / NDS) & 1, limit);
                const uint32_t wback = wcnt < NWS ? wcnt : NWS;
                for (uint32_t i = wcnt - wback; i < wcnt; i++)
                    mbar_drain(&wsfull[i % NWS], (i / NWS) & 1, limit);
            }
        }
    } else if (warp == MMA_WARP || warp == MMA_WARP2) {
        // one TMEM-full commit a block; block accumulators ring through the
        // NTMEM slots. Every count is stepped, none divided, and the
        // descriptors are stepped by adding offsets.
        const uint32_t me = warp == MMA_WARP ? 0u : 1u;
        if (lane == 0 && (SPB != 0 || me == 0)) {
            constexpr uint32_t idesc = i8_instr_desc(BM, BN);
            constexpr uint32_t sdesc_i = bf16_instr_desc(BM, BN);
            const uint64_t desc0 = sw128_kmajor_desc(smem_u32(smem));
            // the start-value tiles: K-major without swizzle, core matrices
            // 128 bytes apart along K and 256 bytes apart along the rows
            const uint64_t seed_a = plain_kmajor_desc(smem_u32(seed), 128, 256);
            const uint64_t seed_b = plain_kmajor_desc(smem_u32(seed + SEED_BYTES), 128, 256);
            uint32_t s = 0, sph = 0;  // stage, its phase
            bool ok = true;
            // Block B (counted over all tiles) goes to TMEM slot B % 4; the
            // slot's previous block B - 4 must have been read out first
            // (phase ((B / 4) & 1) ^ 1 of tempty[B % 4]); block B is
            // committed on tfull[B % 4] after its MMAs.
            uint32_t blk = 0;  // blocks issued or passed (all tiles)
            auto blk_bar = [&](uint32_t b) { return &tfull[b & 3]; };
            if constexpr (SPB == WIDE) {
                // Blocks of whole stages: a stage holds four K steps of one
                // block, unrolled; block b's pair goes to thread (b / 2) & 1,
                // which issues all its stages; the other thread passes them
                // (both release every stage).
                const uint32_t spc = g.qb / BK;  // stages a block
                for (uint32_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
                    uint32_t kst = 0;  // the stage's place in its block
                    for (uint32_t c = 0; c < nc && ok; c++) {
                        if (!mbar_wait(&full[s], sph, abort, limit)) {
                            ok = false;
                            break;
                        }
                        const uint32_t b = blk;
                        if (((b >> 1) & 1) == me) {
                            const uint64_t adesc = desc0 + ((s * STAGE_BYTES) >> 4);
                            const uint64_t bdesc = adesc + (A_BYTES >> 4);
                            const uint32_t slot = b & (NTMEM - 1);
                            const uint32_t ta = tbase + slot * BN;
                            if (kst == 0) {
                                if (!mbar_wait(&tempty[slot], ((b >> 2) & 1) ^ 1, abort, limit)) {
                                    ok = false;
                                    break;
                                }
                                tc_fence_after();
                                if constexpr (EXACT_SUM) umma_bf16(ta, seed_a, seed_b, sdesc_i, 0u);
                            }
#pragma unroll
                            for (uint32_t j = 0; j < 4; j++)
                                umma_i8(ta, adesc + 2 * j, bdesc + 2 * j, idesc, EXACT_SUM ? 1u : (kst | j));
                            if (kst + 1 == spc) umma_commit(blk_bar(b));
                        }
                        umma_commit(&empty[s]);
                        if (++kst == spc) {
                            kst = 0;
                            blk++;
                        }
                        if (++s == NSTAGE) {
                            s = 0;
                            sph ^= 1;
                        }
                    }
                }
            } else if constexpr (SPB != 0) {
                // Staged: every stage starts a block and holds 4 / SPB whole
                // blocks; pair P goes to thread P & 1, so each thread issues
                // into two slots of its own and the two threads' MMAs,
                // commits and waits overlap (the issuing thread, not the
                // tensor core, paces a lone thread at 32-input blocks). The
                // stage's K steps are unrolled.
                constexpr uint32_t BPS = 4 / SPB;  // blocks a stage
                for (uint32_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
                    for (uint32_t c = 0; c < nc && ok; c++) {
                        if (!mbar_wait(&full[s], sph, abort, limit)) {
                            ok = false;
                            break;
                        }
                        const uint64_t adesc = desc0 + ((s * STAGE_BYTES) >> 4);
                        const uint64_t bdesc = adesc + (A_BYTES >> 4);
#pragma unroll
                        for (uint32_t k = 0; k < BPS; k++) {
                            const uint32_t b = blk + k;
                            if (((b >> 1) & 1) != me) continue;
                            const uint32_t slot = b & (NTMEM - 1);
                            const uint32_t ta = tbase + slot * BN;
                            if (!mbar_wait(&tempty[slot], ((b >> 2) & 1) ^ 1, abort, limit)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            if constexpr (EXACT_SUM) umma_bf16(ta, seed_a, seed_b, sdesc_i, 0u);
#pragma unroll
                            for (uint32_t j = 0; j < SPB; j++)
                                umma_i8(ta, adesc + 2 * (k * SPB + j), bdesc + 2 * (k * SPB + j), idesc,
                                        EXACT_SUM ? 1u : j);
                            umma_commit(blk_bar(b));
                        }
                        if (!ok) break;
                        umma_commit(&empty[s]);
                        blk += BPS;
                        if (++s == NSTAGE) {
                            s = 0;
                            sph ^= 1;
                        }
                    }
                }
            } else {
                // any qb and n, one thread
                for (uint32_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
                    uint32_t kpos = 0;   // K step in its block
                    uint32_t left = nk;  // K steps of the tile still to issue
                    for (uint32_t c = 0; c < nc && ok; c++) {
                        if (!mbar_wait(&full[s], sph, abort, limit)) {
                            ok = false;
                            break;
                        }
                        const uint64_t adesc = desc0 + ((s * STAGE_BYTES) >> 4);
                        const uint64_t bdesc = adesc + (A_BYTES >> 4);
                        const uint32_t jn = left < 4 ? left : 4;
                        left -= jn;
                        for (uint32_t j = 0; j < jn; j++) {
                            const uint32_t slot = blk & (NTMEM - 1);
                            const uint32_t ta = tbase + slot * BN;
                            if (kpos == 0) {
                                if (!mbar_wait(&tempty[slot], ((blk >> 2) & 1) ^ 1, abort, limit)) {
                                    ok = false;
                                    break;
                                }
                                tc_fence_after();
                                if constexpr (EXACT_SUM) umma_bf16(ta, seed_a, seed_b, sdesc_i, 0u);
                            }
                            // onto the start value when sums convert exactly, else from zero
                            umma_i8(ta, adesc + 2 * j, bdesc + 2 * j, idesc, EXACT_SUM ? 1u : kpos);
                            if (++kpos == spb) {
                                kpos = 0;
                                umma_commit(blk_bar(blk));
                                blk++;
                            }
                        }
                        umma_commit(&empty[s]);
                        if (++s == NSTAGE) {
                            s = 0;
                            sph ^= 1;
                        }
                    }
                }
            }
            if (!ok) {
                *abort = 1;
                atomicOr(g.err, PKB_DEVERR_TIMEOUT);
                // the MMAs this thread issued: let them finish before TMEM is freed
                umma_commit(&drain[me]);
                mbar_drain(&drain[me], 0, limit);
            }
        }
    } else {
        // epilogue: frame t of the tile is this thread's TMEM lane
        const uint32_t quarter = warp & 3, cgroup = warp >> 2;
        const uint32_t lane_base = 32 * quarter;
        const uint32_t tl = tbase + (lane_base << 16) + EPI_COLS * cgroup;
        float* tw = epi + warp * (32 * EPI_PITCH);  // this warp's 32 x 32 transpose tile
        // its staging boxes, one a group of 32 output rows (1024-aligned)
        uint8_t* stg = reinterpret_cast<uint8_t*>(epi) + warp * EPI_HALVES * STG_BYTES;
        uint32_t gb = 0;            // blocks consumed (all tiles)
        uint32_t dcnt = 0, wcnt = 0;  // scale chunks, row-scale slots consumed
        uint32_t ocnt = 0;          // loads of results to add to
        bool ok = true;
        for (uint32_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
            const uint32_t m0 = (tile / g.tiles_n) * BM;
            const uint32_t n0 = (tile % g.tiles_n) * BN;
            const uint32_t t = m0 + lane_base + lane;
            const bool tvalid = t < g.T;
            const float* drow = g.d + static_cast<size_t>(tvalid ? t : 0) * nb;

            Acc acc;
#pragma unroll
            for (int j = 0; j < EPI_COLS / 2; j++) acc[j] = 0;  // +0, +0

            // the warp's boxes of the results: group h is 32 output rows from
            // col0 + 32 h by 32 frames from frame0; a group past the last row
            // is not stored (the groups that are live come first); K/P panels
            // also take the padding's frames, as zeros
            const uint32_t col0 = n0 + EPI_COLS * cgroup, frame0 = m0 + lane_base;
            const bool live = col0 < g.rows && frame0 < (OM == 3 ? g.tpad : g.T);
            uint32_t nlive = 0;
#pragma unroll
            for (int h = 0; h < EPI_HALVES; h++) nlive += (live && col0 + 32 * h < g.rows) ? 1u : 0u;
            if constexpr (TIO) {
                if (g.add && live && lane == 0) {
                    // the results added to, into the staging boxes once the
                    // previous tile's stores have read them
                    bulk_wait_read();
                    mbar_arrive_expect_tx(&obar[warp], nlive * STG_BYTES);
                    for (uint32_t h = 0; h < nlive; h++)
                        tma_load_2d(&map_o, stg + h * STG_BYTES, &obar[warp], static_cast<int>(col0 + 32 * h),
                                    static_cast<int>(frame0));
                }
            }

            if constexpr (DRING) {
                // four blocks an iteration, a wait each; the frame's four scales
                // one 16-byte shared load out of the chunk of DBLK blocks
                // the scales ring holds (one wait a chunk)
                for (uint32_t b = 0; b < nb; b += CHUNK) {
                    const uint32_t ds = dcnt % NDS;
                    if ((b & (DBLK - 1)) == 0 && !warp_wait<DRING>(&dfull[ds], (dcnt / NDS) & 1, abort, limit)) {
                        ok = false;
                        break;
                    }
                    const float4 dq = *reinterpret_cast<const float4*>(dring + ds * (DS_BYTES / 4) +
                                                                       (lane_base + lane) * DBLK + (b & (DBLK - 1)));
                    if ((b & (DBLK - 1)) == DBLK - CHUNK || b + CHUNK >= nb) {
                        // the chunk's last use (or the tile's): the slot goes back
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&dempty[ds]);
                        dcnt++;
                    }
                    const uint32_t tph = (gb >> 2) & 1;
                    const float dv4[4] = {dq.x, dq.y, dq.z, dq.w};
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        if (!warp_wait<DRING>(&tfull[k], tph, abort, limit)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        epi_block<RM, EXACT_SUM>(acc, tl + k * BN, dv4[k], &tempty[k]);
                    }
                    if (!ok) break;
                    gb += CHUNK;
                }
            } else {
                // one block at a time, the frame's scales from global memory,
                // one block ahead
                float dnext = (tvalid && nb > 0) ? __ldg(drow) : 0.0f;
                for (uint32_t b = 0; b < nb; b++, gb++) {
                    const float dv = dnext;
                    dnext = (tvalid && b + 1 < nb) ? __ldg(drow + b + 1) : 0.0f;
                    if (!warp_wait<DRING>(&tfull[gb & 3], (gb >> 2) & 1, abort, limit)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t slot = gb & (NTMEM - 1);
                    epi_block<RM, EXACT_SUM>(acc, tl + slot * BN, dv, &tempty[slot]);
                }
            }
            if (!ok) break;

            if constexpr (TIO) {
                // Lane i holds frame frame0 + i, i.e. row i of the box, 128
                // bytes of results: into the staging box (its 16-byte chunks
                // swizzled by the row, as the tensor map's 128-byte swizzle
                // lays them out, so the 16-byte stores of a quarter-warp hit
                // distinct banks), then one TMA store of the box while the
                // warp goes on with the next tile.
                // the tile's row scales and biases, one a lane
                const uint32_t wsl = wcnt % NWS;
                if (!warp_wait<DRING>(&wsfull[wsl], (wcnt / NWS) & 1, abort, limit)) {
                    ok = false;
                    break;
                }
                const float* wsv = wsring + wsl * (WS_BYTES / 4) + EPI_COLS * cgroup;
                float ws_l[EPI_HALVES], b_l[EPI_HALVES];
#pragma unroll
                for (int h = 0; h < EPI_HALVES; h++) {
                    const bool in = col0 + 32 * h + lane < g.rows;
                    ws_l[h] = in ? wsv[32 * h + lane] : 0.0f;
                    b_l[h] = (g.bias && in) ? wsv[BN + 32 * h + lane] : 0.0f;
                }
                // the slot goes back now (K/P panels: once staged, as their
                // staging reads the row scales from it)
                if constexpr (OM != 3) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&wsempty[wsl]);
                }
                wcnt++;
                if (live) {
                    if (g.add) {
                        if (!warp_wait<DRING>(&obar[warp], ocnt & 1, abort, limit)) {
                            ok = false;
                            break;
                        }
                        ocnt++;
                    } else {
                        if (lane == 0) bulk_wait_read();
                        __syncwarp();
                    }
#pragma unroll
                    for (int h = 0; h < EPI_HALVES; h++) {
                        if (h >= static_cast<int>(nlive)) break;  // warp-uniform
                        uint8_t* box = stg + h * STG_BYTES;
                        if constexpr (OM == 2) {
                            // V panels (pk_gemm_panels_on, core/passes.c:119-141):
                            // the box is 2 panels x 32 frames x 16 output rows,
                            // 64-byte rows whose 16-byte chunks the map's 64-byte
                            // swizzle permutes by the row (bank-conflict free
                            // for a quarter-warp); frames past T are clipped
#pragma unroll
                            for (int rp = 0; rp < 2; rp++) {
#pragma unroll
                                for (int k = 0; k < 4; k++) {
                                    float v[4];
#pragma unroll
                                    for (int e = 0; e < 4; e++) {
                                        const int j = 16 * rp + 4 * k + e;
                                        v[e] = mul_r<RM>(acc_at(acc, 32 * h + j), __shfl_sync(0xffffffffu, ws_l[h], j));
                                    }
                                    *reinterpret_cast<float4*>(box + (rp * 32 + lane) * 64 +
                                                               ((k ^ ((lane >> 1) & 3)) << 4)) =
                                        make_float4(v[0], v[1], v[2], v[3]);
                                }
                            }
                            continue;
                        }
                        if constexpr (OM == 3) {
                            // K/P panels (pk_panels_tile, core/passes.c:143-196):
                            // two boxes of 16 dimensions x 2 panels x 16 frames,
                            // one a 16-column half (each within one head); the
                            // padding's frames are zeros. A column pair at a
                            // time: one packed multiply by the pair's row scales
                            // (a broadcast load of the ring), then two stores,
                            // lanes 16-31 (the second panel) storing the pair's
                            // columns the other way round, so a store's 32 lanes
                            // cover 32 distinct banks. The product is not added
                            // to (a packed multiply feeding a packed add would be
                            // fused).
                            const uint32_t half = lane >> 4;
                            const bool pad = frame0 + 32 > g.T;  // warp-uniform
                            const bool real = frame0 + lane < g.T;
                            float* fa = reinterpret_cast<float*>(box) + half * 256 + (lane & 15) + 16 * half;
                            float* fz = reinterpret_cast<float*>(box) + half * 256 + (lane & 15) + 16 - 16 * half;
#pragma unroll
                            for (int i = 0; i < 16; i++) {
                                const uint64_t w2 = *reinterpret_cast<const uint64_t*>(wsv + 32 * h + 2 * i);
                                uint64_t pr = mul2_r<RM>(acc[16 * h + i], w2);
                                if (pad && !real) pr = 0;  // +0, +0
                                float p0, p1;
                                unpack2(pr, p0, p1);
                                const int slot = (i >> 3) * 512 + (2 * i & 15) * 16;  // column 2i's place
                                fa[slot] = half ? p1 : p0;
                                fz[slot] = half ? p0 : p1;
                            }
                            continue;
                        }
                        uint8_t* row = box + lane * 128;
#pragma unroll
                        for (int k = 0; k < 8; k++) {
                            float4* c4 = reinterpret_cast<float4*>(row + ((k ^ (lane & 7)) << 4));
                            float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                            if (g.add) {
                                const float4 ov = *c4;
                                o[0] = ov.x;
                                o[1] = ov.y;
                                o[2] = ov.z;
                                o[3] = ov.w;
                            }
                            float v[4];
#pragma unroll
                            for (int e = 0; e < 4; e++) {
                                const int j = 4 * k + e;
                                v[e] = mul_r<RM>(acc_at(acc, 32 * h + j), __shfl_sync(0xffffffffu, ws_l[h], j));
                                if (g.bias) v[e] = add_r<RM>(v[e], __shfl_sync(0xffffffffu, b_l[h], j));
                                if (g.add) v[e] = add_r<RM>(o[e], v[e]);
                            }
                            *c4 = make_float4(v[0], v[1], v[2], v[3]);
                        }
                    }
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        for (uint32_t h = 0; h < nlive; h++) {
                            const uint32_t c = col0 + 32 * h;
                            if constexpr (OM == 2) {
                                // (row in panel, frame, panel)
                                tma_store_3d(&map_o, stg + h * STG_BYTES, 0, static_cast<int>(frame0),
                                             static_cast<int>(c >> 4));
                            } else if constexpr (OM == 3) {
                                // (frame in panel, dimension, panel, head) a half;
                                // rows a multiple of 16, so a half is all in or out
                                for (uint32_t s = 0; s < 2 && c + 16 * s < g.rows; s++) {
                                    const uint32_t cs = c + 16 * s, hd = cs / g.dk;
                                    tma_store_4d(&map_o, stg + h * STG_BYTES + s * 2048, 0,
                                                 static_cast<int>(cs - hd * g.dk), static_cast<int>(frame0 >> 4),
                                                 static_cast<int>(hd));
                                }
                            } else {
                                tma_store_2d(&map_o, stg + h * STG_BYTES, static_cast<int>(c), static_cast<int>(frame0));
                            }
                        }
                        bulk_commit();
                    }
                }
                if constexpr (OM == 3) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&wsempty[wsl]);
                }
            } else if (g.pmode == 2) {
                // K and P panels (pk_panels_tile, core/passes.c:143-196): frame
                // t, dimension d of head h at h tpad dk + (t/16) 16 dk + 16 d +
                // t%16, frames T .. tpad-1 zeros; from the sums as they are (a
                // lane a frame), so 16 lanes store 64 contiguous bytes. The
                // reference's K and P products have no bias and add nothing.
                const uint32_t tt = frame0 + lane;
                float ws_l[EPI_HALVES];
#pragma unroll
                for (int h = 0; h < EPI_HALVES; h++)
                    ws_l[h] = col0 + 32 * h + lane < g.rows ? __ldg(g.ws + col0 + 32 * h + lane) : 0.0f;
#pragma unroll
                for (int j = 0; j < EPI_COLS; j++) {
                    const uint32_t col = col0 + j;
                    const float w = __shfl_sync(0xffffffffu, ws_l[j / 32], j % 32);
                    if (col < g.rows && tt < g.tpad) {
                        const float v = tt < g.T ? mul_r<RM>(acc_at(acc, j), w) : 0.0f;
                        const uint32_t hd = col / g.dk, dd = col - hd * g.dk;
                        g.out[(static_cast<size_t>(hd) * g.tpad + (tt & ~15u)) * g.dk + 16 * dd + (tt & 15)] = v;
                    }
                }
            } else {
                // through shared memory, a group of 32 output rows at a time, so
                // that a lane owns one output row (a column of the tile) and
                // each store is 32 consecutive floats (V panels: 16 of them)
#pragma unroll
                for (int h = 0; h < EPI_HALVES; h++) {
#pragma unroll
                    for (int j = 0; j < 32; j++) tw[lane * EPI_PITCH + j] = acc_at(acc, 32 * h + j);
                    __syncwarp();
                    const uint32_t col = col0 + 32 * h + lane;
                    const bool cvalid = col < g.rows;
                    const float wsv = cvalid ? __ldg(g.ws + col) : 0.0f;
                    const float bv = (g.bias && cvalid) ? __ldg(g.bias + col) : 0.0f;
                    const uint32_t tr0 = m0 + lane_base;
#pragma unroll
                    for (int i0 = 0; i0 < 32; i0 += 8) {
                        float old[8];
                        if (g.add) {
#pragma unroll
                            for (int i = 0; i < 8; i++) {
                                const uint32_t tt = tr0 + i0 + i;
                                old[i] = (cvalid && tt < g.T) ? g.out[out_at(g, tt, col)] : 0.0f;
                            }
                        }
#pragma unroll
                        for (int i = 0; i < 8; i++) {
                            const uint32_t tt = tr0 + i0 + i;
                            if (cvalid && tt < g.T) {
                                float v = mul_r<RM>(tw[(i0 + i) * EPI_PITCH + lane], wsv);
                                if (g.bias) v = add_r<RM>(v, bv);
                                if (g.add) v = add_r<RM>(old[i], v);
                                g.out[out_at(g, tt, col)] = v;
                            }
                        }
                    }
                    __syncwarp();
                }
            }
        }
        if (!ok) {
            *abort = 1;
            atomicOr(g.err, PKB_DEVERR_TIMEOUT);
        }
        // the warp's TMA stores complete before the CTA (and its shared
        // memory) goes
        if (TIO && lane == 0) bulk_wait_all();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == MMA_WARP) {
        tc_fence_after();
        tmem_dealloc(tbase, TMEM_COLS);
    }
}

using KernelFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, GemmArgs);

// The instance for these arguments: the staged MMA paths where qb is 32, 64
// or 128 and n a multiple of BK; om as the kernel's OM (0 where the results
// have no tensor map).
template <int RM, bool EXACT_SUM, int OM>
static KernelFn pick_om(uint32_t n, uint32_t qb) {
    if constexpr (EXACT_SUM) {
        const uint32_t spb = qb / KSTEP;
        if (n % BK == 0 && spb == 1) return gemm_q8_kernel<RM, true, OM, 1>;
        if (n % BK == 0 && spb == 2) return gemm_q8_kernel<RM, true, OM, 2>;
        if (n % BK == 0 && spb == 4) return gemm_q8_kernel<RM, true, OM, 4>;
    }
    if (n % BK == 0 && qb % BK == 0 && qb >= 2 * BK) return gemm_q8_kernel<RM, EXACT_SUM, OM, WIDE>;
    return gemm_q8_kernel<RM, EXACT_SUM, OM, 0>;
}

template <int RM, bool EXACT_SUM>
static KernelFn pick(uint32_t n, uint32_t qb, int om) {
    switch (om) {
    case 0: return pick_om<RM, EXACT_SUM, 0>(n, qb);
    case 1: return pick_om<RM, EXACT_SUM, 1>(n, qb);
    case 2: return pick_om<RM, EXACT_SUM, 2>(n, qb);
    default: return pick_om<RM, EXACT_SUM, 3>(n, qb);
    }
}

template <int RM, bool EXACT_SUM>
static cudaError_t launch_rm(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap* md,
                             const CUtensorMap* mo, const GemmArgs& g, int grid, cudaStream_t stream) {
    const bool tio = mo != nullptr;
    const int om = tio ? 1 + static_cast<int>(g.pmode) : 0;
    const KernelFn kern = pick<RM, EXACT_SUM>(g.n, g.qb, om);
    return launch_pdl(kern, dim3(grid), dim3(THREADS), SMEM_BYTES, stream, ma, mb, md ? *md : ma,
                      tio ? *mo : ma, g);
}

// Every instance's dynamic shared memory allowance, on the current device.
template <int RM, bool EXACT_SUM>
static cudaError_t prepare_rm() {
    for (int om = 0; om < 4; om++) {
        const KernelFn k[5] = {pick<RM, EXACT_SUM>(BK + 1, 32, om), pick<RM, EXACT_SUM>(BK, 32, om),
                               pick<RM, EXACT_SUM>(BK, 64, om), pick<RM, EXACT_SUM>(BK, 128, om),
                               pick<RM, EXACT_SUM>(BK, 2 * BK, om)};
        for (auto f : k) {
            cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
            if (e != cudaSuccess) return e;
        }
    }
    return cudaSuccess;
}

}  // namespace gemm

int gemm_tile_rows() { return gemm::BM; }
int gemm_tile_cols() { return gemm::BN; }
int gemm_box_k() { return gemm::BK; }

int gemm_out_box() { return 32; }
bool gemm_wide_blocks(uint32_t n, uint32_t qb) {
    return n % gemm::BK == 0 && qb % gemm::BK == 0 && qb >= 2 * gemm::BK;
}
int gemm_scale_box() { return gemm::DBLK; }

cudaError_t prepare_gemm_q8() {
    cudaError_t e;
    if ((e = gemm::prepare_rm<0, false>()) != cudaSuccess) return e;
    if ((e = gemm::prepare_rm<0, true>()) != cudaSuccess) return e;
    if ((e = gemm::prepare_rm<1, false>()) != cudaSuccess) return e;
    if ((e = gemm::prepare_rm<1, true>()) != cudaSuccess) return e;
    if ((e = gemm::prepare_rm<2, false>()) != cudaSuccess) return e;
    if ((e = gemm::prepare_rm<2, true>()) != cudaSuccess) return e;
    if ((e = gemm::prepare_rm<3, false>()) != cudaSuccess) return e;
    return gemm::prepare_rm<3, true>();
}

cudaError_t launch_gemm_q8(const CUtensorMap& map_a, const CUtensorMap& map_b, const CUtensorMap* map_d,
                           const CUtensorMap* map_o, const GemmArgs& g, int num_sms, int rmode, cudaStream_t stream) {
    const uint32_t ntiles = g.tiles_m * g.tiles_n;
    const int grid = static_cast<int>(ntiles < static_cast<uint32_t>(num_sms) ? ntiles : num_sms);
    // block sums convert to float exactly through the start-value trick while
    // |s| <= 128 * 127 * qb < 2^22, i.e. qb <= 256; wider blocks round
    // the conversion in the mode, as the reference's (float)s does
    const bool exact = g.qb <= 256;
    switch (rmode * 2 + (exact ? 1 : 0)) {
    case 0: return gemm::launch_rm<0, false>(map_a, map_b, map_d, map_o, g, grid, stream);
    case 1: return gemm::launch_rm<0, true>(map_a, map_b, map_d, map_o, g, grid, stream);
    case 2: return gemm::launch_rm<1, false>(map_a, map_b, map_d, map_o, g, grid, stream);
    case 3: return gemm::launch_rm<1, true>(map_a, map_b, map_d, map_o, g, grid, stream);
    case 4: return gemm::launch_rm<2, false>(map_a, map_b, map_d, map_o, g, grid, stream);
    case 5: return gemm::launch_rm<2, true>(map_a, map_b, map_d, map_o, g, grid, stream);
    case 6: return gemm::launch_rm<3, false>(map_a, map_b, map_d, map_o, g, grid, stream);
    default: return gemm::launch_rm<3, true>(map_a, map_b, map_d, map_o, g, grid, stream);
    }
}

}  // namespace pkb
