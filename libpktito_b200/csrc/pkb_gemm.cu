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
// Warp roles in a 576-thread CTA, one CTA per SM (its 194 KB of shared
// memory keeps a second off), persistent over the tiles:
//   warp 16    TMA producer: 128-byte-swizzled 128x128 tiles of activations
//              and weights into a 6-stage shared-memory ring
//   warp 17    allocates TMEM; one thread issues the MMAs and commits
//   warps 0-15 the epilogue: warp w reads TMEM lanes 32*(w%4).. (the
//              quarter its hardware warp slot may access) and columns
//              32*(w/4)..+31 of each block's accumulator; each thread is one
//              frame and runs the float chain of 32 output rows in registers,
//              then scales, biases, adds and stores them.
//
// The fp32 chain (one FMA per output and block, plus the int->float of the
// sum) is the bound at 32-input blocks, not the tensor core: the MMAs of a
// block take a quarter of the time the epilogue's CUDA cores need for it.
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
constexpr int EPI_WARPS = 16;
constexpr int TMA_WARP = 16;
constexpr int MMA_WARP = 17;
constexpr int THREADS = 18 * 32;
constexpr int A_BYTES = BM * BK;
constexpr int B_BYTES = BN * BK;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_PITCH = 33;      // floats a row of an epilogue warp's transpose tile
constexpr int EPI_BYTES = EPI_WARPS * 32 * EPI_PITCH * 4;
constexpr int BAR_BYTES = 256;
constexpr int SMEM_BYTES = NSTAGE * STAGE_BYTES + EPI_BYTES + BAR_BYTES + 1024;  // + alignment slack

static_assert(TMEM_COLS == 512, "TMEM ring must fit the SM's 512 columns");
static_assert((2 * NSTAGE + 2 * NTMEM + 1) * 8 + 8 <= BAR_BYTES, "barrier area");

// acc[8*half + i] (two output rows each) = fma(float(s), d, acc), for the
// 16 block sums of one TMEM load, two rows an instruction.
template <int RM, bool EXACT_SUM>
__device__ __forceinline__ void chain16(uint64_t (&acc)[16], const uint32_t (&s)[16], int half, float dv) {
    const uint64_t d2 = pack2(dv, dv);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        uint64_t f;
        if constexpr (EXACT_SUM) {
            // the sums plus 0x4B400000 are the floats 1.5 * 2^23 + s; less
            // 1.5 * 2^23, rounded to nearest, they are exactly s
            f = add2_rn(pack2(__uint_as_float(s[2 * i] + 0x4B400000u), __uint_as_float(s[2 * i + 1] + 0x4B400000u)),
                        pack2(-12582912.0f, -12582912.0f));
        } else {
            f = pack2(i2f_r<RM>(static_cast<int>(s[2 * i])), i2f_r<RM>(static_cast<int>(s[2 * i + 1])));
        }
        acc[8 * half + i] = fma2_r<RM>(f, d2, acc[8 * half + i]);
    }
}

template <int RM, bool EXACT_SUM>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_q8_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const GemmArgs g) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* epi = reinterpret_cast<float*>(smem + NSTAGE * STAGE_BYTES);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + NSTAGE * STAGE_BYTES + EPI_BYTES);
    uint64_t* empty = full + NSTAGE;
    uint64_t* tfull = empty + NSTAGE;
    uint64_t* tempty = tfull + NTMEM;
    uint64_t* drain = tempty + NTMEM;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NSTAGE; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < NTMEM; i++) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], EPI_WARPS);
        }
        mbar_init(drain, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == MMA_WARP) {
        tmem_alloc(tslot, TMEM_COLS);
        tmem_relinquish();
    }
    if (warp == TMA_WARP && lane == 0) {
        tma_prefetch_map(&map_a);
        tma_prefetch_map(&map_b);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;

    const uint32_t nk = g.n / KSTEP;            // K steps of a tile
    const uint32_t nc = (g.n + BK - 1) / BK;     // shared-memory stages of a tile
    const uint32_t spb = g.qb / KSTEP;          // K steps a block
    const uint32_t nb = g.n / g.qb;             // blocks
    const uint32_t ntiles = g.tiles_m * g.tiles_n;
    const long long limit = g.timeout;

    if (warp == TMA_WARP) {
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (uint32_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
                const int m0 = static_cast<int>((tile / g.tiles_n) * BM);
                const int n0 = static_cast<int>((tile % g.tiles_n) * BN);
                for (uint32_t c = 0; c < nc; c++, it++) {
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
            }
        }
    } else if (warp == MMA_WARP) {
        if (lane == 0) {
            constexpr uint32_t idesc = i8_instr_desc(BM, BN);
            uint32_t it = 0, tb = 0;
            bool ok = true;
            for (uint32_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
                for (uint32_t c = 0; c < nc && ok; c++, it++) {
                    const uint32_t s = it % NSTAGE, ph = (it / NSTAGE) & 1;
                    if (!mbar_wait(&full[s], ph, abort, limit)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + s * STAGE_BYTES);
                    const uint32_t b_addr = a_addr + A_BYTES;
                    const uint32_t jn = nk - 4 * c < 4 ? nk - 4 * c : 4;
                    for (uint32_t j = 0; j < jn; j++) {
                        const uint32_t pos = (4 * c + j) % spb;
                        const uint32_t ts = tb % NTMEM;
                        if (pos == 0) {
                            if (!mbar_wait(&tempty[ts], ((tb / NTMEM) & 1) ^ 1, abort, limit)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                        }
                        umma_i8(tbase + ts * BN, sw128_kmajor_desc(a_addr + j * KSTEP),
                                sw128_kmajor_desc(b_addr + j * KSTEP), idesc, pos != 0);
                        if (pos == spb - 1) {
                            umma_commit(&tfull[ts]);
                            tb++;
                        }
                    }
                    umma_commit(&empty[s]);
                }
            }
            if (!ok) {
                *abort = 1;
                atomicOr(g.err, PKB_DEVERR_TIMEOUT);
                // the MMAs this thread issued: let them finish before TMEM is freed
                umma_commit(drain);
                mbar_drain(drain, 0, limit);
            }
        }
    } else {
        // epilogue: frame t of the tile is this thread's TMEM lane
        const uint32_t quarter = warp & 3, cgroup = warp >> 2;
        const uint32_t lane_base = 32 * quarter;
        float* tw = epi + warp * (32 * EPI_PITCH);  // this warp's 32 x 32 transpose tile
        uint32_t tb = 0;
        bool ok = true;
        for (uint32_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
            const uint32_t m0 = (tile / g.tiles_n) * BM;
            const uint32_t n0 = (tile % g.tiles_n) * BN;
            const uint32_t t = m0 + lane_base + lane;
            const bool tvalid = t < g.T;
            const float* drow = g.d + static_cast<size_t>(tvalid ? t : 0) * nb;

            uint64_t acc[16];
#pragma unroll
            for (int j = 0; j < 16; j++) acc[j] = 0;  // +0, +0

            // the frame's block scales, four blocks at a time, fetched one
            // chunk of four ahead of their use
            float dc[4];
#pragma unroll
            for (int j = 0; j < 4; j++) dc[j] = (tvalid && static_cast<uint32_t>(j) < nb) ? __ldg(drow + j) : 0.0f;
            for (uint32_t b0 = 0; ok && b0 < nb; b0 += 4) {
                float dn[4];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const uint32_t bb = b0 + 4 + j;
                    dn[j] = (tvalid && bb < nb) ? __ldg(drow + bb) : 0.0f;
                }
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    if (b0 + j >= nb) break;
                    const uint32_t ts = tb % NTMEM;
                    // every lane waits, and the warp goes on only if all saw
                    // the phase: the TMEM loads are whole-warp instructions
                    const bool seen = mbar_wait(&tfull[ts], (tb / NTMEM) & 1, abort, limit);
                    if (!__all_sync(0xffffffffu, seen)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t ta = tbase + (lane_base << 16) + ts * BN + 32 * cgroup;
                    uint32_t s0[16], s1[16];
                    tmem_ld_32x32b_x16(ta, s0);
                    tmem_ld_wait(s0);
                    tmem_ld_32x32b_x16(ta + 16, s1);  // in flight under the first half's chain
                    chain16<RM, EXACT_SUM>(acc, s0, 0, dc[j]);
                    tmem_ld_wait(s1);
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[ts]);
                    chain16<RM, EXACT_SUM>(acc, s1, 1, dc[j]);
                    tb++;
                }
#pragma unroll
                for (int j = 0; j < 4; j++) dc[j] = dn[j];
            }
            if (!ok) break;

            // through shared memory, so that a lane owns one output row (a
            // column of the tile) and each store is 32 consecutive floats
#pragma unroll
            for (int j = 0; j < 16; j++) {
                float lo, hi;
                unpack2(acc[j], lo, hi);
                tw[lane * EPI_PITCH + 2 * j] = lo;
                tw[lane * EPI_PITCH + 2 * j + 1] = hi;
            }
            __syncwarp();
            const uint32_t col = n0 + 32 * cgroup + lane;
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
                        old[i] = (cvalid && tt < g.T) ? g.out[static_cast<size_t>(tt) * g.os + col] : 0.0f;
                    }
                }
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const uint32_t tt = tr0 + i0 + i;
                    if (cvalid && tt < g.T) {
                        float v = mul_r<RM>(tw[(i0 + i) * EPI_PITCH + lane], wsv);
                        if (g.bias) v = add_r<RM>(v, bv);
                        if (g.add) v = add_r<RM>(old[i], v);
                        g.out[static_cast<size_t>(tt) * g.os + col] = v;
                    }
                }
            }
            __syncwarp();
        }
        if (!ok) {
            *abort = 1;
            atomicOr(g.err, PKB_DEVERR_TIMEOUT);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == MMA_WARP) {
        tc_fence_after();
        tmem_dealloc(tbase, TMEM_COLS);
    }
}

template <int RM, bool EXACT_SUM>
static cudaError_t launch_rm(const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& g, int grid,
                             cudaStream_t stream) {
    auto kern = gemm_q8_kernel<RM, EXACT_SUM>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    kern<<<grid, THREADS, SMEM_BYTES, stream>>>(ma, mb, g);
    return cudaGetLastError();
}

}  // namespace gemm

int gemm_tile_rows() { return gemm::BM; }
int gemm_tile_cols() { return gemm::BN; }
int gemm_box_k() { return gemm::BK; }

cudaError_t launch_gemm_q8(const CUtensorMap& map_a, const CUtensorMap& map_b, const GemmArgs& g, int num_sms,
                           int rmode, cudaStream_t stream) {
    const uint32_t ntiles = g.tiles_m * g.tiles_n;
    const int grid = static_cast<int>(ntiles < static_cast<uint32_t>(num_sms) ? ntiles : num_sms);
    // block sums convert to float exactly through the bias trick while
    // |s| <= 128 * 127 * qb < 2^22, i.e. qb <= 256; wider blocks round
    // the conversion in the mode, as the reference's (float)s does
    const bool exact = g.qb <= 256;
    switch (rmode * 2 + (exact ? 1 : 0)) {
    case 0: return gemm::launch_rm<0, false>(map_a, map_b, g, grid, stream);
    case 1: return gemm::launch_rm<0, true>(map_a, map_b, g, grid, stream);
    case 2: return gemm::launch_rm<1, false>(map_a, map_b, g, grid, stream);
    case 3: return gemm::launch_rm<1, true>(map_a, map_b, g, grid, stream);
    case 4: return gemm::launch_rm<2, false>(map_a, map_b, g, grid, stream);
    case 5: return gemm::launch_rm<2, true>(map_a, map_b, g, grid, stream);
    case 6: return gemm::launch_rm<3, false>(map_a, map_b, g, grid, stream);
    default: return gemm::launch_rm<3, true>(map_a, map_b, g, grid, stream);
    }
}

}  // namespace pkb
