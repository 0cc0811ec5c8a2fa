// gemm_tc.cu -- batched Q4_0 x Q8-activation matmul (prefill) on the
// 5th-generation tensor cores: tcgen05 int8 MMA with the weights in tensor
// memory, activations fed by TMA, the per-block fp16 weight scales and fp32
// activation scales applied in the epilogue.
//
// Numerics are the reference's MEMVANTA_FORCE_Q8_ACT=1 prefill
// (tensor_matmul_batch_v06, src/gguf_kernels.cpp:265-266): every activation
// row is quantised per 32-element block (quantize_activations_q8, :174-178)
// and every (token t, row r) output is the decode dot dot_q4_q8 (:189), a
// sequential chain over the blocks b
//     sum = fma(d_w[r,b] * d_a[t,b], float(isum[r,t,b]), sum),  sum = 0 first,
// isum = sum_k (nib_k - 8) * q_k.  The integer block dots come from the
// tensor cores: each block is ONE tcgen05.mma (M = 128 rows, N tokens, K = 32
// = one block) into a TMEM slot of its own, so every slot holds the exact dot
// of one block, and epilogue warps run the chain over the slots in block
// order on the CUDA cores: every output equals the reference's bit for bit.
//
// Exact int -> float without integer instructions:
//   * A is the raw nibble (u8, 0..15), B the Q8 value (s8), so the MMA yields
//     D = isum + 8 * sum_k q_k.
//   * Every D slot is preset to the bit pattern 0x4B400000 (= 1.5 * 2^23 as
//     a float) and the MMA accumulates onto it; |D| < 2^16, so the slot's bits
//     read as a float are exactly 1.5 * 2^23 + D.
//   * The quantiser stores c[t,b] = 1.5 * 2^23 + 8 * sum_k q_k (exact), and
//     (1.5 * 2^23 + D) - c[t,b] = isum exactly (both in [2^23, 2^24)).
//   So the epilogue spends one subtract, one multiply and one FMA per (row,
//   token, block) -- packed two tokens per instruction (f32x2) -- and a
//   tcgen05.st puts the preset back after reading a slot.
//
// Data path, per pipeline stage of G = 4 blocks of a 128-row x N-token tile:
//   raw  smem [128 rows][64 B]  the Q4_0 nibble bytes of the 4 blocks: one 2-D
//                               TMA box over the [rows][nb*16 B] payload plane,
//                               64-byte swizzle (chunk j of row i at j^((i>>1)&3))
//   B    smem [N][128 B]        the Q8 activations of the 4 blocks, K-major,
//                               128-byte swizzle (one TMA box); block g is the
//                               32-byte K slice at +32 g of every row
//   A    TMEM 128 lanes x 32 cols  the nibbles one per byte (lane = row, 4 per
//                               32-bit column), written by the converter warps
//                               with tcgen05.st and read by the MMA from TMEM
//   D    TMEM 128 lanes x 4N cols  one N-column slot per block
// Epilogue data, per group of 16 blocks, in a ring of 4 slots the producer
// fills well ahead of use:
//   dw   [128 rows][32 B]       the fp16 weight scales, 2-D TMA box over the
//                               [rows][dstride] plane, 32-byte swizzle
//   sc   [2][16][N]             the activation scales and the constants c
//                               (block-major [nb][ldb] each, tokens padded to 64)
//
// Tiles: 128 rows x NE tokens, NE <= N (the epilogue reads the first NE
// columns of each N-wide slot; NE = 8 on N = 16 puts twice the CTAs on a
// narrow weight).  The launcher picks NE per weight and batch, and splits a
// weight with more row tiles than SMs into two launches (gemm_q4_q8_tc).
//
// Warp roles (one CTA per SM, persistent over its tiles):
//   warp 0       TMA producer (one lane): stages and epilogue data
//   warps 1-3    MMA issuers (one lane each, stages round-robin: an issuing
//                thread spends ~60 cycles per MMA and more on its waits and
//                commits, so three overlap); warp 1 also allocates TMEM
//   warps 4-7    converters: warp w writes TMEM lanes 32*(w%4).. (its rows)
//   warps 8-15   epilogue: TMEM -> registers -> chain -> y; warp w reads TMEM
//                lanes 32*(w%4).. (its row quadrant), token half (w-8)/4:
//                two warps per quadrant hide one another's TMEM and barrier
//                latencies (measured against one and four: two is 2-3%
//                faster than four on every prefill shape, one 10-25% slower)
// Rings: S smem stages (full: TMA bytes landed; empty: converters read the
// nibbles and the MMAs read B), 4 TMEM A stages (aready: converters wrote;
// aempty: MMAs read), the TMEM D groups (tfull: MMAs done; tempty: epilogue
// read them and restored the preset) and 4 epilogue-data slots (efull: TMA
// bytes landed; eempty: epilogue done).  Every wait is bounded (tc.cuh).
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.cuh"
#include "tc.cuh"

namespace mvb {

__device__ int g_tc_status = 0;

cudaError_t tc_status(cudaStream_t s, int* status) {
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return e;
    int v = 0;
    e = cudaMemcpyFromSymbol(&v, g_tc_status, sizeof(int));
    if (e == cudaSuccess && v != 0) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_tc_status, &zero, sizeof(int));
    }
    *status = v;
    if (e == cudaSuccess) e = f16_status_take(status);
    if (e == cudaSuccess) e = gemv_status_take(status);
    if (e == cudaSuccess) e = attn_status_take(status);
    return e;
}

uint64_t gemm_tc_ldb(uint64_t batch) { return (batch + 63) / 64 * 64; }

namespace {

constexpr int kM = 128;  // weight rows per tile = TMEM lanes
constexpr int kG = 4;    // Q4_0 blocks per pipeline stage
constexpr int kMmaWarps = 3;
constexpr int kConvWarp0 = 1 + kMmaWarps;
constexpr int kConvWarps = 4;
constexpr int kEpiWarp0 = kConvWarp0 + kConvWarps;
constexpr int kEW = 2;  // epilogue warps per TMEM lane quadrant
constexpr int kEpiWarps = 4 * kEW;
constexpr int kThreads = (kEpiWarp0 + kEpiWarps) * 32;
constexpr uint32_t kPreset = 0x4B400000u;   // 1.5 * 2^23 as a float
constexpr int kEB = 16;                     // blocks per epilogue-data slot
constexpr int kES = 4;                      // epilogue-data slots
constexpr int kSA = 4;                      // TMEM A stages
constexpr int kACols = kG * 8;              // TMEM columns of one A stage
constexpr int kDCols = 512 - kSA * kACols;  // TMEM columns of the D ring

// N = MMA width (tokens per MMA), NE = tokens of the tile the epilogue
// keeps (NE < N: the MMA's other columns are never read; tiles of NE = 8
// tokens put twice as many CTAs on a narrow weight as N = 16 can)
template <int N, int NE>
struct Cfg {
    static constexpr int kTT = NE / kEW;       // tokens per epilogue thread
    static constexpr int kRaw = kM * kG * 16;  // [128][64 B]
    static constexpr int kB = N * kG * 32;     // [N][128 B]
    static constexpr int kStage = kRaw + kB;
    static constexpr int kDw = kM * kEB * 2;            // weight scales [128][16] fp16
    static constexpr int kEpi = kDw + 2 * kEB * N * 4;  // + [2][16][N] fp32: scales, constants c
    static constexpr int kS = 12;
    static constexpr int kTG = kDCols / (kG * N);  // TMEM D groups
    static constexpr int kEpiOff = kS * kStage;
    static constexpr int kBarOff = kEpiOff + kES * kEpi;
    static constexpr int kBars = 2 * kS + 2 * kSA + 2 * kTG + 2 * kES + 1;
    static constexpr int kSmem = kBarOff + kBars * 8 + 16 + 1024;  // + alignment slack
    static_assert(kTG >= 2, "two TMEM D groups at least");
    static_assert(kStage % 1024 == 0 && kEpi % 1024 == 0, "swizzled TMA tiles need 1024-byte alignment");
    static_assert(kEB % kG == 0 && kTT % 4 == 0 && NE <= N, "tile shape");
    static_assert(kSmem <= 227 * 1024, "shared memory");
};

struct TcArgs {
    float* y;  // row r of token t at y[t * ldy + r]
    int rows, nb, batch, n_ttiles, n_tiles, accumulate, ldy;
};

template <int TT>
__device__ __forceinline__ void tmem_load(uint32_t taddr, uint32_t (&v)[TT]) {
    if constexpr (TT == 4) {
        tc::tmem_ld4(taddr, v);
    } else if constexpr (TT == 8) {
        tc::tmem_ld8(taddr, v);
    } else if constexpr (TT == 16) {
        tc::tmem_ld16(taddr, v);
    } else {
        tc::tmem_ld32(taddr, v);
    }
}
template <int TT>
__device__ __forceinline__ void tmem_preset(uint32_t taddr) {
    if constexpr (TT == 4) {
        tc::tmem_fill4(taddr, kPreset);
    } else if constexpr (TT == 8) {
        tc::tmem_fill8(taddr, kPreset);
    } else if constexpr (TT == 16) {
        tc::tmem_fill16(taddr, kPreset);
    } else {
        tc::tmem_fill32(taddr, kPreset);
    }
}

__device__ __forceinline__ uint64_t pack2(float a, float b) {
    return (uint64_t)__float_as_uint(a) | ((uint64_t)__float_as_uint(b) << 32);
}

template <int N, int NE>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                   const __grid_constant__ CUtensorMap dmap, const __grid_constant__ CUtensorMap smap,
                   const TcArgs a) {
    using C = Cfg<N, NE>;
    constexpr int TT = C::kTT, LB = 32 / TT < kG ? 32 / TT : kG;  // blocks per TMEM load batch
    extern __shared__ unsigned char smem_dyn[];
    const uint32_t s0 = tc::smem_u32(smem_dyn);
    const uint32_t pad = ((s0 + 1023u) & ~1023u) - s0;
    unsigned char* const sm = smem_dyn + pad;
    const uint32_t sbase = s0 + pad;
    const uint32_t bars = sbase + C::kBarOff;
    const uint32_t full0 = bars;
    const uint32_t empty0 = full0 + 8u * C::kS;
    const uint32_t aready0 = empty0 + 8u * C::kS;
    const uint32_t aempty0 = aready0 + 8u * kSA;
    const uint32_t tfull0 = aempty0 + 8u * kSA;
    const uint32_t tempty0 = tfull0 + 8u * C::kTG;
    const uint32_t efull0 = tempty0 + 8u * C::kTG;
    const uint32_t eempty0 = efull0 + 8u * kES;
    const uint32_t done_bar = eempty0 + 8u * kES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + C::kBarOff + C::kBars * 8);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + C::kBarOff + C::kBars * 8 + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool epi = warp >= kEpiWarp0;
    const int quad = warp & 3;                  // converter/epilogue: TMEM lanes 32*quad .. +31
    const int slice = (warp - kEpiWarp0) >> 2;  // epilogue: tokens slice*TT .. +TT-1 of a tile
    pdl_trigger();
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kS; ++s) {
            tc::mbar_init(full0 + 8 * s, 1);
            tc::mbar_init(empty0 + 8 * s, kConvWarps + 1);  // nibbles read + the MMAs' commit
        }
        for (int i = 0; i < kSA; ++i) {
            tc::mbar_init(aready0 + 8 * i, kConvWarps);
            tc::mbar_init(aempty0 + 8 * i, 1);
        }
        for (int g = 0; g < C::kTG; ++g) {
            tc::mbar_init(tfull0 + 8 * g, 1);
            tc::mbar_init(tempty0 + 8 * g, kEpiWarps);
        }
        for (int e = 0; e < kES; ++e) {
            tc::mbar_init(efull0 + 8 * e, 1);
            tc::mbar_init(eempty0 + 8 * e, kEpiWarps);
        }
        tc::mbar_init(done_bar, kMmaWarps);
        *abort_flag = 0;
        tc::mbar_fence_init();
        tc::tma_prefetch_map(&wmap);
        tc::tma_prefetch_map(&xmap);
        tc::tma_prefetch_map(&dmap);
        tc::tma_prefetch_map(&smap);
    }
    if (warp == 1) {
        tc::tmem_alloc(tc::smem_u32(tmem_slot), 512);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lanes = (uint32_t)(quad * 32) << 16;  // this warp's TMEM lane quadrant
    const uint32_t tl = tmem + lanes + slice * TT;         // epilogue's TMEM corner
    if (epi) {
        // preset every D slot this warp reads (its lanes x its token columns)
        for (int col = 0; col < C::kTG * kG * N; col += N) tmem_preset<TT>(tl + col);
        tc::tmem_wait_st();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    // programmatic dependent launch: the set-up above overlaps the previous
    // kernel; activations, scales and y are touched only after it completed
    pdl_wait();

    if (warp == 0) {
        // ---------------------------------------------------- TMA producer
        if (lane == 0) {
            uint32_t k = 0, j = 0;  // stages, epilogue-data groups issued
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < a.n_tiles; tile += gridDim.x) {
                const int row0 = (tile / a.n_ttiles) * kM, t0 = (tile % a.n_ttiles) * NE;
                for (int b0 = 0; b0 < a.nb; b0 += kG) {
                    if (b0 % kEB == 0) {
                        const int e = j % kES;
                        if (!tc::mbar_wait(eempty0 + 8 * e, ((j / kES) & 1u) ^ 1u, abort_flag, &g_tc_status, 10)) {
                            ok = false;
                            break;
                        }
                        const uint32_t ed = sbase + C::kEpiOff + e * C::kEpi;
                        tc::mbar_expect_tx(efull0 + 8 * e, C::kEpi);
                        tc::tma_load_2d(ed, &smap, b0, row0, efull0 + 8 * e);
                        tc::tma_load_3d(ed + C::kDw, &dmap, t0, b0, 0, efull0 + 8 * e);
                        ++j;
                    }
                    const int s = k % C::kS;
                    if (!tc::mbar_wait(empty0 + 8 * s, ((k / C::kS) & 1u) ^ 1u, abort_flag, &g_tc_status, 1)) {
                        ok = false;
                        break;
                    }
                    const uint32_t st = sbase + s * C::kStage;
                    tc::mbar_expect_tx(full0 + 8 * s, C::kStage);
                    tc::tma_load_2d(st, &wmap, b0 * 16, row0, full0 + 8 * s);
                    tc::tma_load_2d(st + C::kRaw, &xmap, b0 * 32, t0, full0 + 8 * s);
                    ++k;
                }
            }
            // drain: the latest load of every slot has landed before the CTA exits
            for (uint32_t i = k > (uint32_t)C::kS ? k - C::kS : 0; i < k; ++i)
                tc::mbar_wait(full0 + 8 * (i % C::kS), (i / C::kS) & 1u, abort_flag, &g_tc_status, 2, false);
            for (uint32_t i = j > (uint32_t)kES ? j - kES : 0; i < j; ++i)
                tc::mbar_wait(efull0 + 8 * (i % kES), (i / kES) & 1u, abort_flag, &g_tc_status, 11, false);
        }
    } else if (warp <= kMmaWarps) {
        // ---------------------------------------------------- MMA issuers
        const uint32_t mine = warp - 1;
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_u8s8(kM, N);
            const uint64_t bdesc0 = tc::sdesc_kmajor_sw128(sbase + C::kRaw);  // stage 0's B tile
            uint32_t k = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < a.n_tiles; tile += gridDim.x) {
                for (int b0 = 0; b0 < a.nb; b0 += kG, ++k) {
                    if (k % kMmaWarps != mine) continue;
                    const int s = k % C::kS, ai = k % kSA, tg = k % C::kTG;
                    if (!tc::mbar_wait(full0 + 8 * s, (k / C::kS) & 1u, abort_flag, &g_tc_status, 3) ||
                        !tc::mbar_wait(aready0 + 8 * ai, (k / kSA) & 1u, abort_flag, &g_tc_status, 4) ||
                        !tc::mbar_wait(tempty0 + 8 * tg, ((k / C::kTG) & 1u) ^ 1u, abort_flag, &g_tc_status, 5)) {
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
                    // block g: A at +8 g columns, B = the 32-byte K slice at +32 g (+2 in the address field)
                    const uint64_t bd = bdesc0 + (uint64_t)(s * (C::kStage >> 4));
                    const uint32_t ad = tmem + kDCols + ai * kACols;
                    const uint32_t d0 = tmem + tg * (kG * N);
                    const int nblk = a.nb - b0 < kG ? a.nb - b0 : kG;
                    for (int g = 0; g < nblk; ++g) tc::mma_i8_ts(d0 + g * N, ad + 8 * g, bd + 2 * g, idesc, 1u);
                    tc::mma_commit(empty0 + 8 * s);
                    tc::mma_commit(aempty0 + 8 * ai);
                    tc::mma_commit(tfull0 + 8 * tg);
                }
            }
            // every MMA issued has completed before TMEM is released
            tc::mma_commit(done_bar);
            tc::mbar_wait(done_bar, 0, abort_flag, &g_tc_status, 6, false);
        }
    } else if (!epi) {
        // ------------------------------------------------------ converters
        const int c = quad * 32 + lane;  // row of the tile = this thread's TMEM lane
        const int rsw = (c >> 1) & 3;    // 64-byte swizzle phase of raw row c
        uint32_t k = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < a.n_tiles; tile += gridDim.x) {
            for (int b0 = 0; b0 < a.nb; b0 += kG, ++k) {
                const int s = k % C::kS, ai = k % kSA;
                const bool got =
                    tc::mbar_wait(full0 + 8 * s, (k / C::kS) & 1u, abort_flag, &g_tc_status, 7) &&
                    tc::mbar_wait(aempty0 + 8 * ai, ((k / kSA) & 1u) ^ 1u, abort_flag, &g_tc_status, 12);
                // warp-uniform outcome: the TMEM store below is .sync.aligned
                if (!__all_sync(0xffffffffu, got)) {
                    ok = false;
                    break;
                }
                tc::tc_fence_after();
                const unsigned char* raw = sm + s * C::kStage + c * 64;
                uint32_t v[32];
#pragma unroll
                for (int g = 0; g < kG; ++g) {
                    // GGUF order: byte i holds element i (low nibble) and 16 + i (high)
                    const uint4 w = *reinterpret_cast<const uint4*>(raw + ((g ^ rsw) << 4));
                    v[8 * g + 0] = w.x & 0x0F0F0F0Fu;
                    v[8 * g + 1] = w.y & 0x0F0F0F0Fu;
                    v[8 * g + 2] = w.z & 0x0F0F0F0Fu;
                    v[8 * g + 3] = w.w & 0x0F0F0F0Fu;
                    v[8 * g + 4] = (w.x >> 4) & 0x0F0F0F0Fu;
                    v[8 * g + 5] = (w.y >> 4) & 0x0F0F0F0Fu;
                    v[8 * g + 6] = (w.z >> 4) & 0x0F0F0F0Fu;
                    v[8 * g + 7] = (w.w >> 4) & 0x0F0F0F0Fu;
                }
                tc::tmem_st32(tmem + lanes + kDCols + ai * kACols, v);
                tc::tmem_wait_st();
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    tc::mbar_arrive(aready0 + 8 * ai);
                    tc::mbar_arrive(empty0 + 8 * s);
                }
            }
        }
    } else {
        // -------------------------------------------------------- epilogue
        const int rr = quad * 32 + lane;
        const int dsw = (rr >> 2) & 1;  // 32-byte swizzle phase of this row's weight scales
        uint32_t k = 0, j = 0;          // stages, epilogue-data groups consumed
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < a.n_tiles; tile += gridDim.x) {
            const int r = (tile / a.n_ttiles) * kM + rr;
            const int tb = (tile % a.n_ttiles) * NE + slice * TT;
            uint64_t acc[TT / 2];  // token pairs, (+0, +0) first
#pragma unroll
            for (int t = 0; t < TT / 2; ++t) acc[t] = 0ull;
            for (int b16 = 0; b16 < a.nb; b16 += kEB) {
                const int e = j % kES;
                if (!__all_sync(0xffffffffu,
                                tc::mbar_wait(efull0 + 8 * e, (j / kES) & 1u, abort_flag, &g_tc_status, 13))) {
                    ok = false;
                    break;
                }
                const unsigned char* ed = sm + C::kEpiOff + e * C::kEpi;
                const uint4 w0 = *reinterpret_cast<const uint4*>(ed + rr * 32 + ((0 ^ dsw) << 4));
                const uint4 w1 = *reinterpret_cast<const uint4*>(ed + rr * 32 + ((1 ^ dsw) << 4));
                const uint32_t dwp[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                const float* da = reinterpret_cast<const float*>(ed + C::kDw);  // [16][N]
                const float* cb = da + kEB * N;                                 // [16][N]
#pragma unroll
                for (int h = 0; h < kEB / kG; ++h) {  // the stages of this group
                    const int b0 = b16 + h * kG;
                    if (b0 >= a.nb) break;
                    const int nblk = a.nb - b0;
                    const int tg = k % C::kTG;
                    // warp-uniform outcome: the TMEM accesses below are .sync.aligned
                    if (!__all_sync(0xffffffffu, tc::mbar_wait(tfull0 + 8 * tg, (k / C::kTG) & 1u, abort_flag,
                                                               &g_tc_status, 8))) {
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
                    // LB slots in flight at once (32 registers), one wait, then the presets back
#pragma unroll
                    for (int gb = 0; gb < kG; gb += LB) {
                    uint32_t v[LB][TT];
#pragma unroll
                    for (int i = 0; i < LB; ++i) tmem_load<TT>(tl + tg * (kG * N) + (gb + i) * N, v[i]);
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < LB; ++i) tmem_preset<TT>(tl + tg * (kG * N) + (gb + i) * N);
#pragma unroll
                    for (int i = 0; i < LB; ++i) {
                        const int g = gb + i;
                        if (g < nblk) {
                            const int eb = h * kG + g;  // block index in the group of 16
                            const uint32_t word = dwp[eb >> 1];
                            const float dw = half_bits_to_float((unsigned short)((eb & 1) ? word >> 16 : word));
                            const uint64_t dw2 = pack2(dw, dw);
                            const ulonglong2* d4p = reinterpret_cast<const ulonglong2*>(da + eb * N + slice * TT);
                            const ulonglong2* c4p = reinterpret_cast<const ulonglong2*>(cb + eb * N + slice * TT);
#pragma unroll
                            for (int t4 = 0; t4 < TT / 4; ++t4) {
                                const ulonglong2 d4 = d4p[t4], c4 = c4p[t4];
                                const uint64_t v0 = (uint64_t)v[i][4 * t4] | ((uint64_t)v[i][4 * t4 + 1] << 32);
                                const uint64_t v1 = (uint64_t)v[i][4 * t4 + 2] | ((uint64_t)v[i][4 * t4 + 3] << 32);
                                acc[2 * t4] = tc::f2_fma(tc::f2_mul(dw2, d4.x), tc::f2_sub(v0, c4.x), acc[2 * t4]);
                                acc[2 * t4 + 1] =
                                    tc::f2_fma(tc::f2_mul(dw2, d4.y), tc::f2_sub(v1, c4.y), acc[2 * t4 + 1]);
                            }
                        }
                    }
                    }
                    tc::tmem_wait_st();
                    tc::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(tempty0 + 8 * tg);
                    ++k;
                }
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(eempty0 + 8 * e);
                ++j;
            }
            if (!ok) break;
            if (r < a.rows) {
#pragma unroll
                for (int t = 0; t < TT; ++t) {
                    if (tb + t < a.batch) {
                        const float v = __uint_as_float((uint32_t)(acc[t / 2] >> (32 * (t & 1))));
                        float* p = a.y + (size_t)(tb + t) * a.ldy + r;
                        *p = a.accumulate ? *p + v : v;
                    }
                }
            }
        }
    }

    // teardown: every role is out of its loop, copies and MMAs have drained
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 512);
    }
}

using tc::EncodeFn;
using tc::encode;
using tc::encode_fn;

template <int N, int NE>
cudaError_t launch_tc(const mv_weight_s& w, const int8_t* q, const float* dT, uint64_t ldb, uint64_t batch, float* y,
                      uint64_t ldy, cudaStream_t s, bool accumulate) {
    using C = Cfg<N, NE>;
    const EncodeFn enc = encode_fn();
    if (!enc) {
        set_last_error("cuTensorMapEncodeTiled is unavailable in this driver");
        return cudaErrorNotSupported;
    }
    CUtensorMap wmap, xmap, dmap, smap;
    // payload plane [rows][nb*16 B] -> raw [128][64 B], 64-byte swizzle
    const cuuint64_t wdims[2] = {w.nb * 16, w.rows}, wstr[1] = {w.nb * 16};
    const cuuint32_t wbox[2] = {(cuuint32_t)(kG * 16), (cuuint32_t)kM};
    // activations [batch][K] -> B [N][128 B], 128-byte swizzle
    const cuuint64_t xdims[2] = {w.nb * 32, batch}, xstr[1] = {w.nb * 32};
    const cuuint32_t xbox[2] = {(cuuint32_t)(kG * 32), (cuuint32_t)N};
    // scales and constants [2][nb][ldb] fp32 -> [2][16][N]
    const cuuint64_t ddims[3] = {ldb, w.nb, 2}, dstr[2] = {ldb * 4, w.nb * ldb * 4};
    const cuuint32_t dbox[3] = {(cuuint32_t)N, (cuuint32_t)kEB, 2};
    // weight scales [rows][dstride] fp16 -> [128][16], 32-byte swizzle
    const cuuint64_t sdims[2] = {w.dstride, w.rows}, sstr[1] = {w.dstride * 2};
    const cuuint32_t sbox[2] = {(cuuint32_t)kEB, (cuuint32_t)kM};
    if (!encode(enc, &wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w.qs, wdims, wstr, wbox, CU_TENSOR_MAP_SWIZZLE_64B) ||
        !encode(enc, &xmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(q), xdims, xstr, xbox,
                CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode(enc, &dmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(dT), ddims, dstr, dbox,
                CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode(enc, &smap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, w.d, sdims, sstr, sbox, CU_TENSOR_MAP_SWIZZLE_32B)) {
        set_last_error("cuTensorMapEncodeTiled rejected a tensor map of the tensor-core GEMM");
        return cudaErrorInvalidValue;
    }
    const int n_ttiles = (int)((batch + NE - 1) / NE);
    const int n_tiles = (int)((w.rows + kM - 1) / kM) * n_ttiles;
    const TcArgs args{y, (int)w.rows, (int)w.nb, (int)batch, n_ttiles, n_tiles, accumulate ? 1 : 0, (int)ldy};
    ensure_smem_attr(gemm_tc_kernel<N, NE>, C::kSmem);
    const int grid = n_tiles < num_sms() ? n_tiles : num_sms();
    return launch_pdl(gemm_tc_kernel<N, NE>, dim3(grid), dim3(kThreads), C::kSmem, s, wmap, xmap, dmap, smap, args);
}

}  // namespace

cudaError_t gemm_q4_q8_tc(const mv_weight_s& w, const int8_t* q, const float* dT, uint64_t ldb, uint64_t batch,
                          float* y, cudaStream_t s, bool accumulate) {
    if (!batch) return cudaSuccess;
    if (w.type != 2 || ldb < gemm_tc_ldb(batch) || ldb % 4 || w.rows >= (1ull << 31) || batch >= (1ull << 31))
        return cudaErrorInvalidValue;
    // Tile width (tokens per tile): the epilogue's share grows with it, the
    // per-block MMA, conversion and synchronisation share does not; pick the
    // width with the fewest waves x relative cost of one tile (8 tokens
    // ~0.42, 16 ~0.6 of a 32-token tile).
    const uint64_t sms = (uint64_t)num_sms();
    auto plan = [&](uint64_t row_tiles, int& ne) {
        auto waves = [&](uint64_t e) { return (double)((row_tiles * ((batch + e - 1) / e) + sms - 1) / sms); };
        ne = 32;
        double best = waves(32) * 100.0;
        if (waves(16) * 60.0 <= best) ne = 16, best = waves(16) * 60.0;
        if (waves(8) * 42.0 < best) ne = 8, best = waves(8) * 42.0;
        return best;
    };
    auto run = [&](const mv_weight_s& v, float* yv, int ne) {
        return ne == 8    ? launch_tc<16, 8>(v, q, dT, ldb, batch, yv, w.rows, s, accumulate)
               : ne == 16 ? launch_tc<16, 16>(v, q, dT, ldb, batch, yv, w.rows, s, accumulate)
                          : launch_tc<32, 32>(v, q, dT, ldb, batch, yv, w.rows, s, accumulate);
    };
    const uint64_t row_tiles = (w.rows + kM - 1) / kM;
    int ne = 32, ne_rest = 32;
    const double one = plan(row_tiles, ne);
    // One token tile and more 128-row tiles than SMs: a launch of one
    // 32-token tile per SM, then the remaining rows in narrower tiles (each
    // CTA of the second launch starts as an SM frees up), instead of uneven
    // rounds of one launch (gate|up at 32 tokens: 172 row tiles).
    if (batch <= 32 && row_tiles > sms && 100.0 + plan(row_tiles - sms, ne_rest) < one) {
        mv_weight_s head = w, tail = w;
        const uint64_t r0 = sms * kM;
        head.rows = r0;
        tail.rows = w.rows - r0;
        tail.qs = w.qs + r0 * w.nb * 16;  // 16-byte aligned: whole rows of 16-byte payloads
        tail.d = w.d + r0 * w.dstride;    // dstride is a multiple of 8 fp16
        const cudaError_t e = run(head, y, 32);
        return e != cudaSuccess ? e : run(tail, y + r0, ne_rest);
    }
    return run(w, y, ne);
}

}  // namespace mvb
