// gemm_f16.cu -- batched Q4_0 x Q8-activation matmul (prefill) on the
// 5th-generation tensor cores with fp16 operands, for batches of 64 tokens
// and more.
//
// Numerics are the reference's MEMVANTA_FORCE_Q8_ACT=1 prefill
// (tensor_matmul_batch_v06, src/gguf_kernels.cpp:265-266): per (token t,
// row r) the sequential chain over the 32-element blocks b
//     sum = fma(fp16(d_w[r,b]) * d_a[t,b], float(isum[r,t,b]), sum)
// with isum = sum_k (nib_k - 8) * q_k (dot_q4_q8, :189).  The block dots come
// from tcgen05.mma kind::f16 with fp32 accumulation: A = nib - 8 and B = q
// are small integers, exact in fp16, every product and partial sum is an
// integer below 2^16, so the accumulator holds float(isum) exactly whatever
// the order of the tensor core's additions.  Each block gets a TMEM slot of
// its own (two K = 16 MMAs), so the epilogue reads every block's dot apart and
// runs the chain in block order: one packed multiply and one packed FMA per
// two (row, token) pairs and block -- no int->float step, no constant to
// subtract, no slot to reset between uses.
//
// Per pipeline stage of kG = 2 blocks of a 128-row x NT-token tile:
//   raw  smem [128][32 B]       the Q4_0 nibble bytes (TMA, no swizzle)
//   B    smem [NT][128 B]       the fp16 activations (TMA, 128-byte swizzle)
//   A    smem [128][128 B]      the weights as fp16 (nib - 8), K-major,
//                               128-byte swizzle -- written by 4 converter
//                               warps (thread = row) from raw into a ring of
//                               its own, so the TMA ring (raw + B, 8 stages)
//                               is not held while A waits for the MMAs
//   D    TMEM 128 lanes x NT    one slot per block, 512 / NT slots in a ring
// Epilogue data per 16 blocks: the rows' fp16 weight scales (TMA, 32-byte
// swizzle) and the tokens' fp32 activation scales (TMA, block-major).
//
// Warps: 0 TMA producer, 1-2 MMA issuers (1 also owns TMEM), 3-6 converters,
// then NT/32 epilogue warps per TMEM lane quadrant (32 tokens each).  Every
// wait is bounded (tc.cuh): a wait that runs out raises the CTA's abort flag,
// records a site in the status word, and every role drains and returns.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.cuh"
#include "tc.cuh"

namespace mvb {

__device__ int g_f16_status = 0;  // site of an expired bounded wait (0: none)

// Adds this kernel's status to *status (first site wins) and clears it;
// tc_status (gemm_tc.cu) reports both tensor-core GEMMs through it.
cudaError_t f16_status_take(int* status) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_f16_status, sizeof(int));
    if (e == cudaSuccess && v != 0) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_f16_status, &zero, sizeof(int));
        if (!*status) *status = v;
    }
    return e;
}

namespace {

constexpr int kM = 128;        // weight rows per tile = TMEM lanes
constexpr int kG = 2;          // blocks per stage: K = 64 fp16 = one 128-byte swizzle row
constexpr int kEB = 16;        // blocks per epilogue-data slot
constexpr int kES = 2;         // epilogue-data slots
constexpr int kMmaWarps = 2;   // warps 1, 2: MMA issuers, stages alternating
constexpr int kConv0 = 1 + kMmaWarps;  // first converter warp
constexpr int kConvWarps = 4;
constexpr int kEpi0 = kConv0 + kConvWarps;

template <int NT>
struct Cfg {
    static constexpr int kEpiWarps = 4 * (NT / 32);
    static constexpr int kThreads = (kEpi0 + kEpiWarps) * 32;
    static constexpr int kA = kM * kG * 64;   // 16 KB: one A slot
    static constexpr int kSA = 3;             // A slots (converters -> MMAs)
    static constexpr int kB = NT * kG * 64;   // NT x 128 B
    static constexpr int kRaw = kM * kG * 16; // 4 KB
    static constexpr int kStage = kB + kRaw;  // one TMA stage
    static constexpr int kS = NT > 64 ? 6 : 8;  // TMA stages: deep enough to cover the load latency
    static constexpr int kR = 16;             // stage-completion barriers (one MMA commit per stage)
    static constexpr int kDw = kM * kEB * 2;  // [128][16] fp16
    static constexpr int kDa = kEB * NT * 4;  // [16][NT] fp32
    static constexpr int kEpi = kDw + kDa;
    static constexpr int kSlots = 512 / NT;   // TMEM D slots, one block each
    static constexpr int kPairs = kSlots / 2; // a stage's two blocks use a pair of slots
    static constexpr int kStageOff = kSA * kA;
    static constexpr int kEpiOff = kStageOff + kS * kStage;
    static constexpr int kBarOff = kEpiOff + kES * kEpi;
    static constexpr int kBars = kS + kSA + kR + kPairs + 2 * kES + 1;
    static constexpr int kSmem = kBarOff + kBars * 8 + 16 + 1024;
    static_assert(kA % 1024 == 0 && kB % 1024 == 0 && kStage % 1024 == 0 && kEpi % 1024 == 0, "alignment");
    static_assert(kSmem <= 227 * 1024, "shared memory");
    static_assert(kG == 2 && kPairs >= 2, "two stages of D slot pairs");
    static_assert(kR > kS && kR > kSA && kR > kPairs, "a stage's completion is awaited before its barrier recurs");
};

struct F16Args {
    float* y;  // row r of token t at y[t * ldy + r]
    int rows, nb, batch, n_ttiles, n_tiles, accumulate, ldy;
    uint64_t wait_ns;  // bound of every mbarrier wait
    int skip_commit;   // test hook: the stage whose MMA commit is left out (-1: none)
};

// Instruction descriptor of kind::f16: f16 x f16 -> f32, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4)                      // D format: f32
           | (0u << 7) | (0u << 10)       // A, B: f16
           | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (=|+=) A[smem] * B[smem]^T, kind::f16, issued by one thread.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

__device__ __forceinline__ uint64_t pack2(float a, float b) {
    return (uint64_t)__float_as_uint(a) | ((uint64_t)__float_as_uint(b) << 32);
}

// Two nibbles of each of the bytes 2p, 2p+1 of w (p = 0, 1) as fp16 (nib - 8)
// pairs: (0x6400 | nib) is 1024 + nib in fp16, minus 1032 exactly.
__device__ __forceinline__ uint32_t nib_pair(uint32_t w, uint32_t sel, int shift) {
    const uint32_t t = __byte_perm(w, 0u, sel);  // bytes 2p, 2p+1 in the low bytes of each half
    const uint32_t h = ((t >> shift) & 0x000F000Fu) | 0x64006400u;
    const __half2 v = __hsub2(*reinterpret_cast<const __half2*>(&h), __halves2half2(__ushort_as_half(0x6408),
                                                                                     __ushort_as_half(0x6408)));
    return *reinterpret_cast<const uint32_t*>(&v);
}

template <int NT>
__global__ void __launch_bounds__(Cfg<NT>::kThreads, 1)
    gemm_f16_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                    const __grid_constant__ CUtensorMap dmap, const __grid_constant__ CUtensorMap smap,
                    const F16Args a) {
    using C = Cfg<NT>;
    constexpr int TT = 32;              // tokens per epilogue warp
    constexpr int LB = NT > 64 ? 1 : 2; // TMEM slots per load round trip
    extern __shared__ unsigned char smem_dyn[];
    const uint32_t s0 = tc::smem_u32(smem_dyn);
    const uint32_t pad = ((s0 + 1023u) & ~1023u) - s0;
    unsigned char* const sm = smem_dyn + pad;
    const uint32_t sbase = s0 + pad;
    const uint32_t bars = sbase + C::kBarOff;
    const uint32_t full0 = bars;                      // TMA bytes of a stage landed
    const uint32_t aready0 = full0 + 8u * C::kS;      // converters wrote an A slot
    // stage k's MMAs completed (one commit): its TMA slot, its A slot and its
    // D slot pair -- whose dots the epilogue then reads -- are all released
    const uint32_t done0 = aready0 + 8u * C::kSA;
    const uint32_t tempty0 = done0 + 8u * C::kR;      // a D slot pair read by every epilogue warp
    const uint32_t efull0 = tempty0 + 8u * C::kPairs;
    const uint32_t eempty0 = efull0 + 8u * kES;
    const uint32_t done_bar = eempty0 + 8u * kES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + C::kBarOff + C::kBars * 8);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + C::kBarOff + C::kBars * 8 + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int quad = warp & 3;
    pdl_trigger();
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kS; ++s) {
            tc::mbar_init(full0 + 8 * s, 1);
        }
        for (int i = 0; i < C::kSA; ++i) tc::mbar_init(aready0 + 8 * i, kConvWarps);
        for (int i = 0; i < C::kR; ++i) tc::mbar_init(done0 + 8 * i, 1);
        for (int j = 0; j < C::kPairs; ++j) tc::mbar_init(tempty0 + 8 * j, C::kEpiWarps);
        for (int e = 0; e < kES; ++e) {
            tc::mbar_init(efull0 + 8 * e, 1);
            tc::mbar_init(eempty0 + 8 * e, C::kEpiWarps);
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
    // the set-up above overlaps the previous kernel; activations, scales and
    // y are touched only after it completed
    pdl_wait();

    if (warp == 0) {
        // ---------------------------------------------------- TMA producer
        if (lane == 0) {
            uint32_t k = 0, j = 0;  // stages, epilogue-data groups issued
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < a.n_tiles; tile += gridDim.x) {
                const int row0 = (tile / a.n_ttiles) * kM, t0 = (tile % a.n_ttiles) * NT;
                for (int b0 = 0; b0 < a.nb; b0 += kG) {
                    if (b0 % kEB == 0) {
                        const int e = j % kES;
                        if (!tc::mbar_wait(eempty0 + 8 * e, ((j / kES) & 1u) ^ 1u, abort_flag, &g_f16_status, 21, true, a.wait_ns)) {
                            ok = false;
                            break;
                        }
                        const uint32_t ed = sbase + C::kEpiOff + e * C::kEpi;
                        tc::mbar_expect_tx(efull0 + 8 * e, C::kEpi);
                        tc::tma_load_2d(ed, &smap, b0, row0, efull0 + 8 * e);
                        tc::tma_load_2d(ed + C::kDw, &dmap, t0, b0, efull0 + 8 * e);
                        ++j;
                    }
                    const int s = k % C::kS;
                    // the slot's previous stage, k - kS, was converted and multiplied
                    if (k >= (uint32_t)C::kS) {
                        const uint32_t pk = k - C::kS;
                        if (!tc::mbar_wait(done0 + 8 * (pk % C::kR), (pk / C::kR) & 1u, abort_flag, &g_f16_status,
                                           22, true, a.wait_ns)) {
                            ok = false;
                            break;
                        }
                    }
                    const uint32_t st = sbase + C::kStageOff + s * C::kStage;
                    tc::mbar_expect_tx(full0 + 8 * s, C::kB + C::kRaw);
                    tc::tma_load_2d(st, &xmap, b0 * 32, t0, full0 + 8 * s);
                    tc::tma_load_2d(st + C::kB, &wmap, b0 * 16, row0, full0 + 8 * s);
                    ++k;
                }
            }
            // drain: the latest load of every slot has landed before the CTA exits
            for (uint32_t i = k > (uint32_t)C::kS ? k - C::kS : 0; i < k; ++i)
                tc::mbar_wait(full0 + 8 * (i % C::kS), (i / C::kS) & 1u, abort_flag, &g_f16_status, 23, false, a.wait_ns);
            for (uint32_t i = j > (uint32_t)kES ? j - kES : 0; i < j; ++i)
                tc::mbar_wait(efull0 + 8 * (i % kES), (i / kES) & 1u, abort_flag, &g_f16_status, 24, false, a.wait_ns);
        }
    } else if (warp <= kMmaWarps) {
        // --------------------------------------------------- MMA issuers
        // (an issuing thread spends tens of cycles per MMA, commit and
        // wait: two threads take the stages in turn)
        const uint32_t mine = warp - 1;
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(kM, NT);
            uint32_t k = 0;  // stages
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < a.n_tiles; tile += gridDim.x) {
                for (int b0 = 0; b0 < a.nb; b0 += kG, ++k) {
                    if (k % kMmaWarps != mine) continue;
                    const int ai = k % C::kSA, pr = k % C::kPairs, s = k % C::kS;
                    if (!tc::mbar_wait(aready0 + 8 * ai, (k / C::kSA) & 1u, abort_flag, &g_f16_status, 25, true, a.wait_ns) ||
                        !tc::mbar_wait(tempty0 + 8 * pr, ((k / C::kPairs) & 1u) ^ 1u, abort_flag, &g_f16_status,
                                       26, true, a.wait_ns)) {
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
                    const uint64_t ad = tc::sdesc_kmajor_sw128(sbase + ai * C::kA);
                    const uint64_t bd = tc::sdesc_kmajor_sw128(sbase + C::kStageOff + s * C::kStage);
                    const int nblk = a.nb - b0 < kG ? a.nb - b0 : kG;
                    for (int g = 0; g < nblk; ++g) {
                        // block g: K slices 2g, 2g+1 of 16 fp16 = 32 bytes each (+2 in the address field)
                        const uint32_t d = tmem + (2 * pr + g) * NT;
                        mma_f16(d, ad + 2 * (2 * g), bd + 2 * (2 * g), idesc, 0u);
                        mma_f16(d, ad + 2 * (2 * g + 1), bd + 2 * (2 * g + 1), idesc, 1u);
                    }
                    if ((int)k != a.skip_commit) tc::mma_commit(done0 + 8 * (k % C::kR));
                }
            }
            // every MMA issued has completed before TMEM is released
            tc::mma_commit(done_bar);
            tc::mbar_wait(done_bar, 0, abort_flag, &g_f16_status, 27, false, a.wait_ns);
        }
    } else if (warp < kEpi0) {
        // ------------------------------------------------------ converters
        const int r = quad * 32 + lane;  // row of the tile
        uint32_t k = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < a.n_tiles; tile += gridDim.x) {
            for (int b0 = 0; b0 < a.nb; b0 += kG, ++k) {
                const int s = k % C::kS, ai = k % C::kSA;
                // the A slot's previous stage, k - kSA, was multiplied
                const uint32_t pk = k - C::kSA;
                const bool got =
                    tc::mbar_wait(full0 + 8 * s, (k / C::kS) & 1u, abort_flag, &g_f16_status, 28, true, a.wait_ns) &&
                    (k < (uint32_t)C::kSA ||
                     tc::mbar_wait(done0 + 8 * (pk % C::kR), (pk / C::kR) & 1u, abort_flag, &g_f16_status, 31, true, a.wait_ns));
                if (!__all_sync(0xffffffffu, got)) {
                    ok = false;
                    break;
                }
                const uint4* raw = reinterpret_cast<const uint4*>(sm + C::kStageOff + s * C::kStage + C::kB + r * 32);
                unsigned char* arow = sm + ai * C::kA + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
                for (int g = 0; g < kG; ++g) {
                    // GGUF order: byte i holds element i (low nibble) and 16 + i (high)
                    const uint4 w = raw[g];
                    const uint4 c[4] = {
                        make_uint4(nib_pair(w.x, 0x4140u, 0), nib_pair(w.x, 0x4342u, 0), nib_pair(w.y, 0x4140u, 0),
                                   nib_pair(w.y, 0x4342u, 0)),
                        make_uint4(nib_pair(w.z, 0x4140u, 0), nib_pair(w.z, 0x4342u, 0), nib_pair(w.w, 0x4140u, 0),
                                   nib_pair(w.w, 0x4342u, 0)),
                        make_uint4(nib_pair(w.x, 0x4140u, 4), nib_pair(w.x, 0x4342u, 4), nib_pair(w.y, 0x4140u, 4),
                                   nib_pair(w.y, 0x4342u, 4)),
                        make_uint4(nib_pair(w.z, 0x4140u, 4), nib_pair(w.z, 0x4342u, 4), nib_pair(w.w, 0x4140u, 4),
                                   nib_pair(w.w, 0x4342u, 4))};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int chunk = 4 * g + q;  // 128-byte swizzle: chunk j of row r at j ^ (r & 7)
                        *reinterpret_cast<uint4*>(arow + ((chunk ^ (r & 7)) << 4)) = c[q];
                    }
                }
                tc::fence_proxy_async_smem();  // generic-proxy writes -> the tensor core's reads
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(aready0 + 8 * ai);
            }
        }
    } else {
        // -------------------------------------------------------- epilogue
        const int slice = (warp - kEpi0) >> 2;  // tokens slice*32 .. +31 of a tile
        const int rr = quad * 32 + lane;        // row of the tile = TMEM lane
        const int dsw = (rr >> 2) & 1;          // 32-byte swizzle phase of this row's weight scales
        const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16) + slice * TT;
        uint32_t ke = 0, j = 0;  // stages, epilogue-data groups consumed
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < a.n_tiles; tile += gridDim.x) {
            const int r = (tile / a.n_ttiles) * kM + rr;
            const int tb = (tile % a.n_ttiles) * NT + slice * TT;
            uint64_t acc[TT / 2];  // token pairs, (+0, +0) first
#pragma unroll
            for (int t = 0; t < TT / 2; ++t) acc[t] = 0ull;
            for (int b16 = 0; ok && b16 < a.nb; b16 += kEB) {
                const int e = j % kES;
                if (!__all_sync(0xffffffffu,
                                tc::mbar_wait(efull0 + 8 * e, (j / kES) & 1u, abort_flag, &g_f16_status, 29, true, a.wait_ns))) {
                    ok = false;
                    break;
                }
                const unsigned char* ed = sm + C::kEpiOff + e * C::kEpi;
                // this row's 16 fp16 weight scales: blocks 8c..8c+7 in 16-byte chunk c ^ dsw
                const unsigned char* dwrow = ed + rr * 32;
                const float* da = reinterpret_cast<const float*>(ed + C::kDw);  // [16][NT]
                const int neb = a.nb - b16 < kEB ? a.nb - b16 : kEB;
                // the group's pairs unrolled; a stage's two blocks per TMEM round trip
                // (LB = 2: both slots loaded, one wait) or, at 128 tokens, each
                // block in two 16-column halves (registers: no spills)
#pragma unroll
                for (int eb = 0; eb < kEB; eb += 2, ++ke) {
                    if (eb >= neb) break;                        // warp-uniform
                    const int nl = neb - eb < 2 ? neb - eb : 2;  // warp-uniform
                    const uint32_t pr = ke % C::kPairs;
                    // warp-uniform outcome: the TMEM loads below are .sync.aligned
                    if (!__all_sync(0xffffffffu, tc::mbar_wait(done0 + 8 * (ke % C::kR), (ke / C::kR) & 1u, abort_flag,
                                                               &g_f16_status, 30, true, a.wait_ns))) {
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
                    // the pair's two weight scales (blocks eb, eb + 1)
                    const uint32_t word =
                        *reinterpret_cast<const uint32_t*>(dwrow + (((eb >> 3) ^ dsw) << 4) + (eb & 7) * 2);
                    // the products of block b with its TMEM values w (tokens 4*t4.. of this warp's slice)
                    auto step = [&](int b, int t4, const uint32_t* w) {
                        const float dw = half_bits_to_float((unsigned short)((b & 1) ? word >> 16 : word));
                        const uint64_t dw2 = pack2(dw, dw);
                        const ulonglong2 d4 = reinterpret_cast<const ulonglong2*>(da + b * NT + slice * TT)[t4];
                        const uint64_t v0 = (uint64_t)w[0] | ((uint64_t)w[1] << 32);
                        const uint64_t v1 = (uint64_t)w[2] | ((uint64_t)w[3] << 32);
                        // fma(fp16(d_w) * d_a, float(isum), sum): the product rounded first
                        acc[2 * t4] = tc::f2_fma(tc::f2_mul(dw2, d4.x), v0, acc[2 * t4]);
                        acc[2 * t4 + 1] = tc::f2_fma(tc::f2_mul(dw2, d4.y), v1, acc[2 * t4 + 1]);
                    };
                    auto release = [&]() {  // the pair's last loads: the slots are free for the MMAs
                        tc::tc_fence_before();
                        __syncwarp();
                        if (lane == 0) tc::mbar_arrive(tempty0 + 8 * pr);
                    };
                    if constexpr (LB == 2) {
                        uint32_t v[2][TT];
#pragma unroll
                        for (int i = 0; i < 2; ++i)
                            if (i < nl) tc::tmem_ld32(tl + (2 * pr + i) * NT, v[i]);
                        tc::tmem_wait_ld();
                        release();
#pragma unroll
                        for (int i = 0; i < 2; ++i)
                            if (i < nl) {
#pragma unroll
                                for (int t4 = 0; t4 < TT / 4; ++t4) step(eb + i, t4, &v[i][4 * t4]);
                            }
                    } else {
#pragma unroll
                        for (int i = 0; i < 2; ++i) {
                            if (i >= nl) break;
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                uint32_t v[TT / 2];
                                tc::tmem_ld16(tl + (2 * pr + i) * NT + h * (TT / 2), v);
                                tc::tmem_wait_ld();
                                if (i == nl - 1 && h == 1) release();
#pragma unroll
                                for (int t4 = 0; t4 < TT / 8; ++t4) step(eb + i, h * (TT / 8) + t4, &v[4 * t4]);
                            }
                        }
                    }
                }
                if (!ok) break;
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(eempty0 + 8 * e);
                ++j;
            }
            if (!ok) break;
            if (r < a.rows) {
#pragma unroll
                for (int t = 0; t < TT; ++t) {
                    if (tb + t < a.batch) {
                        const float val = __uint_as_float((uint32_t)(acc[t / 2] >> (32 * (t & 1))));
                        float* p = a.y + (size_t)(tb + t) * a.ldy + r;
                        *p = a.accumulate ? *p + val : val;
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

// Test hook (gemm_f16_test_stall): one launch with a shorter wait bound and
// one MMA commit left out, so that its waits run out and it returns with a
// status instead of its results.
struct TestStall {
    uint64_t wait_ns = tc::kWaitLimitNs;
    int skip_commit = -1;
};
std::mutex g_stall_mu;
TestStall g_stall;

TestStall take_test_stall() {
    std::lock_guard<std::mutex> lock(g_stall_mu);
    const TestStall t = g_stall;
    g_stall = TestStall{};
    return t;
}

template <int NT>
cudaError_t launch_f16(const mv_weight_s& w, const uint16_t* qh, const float* dT, uint64_t ldb, uint64_t batch,
                       float* y, uint64_t ldy, cudaStream_t s, bool accumulate) {
    using C = Cfg<NT>;
    const tc::EncodeFn enc = tc::encode_fn();
    if (!enc) {
        set_last_error("cuTensorMapEncodeTiled is unavailable in this driver");
        return cudaErrorNotSupported;
    }
    CUtensorMap wmap, xmap, dmap, smap;
    // payload plane [rows][nb*16 B] -> raw [128][32 B]
    const cuuint64_t wdims[2] = {w.nb * 16, w.rows}, wstr[1] = {w.nb * 16};
    const cuuint32_t wbox[2] = {(cuuint32_t)(kG * 16), (cuuint32_t)kM};
    // fp16 activations [batch][K] -> B [NT][128 B], 128-byte swizzle
    const cuuint64_t xdims[2] = {w.nb * 32, batch}, xstr[1] = {w.nb * 32 * 2};
    const cuuint32_t xbox[2] = {(cuuint32_t)(kG * 32), (cuuint32_t)NT};
    // activation scales [nb][ldb] fp32 -> [16][NT]
    const cuuint64_t ddims[2] = {ldb, w.nb}, dstr[1] = {ldb * 4};
    const cuuint32_t dbox[2] = {(cuuint32_t)NT, (cuuint32_t)kEB};
    // weight scales [rows][dstride] fp16 -> [128][16], 32-byte swizzle
    const cuuint64_t sdims[2] = {w.dstride, w.rows}, sstr[1] = {w.dstride * 2};
    const cuuint32_t sbox[2] = {(cuuint32_t)kEB, (cuuint32_t)kM};
    if (!tc::encode(enc, &wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w.qs, wdims, wstr, wbox, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !tc::encode(enc, &xmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t*>(qh), xdims, xstr, xbox,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
        !tc::encode(enc, &dmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(dT), ddims, dstr, dbox,
                    CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !tc::encode(enc, &smap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, w.d, sdims, sstr, sbox, CU_TENSOR_MAP_SWIZZLE_32B)) {
        set_last_error("cuTensorMapEncodeTiled rejected a tensor map of the fp16 tensor-core GEMM");
        return cudaErrorInvalidValue;
    }
    const int n_ttiles = (int)((batch + NT - 1) / NT);
    const int n_tiles = (int)((w.rows + kM - 1) / kM) * n_ttiles;
    const TestStall ts = take_test_stall();
    const F16Args args{y,        (int)w.rows,         (int)w.nb, (int)batch, n_ttiles, n_tiles, accumulate ? 1 : 0,
                       (int)ldy, ts.wait_ns,          ts.skip_commit};
    ensure_smem_attr(gemm_f16_kernel<NT>, C::kSmem);
    const int grid = n_tiles < num_sms() ? n_tiles : num_sms();
    return launch_pdl(gemm_f16_kernel<NT>, dim3(grid), dim3(C::kThreads), C::kSmem, s, wmap, xmap, dmap, smap, args);
}

}  // namespace

void gemm_f16_test_stall(int skip_commit, uint64_t wait_ns) {
    std::lock_guard<std::mutex> lock(g_stall_mu);
    g_stall.skip_commit = skip_commit;
    g_stall.wait_ns = wait_ns ? wait_ns : tc::kWaitLimitNs;
}

bool gemm_f16_preferred(uint64_t batch) {
    static const bool off = [] {
        const char* e = std::getenv("MV_GEMM_F16");
        return e && std::string(e) == "0";
    }();
    return batch >= 64 && !off;
}

cudaError_t gemm_q4_q8_f16(const mv_weight_s& w, const uint16_t* qh, const float* dT, uint64_t ldb, uint64_t batch,
                           float* y, cudaStream_t s, bool accumulate) {
    if (!batch) return cudaSuccess;
    if (w.type != 2 || ldb < gemm_tc_ldb(batch) || ldb % 4 || w.rows >= (1ull << 31) || batch >= (1ull << 31))
        return cudaErrorInvalidValue;
    // Token-tile width: a tile's time is a fixed part (the converters expand
    // the weight tile whatever its width, the MMA issue and the hand-offs)
    // plus a part per token (measured at K = 4096: ~19.5 us + 0.42 us per
    // token); tiles run in waves of one per SM.  Wide tiles share the fixed
    // part among more tokens, narrow ones give narrow weights (o, down: 32
    // row tiles) enough tiles to fill the SMs.  (Checked at 512 tokens on the
    // four 7B shapes: 128-token tiles 213 / 81 / 344 / 205 us against 267 / 95 /
    // 449 / 248 with 64 and 393 / 153 / 666 / 401 with 32; with the epilogue
    // free of spills the 128-token tiles take 179 / 76 / 294 / 170 us, about
    // 61 us per tile at K = 4096, so the model's choices for these shapes stand.)
    const uint64_t row_tiles = (w.rows + kM - 1) / kM, sms = (uint64_t)num_sms();
    int best = 128;
    double best_t = 1e30;
    for (int nt : {128, 64, 32}) {
        const uint64_t tiles = row_tiles * ((batch + nt - 1) / nt);
        const double t = (double)((tiles + sms - 1) / sms) * (19.5 + 0.42 * nt);
        if (t < best_t * 0.999) best_t = t, best = nt;
    }
    if (best == 128) return launch_f16<128>(w, qh, dT, ldb, batch, y, w.rows, s, accumulate);
    if (best == 64) return launch_f16<64>(w, qh, dT, ldb, batch, y, w.rows, s, accumulate);
    return launch_f16<32>(w, qh, dT, ldb, batch, y, w.rows, s, accumulate);
}

}  // namespace mvb
