// decode_mk.cu -- the layers of one decode step (LlamaModel::forward,
// src/llama_model.cpp:253-259) as ONE persistent kernel: one CTA per SM,
// launched cooperatively so every CTA is resident at once.
//
// Why.  A token reads 3.75 GB of weights, so decode is HBM-bound, but as a
// chain of 160 dependent kernels (5 per layer) every kernel boundary drains
// the memory pipeline: the next GEMV cannot start streaming its weights
// until the previous one has left the SMs, and its activation prologue
// (RMSNorm + Q8 quantisation) then runs with HBM idle.  Here the weight
// stream never stops: a producer warp in every CTA walks this CTA's share of
// every layer's weight tiles, in the order they will be used, and keeps a
// ring of shared-memory stages full with bulk copies (cp.async.bulk, no
// multicast) regardless of phase boundaries.  The activations move through
// grid-wide barriers; while one phase waits for the whole grid (or for the
// attention of a layer), the rings fill with the next phases' tiles.
//
// Per layer, five phases separated by grid barriers:
//   QKV   x -> RMSNorm -> Q8 -> q|k|v rows (exact GEMV chain)       -> qkv
//   ATT   one CTA per query head: RoPE, KV append, exact attention -> att
//   O     att -> Q8 -> o rows, added to the residual                -> x
//   GU    x -> RMSNorm -> Q8 -> (gate_i, up_i) rows, SiLU gate        -> ff
//   DOWN  ff -> Q8 -> down rows, added to the residual              -> x
// The arithmetic is exactly that of the separate kernels (gemv_q4.cu's row
// tile and attention.cu's fused decode attention): per 32-element block the
// dp4a integer dot, fp16(d_w) * d_a, and one lane per row running the
// reference's FMA chain over the blocks in order; attention in the
// reference's order (8-lane key dots, double denominator, per-dimension FMA
// chain over the tokens).  Outputs are bit-identical to the per-kernel path.
//
// Work split: a GEMV phase's tiles (16 rows x all blocks) go round-robin over
// the CTAs, the starting CTA rotating from phase to phase so the CTAs that
// took one tile more in one phase take one less later.  A tile is streamed
// as chunks of 32 blocks (16 x 512 B of nibbles + 16 x 64 B of scales).
//
// Warps: 16 compute warps turn a staged chunk into per-block terms
// (d_w * d_a, float(isum)), warp w for row w of the tile and lane b for
// block b of the chunk; warp 16 runs the 16 rows' chains and writes the
// outputs; warp 17 is the producer.  Warps 0-16 also run each phase's
// prologue (one pass, x held in registers, the RMSNorm weights fetched
// before the barrier) and, in CTAs 0..n_head-1, the attention, whose cached
// K/V are requested at the start of the layer.
//
// Every wait is bounded (2 s without progress, tc::mbar_wait and the grid
// barrier's spin): a wait that runs out raises the device-wide abort word
// (status[1]) and records a site code (status[0]); every CTA then runs its
// remaining phases as no-ops, the producer drains the copies it has in
// flight, and the kernel returns.  The host reads the status word after the
// step and clears it.
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"
#include "kernels.cuh"
#include "tc.cuh"

namespace mvb {

namespace {

constexpr int kComp = 16;                    // compute warps (warp w = row w of a tile)
constexpr int kProdWarp = kComp + 1;         // warp 17
constexpr int kWork = (kComp + 1) * 32;      // compute + chain threads
constexpr int kThreads = kWork + 32;         // + producer
constexpr int kTR = 16;                      // rows per tile
constexpr int kTC = 32;                      // blocks per chunk
constexpr int kPayRow = kTC * 16;            // staged nibble bytes per row (one TMA box row)
constexpr int kScRow = kTC * 2;              // staged scale bytes per row
constexpr int kStage = kTR * (kPayRow + kScRow);
constexpr int kTT = kTC + 2;                 // float2 per term row (padded)
constexpr int kMaxNb = 384;                  // blocks of the widest input (K <= 12288)

// named barriers (0 is not used once the producer has split off)
constexpr int kBarHand = 2;  // compute warps + chain warp: terms hand-off
constexpr int kBarWork = 3;  // compute warps + chain warp: phase boundaries
constexpr int kBarAttn = 4;  // the HD attention threads

__device__ __forceinline__ void bar_named(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ float expf_cr(float x) { return (float)exp((double)x); }

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

constexpr uint32_t kLoNib = 0x0F0F0F0Fu;
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// sum_k (nib_k - 8) * a_k of one block (as gemv_q4.cu): the low nibbles
// against elements 0..15, the high nibbles in place (an unsigned dot) against
// elements 16..31 and shifted back, minus c8 = 8 * sum(a)
__device__ __forceinline__ int block_isum(const uint4 w, const int4 alo, const int4 ahi, int c8) {
    int s = dp4a((int)(w.x & kLoNib), alo.x, 0);
    s = dp4a((int)(w.y & kLoNib), alo.y, s);
    s = dp4a((int)(w.z & kLoNib), alo.z, s);
    s = dp4a((int)(w.w & kLoNib), alo.w, s);
    int h = dp4a_us(w.x & ~kLoNib, ahi.x, 0);
    h = dp4a_us(w.y & ~kLoNib, ahi.y, h);
    h = dp4a_us(w.z & ~kLoNib, ahi.z, h);
    h = dp4a_us(w.w & ~kLoNib, ahi.w, h);
    return s + (h >> 4) - c8;
}

// ------------------------------------------------------------ layout
// Attention staging (the fused decode attention's plan).
__host__ __device__ inline int mk_ktile(int hd, int kv_type) {
    const int esize = kv_type == 0 ? 4 : 2;
    int kt = 65536 / (hd * esize + 16);
    if (kt > hd) kt = hd;
    if (kt > 64) kt = 64;
    return kt / 32 * 32;
}
constexpr int kVTile = 32;
__host__ __device__ inline int mk_vstages(int hd, int kv_type) { return hd * (kv_type == 0 ? 4 : 2) <= 256 ? 5 : 4; }

struct MkSmem {
    uint32_t act, terms, q, table, sc, knew, vnew, kring, vring, ring, bars, flag, total;
};
__host__ __device__ inline MkSmem mk_plan(int hd, int max_ctx, int max_pages, int kv_type, int stages) {
    auto up = [](uint32_t n) { return (n + 127u) / 128u * 128u; };
    const uint32_t esize = kv_type == 0 ? 4 : 2;
    MkSmem p;
    p.act = 0;                                          // lo, hi int4 + dc float2 per block
    p.terms = up(kMaxNb * 40);
    p.q = p.terms + up(2 * kTR * kTT * 8);
    p.table = p.q + up(hd * 4);
    p.sc = p.table + up(max_pages * 4);
    p.knew = p.sc + up((max_ctx + 1) * 4);
    p.vnew = p.knew + up(hd * esize);
    p.kring = p.vnew + up(hd * esize);
    p.vring = p.kring + up(2 * mk_ktile(hd, kv_type) * (hd * esize + 16));
    p.ring = p.vring + up(mk_vstages(hd, kv_type) * kVTile * hd * esize);
    p.bars = p.ring + (uint32_t)stages * kStage;
    p.flag = p.bars + 2 * 8 * stages;
    p.total = p.flag + 16;
    return p;
}

// ----------------------------------------------------------- sequence
// The tiles of GEMV phase `ph` of layer `l` that CTA `cta` of `G` owns:
// t = t0, t0 + G, ... < T.  `off` is the phase's rotation (sum of the tile
// counts of the phases before it, mod G).
struct Seq {
    int T, nch, t0;
};
__device__ __forceinline__ Seq seq_of(const MkGemv& w, int cta, int G, int off) {
    Seq q;
    q.T = (w.rows + kTR - 1) / kTR;
    q.nch = (w.nb + kTC - 1) / kTC;
    q.t0 = ((cta - off) % G + G) % G;
    return q;
}

// ------------------------------------------------------- grid barrier
// Arrive (after the CTA's outputs of the phase), then wait until all G CTAs
// of barrier `n` (1-based, counted from the launch) have arrived.  Called by
// the kWork threads; thread 0 does the atomic and the spin.
__device__ __forceinline__ void grid_sync(const MkArgs& a, unsigned n, volatile int* cta_abort) {
    bar_named(kBarWork, kWork);
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(a.bar, 1u);
        const unsigned target = n * gridDim.x;
        if (!*cta_abort) {
            const uint64_t t0 = tc::globaltimer();
            for (uint32_t i = 0;; ++i) {
                if (ld_acquire_u32(a.bar) >= target) break;
                if ((i & 15u) == 15u) {
                    if (*(volatile int*)(a.status + 1)) {
                        *cta_abort = 1;
                        break;
                    }
                    if (tc::globaltimer() - t0 > tc::kWaitLimitNs) {
                        *(volatile int*)(a.status + 1) = 1;
                        atomicCAS(a.status, 0, 40);
                        *cta_abort = 1;
                        break;
                    }
                }
            }
        }
        __threadfence();
        if (*(volatile int*)(a.status + 1)) *cta_abort = 1;
    }
    bar_named(kBarWork, kWork);
}

// --------------------------------------------------- activation prologue
struct Act {
    int4* lo;
    int4* hi;
    float2* dc;
};

// Groups of 8 activations a work thread owns at most (kMaxNb * 4 groups).
constexpr int kKeep = (kMaxNb * 4 + kWork - 1) / kWork;

// RMSNorm weights of this thread's groups: immutable, so fetched before the
// grid barrier that precedes the prologue.  The normalised input is n_embd
// wide: at most kNormKeep groups per thread (n_embd <= kNormKeep * 8 * kWork).
constexpr int kNormKeep = 2;
struct NormPre {
    float4 w[kNormKeep][2];
};
__device__ __forceinline__ void norm_fetch(NormPre& np, const float* __restrict__ norm_w, int nb) {
    const int G = nb * 4, tid = threadIdx.x;
#pragma unroll
    for (int it = 0; it < kNormKeep; ++it) {
        const int g = tid + it * kWork;
        np.w[it][0] = np.w[it][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (g < G) {
            np.w[it][0] = __ldg(reinterpret_cast<const float4*>(norm_w) + 2 * g);
            np.w[it][1] = __ldg(reinterpret_cast<const float4*>(norm_w) + 2 * g + 1);
        }
    }
}

// Quantised activations of x (optionally RMS-normalised: np != nullptr) into
// shared memory, by the kWork threads, in one pass: every thread's groups of
// x are loaded at once and kept in registers through the sum of squares and
// the quantisation.  x was written by other CTAs in this launch: it is read
// from L2 (ld.cg), never from a possibly stale L1 line.
__device__ void prologue(const float* x, const NormPre* np, float eps, int nb, const Act& a, double* red) {
    const int G = nb * 4, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int iters = (G + kWork - 1) / kWork;  // uniform
    const float4* x4 = reinterpret_cast<const float4*>(x);
    float4 xv[kKeep][2];
#pragma unroll
    for (int it = 0; it < kKeep; ++it) {
        const int g = tid + it * kWork;
        xv[it][0] = xv[it][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (it < iters && g < G) {
            xv[it][0] = __ldcg(x4 + 2 * g);
            xv[it][1] = __ldcg(x4 + 2 * g + 1);
        }
    }
    float inv = 1.0f;
    if (np) {
        double ss = 0.0;
#pragma unroll
        for (int it = 0; it < kKeep; ++it) {
            const float4 u = xv[it][0], v = xv[it][1];
            ss += (double)u.x * u.x + (double)u.y * u.y + (double)u.z * u.z + (double)u.w * u.w;
            ss += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
        }
        ss = warp_sum_d(ss);
        if (lane == 0) red[warp] = ss;
        bar_named(kBarWork, kWork);
        double tot = 0.0;
#pragma unroll
        for (int w = 0; w < kWork / 32; ++w) tot += red[w];
        inv = 1.0f / sqrtf((float)(tot / (double)(nb * 32)) + eps);
    }
#pragma unroll
    for (int it = 0; it < kKeep; ++it) {
        if (it >= iters) break;  // uniform across the CTA
        const int g = tid + it * kWork;
        const bool active = g < G;  // uniform over the 4 lanes of a block
        float v[8] = {xv[it][0].x, xv[it][0].y, xv[it][0].z, xv[it][0].w,
                      xv[it][1].x, xv[it][1].y, xv[it][1].z, xv[it][1].w};
        if (np && it < kNormKeep) {
            const float nw[8] = {np->w[it][0].x, np->w[it][0].y, np->w[it][0].z, np->w[it][0].w,
                                 np->w[it][1].x, np->w[it][1].y, np->w[it][1].z, np->w[it][1].w};
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = v[i] * inv * nw[i];  // (x*inv)*w as the reference
        }
        // quantize_q8 (src/gguf_kernels.cpp:161-172): 4 neighbouring lanes hold one block
        float m = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(v[i]));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        const float d = m > 0.0f ? m / 127.0f : 1.0f;
        const float id = 1.0f / d;
        uint32_t pk[2] = {0u, 0u};
        int sum = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int q = (int)fminf(fmaxf(roundf(v[i] * id), -127.0f), 127.0f);
            sum += q;
            pk[i >> 2] |= (uint32_t)(q & 0xff) << (8 * (i & 3));
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if (active) {
            const int b = g >> 2, sub = g & 3;
            *(reinterpret_cast<uint2*>(sub < 2 ? &a.lo[b] : &a.hi[b]) + (sub & 1)) = make_uint2(pk[0], pk[1]);
            if (sub == 0) a.dc[b] = make_float2(d, __int_as_float(8 * sum));
        }
    }
    bar_named(kBarWork, kWork);
}

// --------------------------------------------------------- attention
// One query head, by threads 0..HD-1 of the work group: the fused decode
// attention of attention.cu (attn_decode_fused_kernel, one-GPU form) with
// named barriers in place of __syncthreads.  prefetch() issues the cached
// K/V loads (tokens 0..p-1 were written by earlier steps), run() does the rest
// once the q|k|v rows of this token are complete.
template <int HD, int VS>
struct Attn {
    const MkArgs& a;
    const MkLayer& L;
    unsigned char* sm;
    MkSmem P;
    int h, tid, kh, p, npg, KT, nkt, nvt;
    size_t row_bytes, head_off;
    int slice, kvt, esize;

    __device__ Attn(const MkArgs& a_, const MkLayer& L_, unsigned char* sm_, const MkSmem& P_, int h_)
        : a(a_), L(L_), sm(sm_), P(P_), h(h_) {
        tid = threadIdx.x;
        const int G = a.n_head / a.n_head_kv;
        kh = h / G;
        kvt = a.kv_type;
        esize = kvt == 0 ? 4 : 2;
        row_bytes = (size_t)a.n_head_kv * HD * esize;
        head_off = (size_t)kh * HD * esize;
        slice = HD * esize;
        p = a.pos[0];
        npg = (p + a.page) / a.page;
        KT = mk_ktile(HD, kvt);
        nkt = (p + KT - 1) / KT;
        nvt = (p + kVTile - 1) / kVTile;
    }
    __device__ int* tbl() const { return reinterpret_cast<int*>(sm + P.table); }
    __device__ size_t slot_of(int t) const { return (size_t)tbl()[t / a.page] * a.page + t % a.page; }

    __device__ void issue_k(int tile, int buf) const {
        const int t = tile * KT + tid;
        if (tid < KT && t < p) {
            const uint8_t* src = L.k_pages + slot_of(t) * row_bytes + head_off;
            uint8_t* dst = sm + P.kring + ((size_t)buf * KT + tid) * (slice + 16);
            for (int c = 0; c < slice; c += 16) cp_async16(dst + c, src + c);
        }
        cp_async_commit();
    }
    __device__ void issue_v(int tile) const {
        if (tile < nvt) {
            const int chunks = kVTile * slice / 16;
            uint8_t* dst = sm + P.vring + (size_t)(tile % VS) * kVTile * slice;
            for (int c = tid; c < chunks; c += HD) {
                const int tt = c / (slice / 16), off = (c % (slice / 16)) * 16;
                const int t = tile * kVTile + tt;
                if (t < p) cp_async16(dst + tt * slice + off, L.v_pages + slot_of(t) * row_bytes + head_off + off);
            }
        }
        cp_async_commit();
    }
    // threads < HD: block table, then V tiles 0..VS-2 and K tiles 0, 1 in flight
    __device__ void prefetch() const {
        for (int i = tid; i < npg; i += HD) tbl()[i] = a.block_table[i];
        bar_named(kBarAttn, HD);
        for (int k = 0; k < VS - 1; ++k) issue_v(k);
        issue_k(0, 0);
        if (nkt > 1) issue_k(1, 1);
    }

    __device__ float dot_row(const uint8_t* krw, const float* qs) const {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (kvt == 1) {
#pragma unroll 4
            for (int d = 0; d < HD; d += 8) {
                const uint4 w = *reinterpret_cast<const uint4*>(krw + d * 2);
                const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int l = 0; l < 8; ++l)
                    acc[l] = fmaf(qs[d + l], half_bits_to_float((unsigned short)(ws[l / 2] >> (16 * (l & 1)))), acc[l]);
            }
        } else {
#pragma unroll 4
            for (int d = 0; d < HD; d += 8) {
                const float4 u = *reinterpret_cast<const float4*>(krw + d * 4);
                const float4 v = *reinterpret_cast<const float4*>(krw + d * 4 + 16);
                const float ks[8] = {u.x, u.y, u.z, u.w, v.x, v.y, v.z, v.w};
#pragma unroll
                for (int l = 0; l < 8; ++l) acc[l] = fmaf(qs[d + l], ks[l], acc[l]);
            }
        }
        float dot = acc[0];
#pragma unroll
        for (int l = 1; l < 8; ++l) dot += acc[l];
        return dot / sqrtf((float)HD);
    }

    __device__ void run(float* redf, double* redd) const {
        const int lane = tid & 31, warp = tid >> 5, half = HD / 2;
        const int D = a.n_head * HD, kv_dim = a.n_head_kv * HD;
        float* qs = reinterpret_cast<float*>(sm + P.q);
        float* sc = reinterpret_cast<float*>(sm + P.sc);
        uint8_t* knew = sm + P.knew;
        uint8_t* vnew = sm + P.vnew;
        const uint8_t* kring = sm + P.kring;
        const uint8_t* vring = sm + P.vring;
        const int G = a.n_head / a.n_head_kv;
        // this token: RoPE of q (head h) and k (kv head kh), k and v in cache form
        if (tid < half) {
            const float c = __ldg(a.cos_t + (size_t)p * half + tid), sn = __ldg(a.sin_t + (size_t)p * half + tid);
            const float q0 = __ldcg(a.qkv + h * HD + tid), q1 = __ldcg(a.qkv + h * HD + tid + half);
            qs[tid] = __fmaf_rn(q0, c, -__fmul_rn(q1, sn));
            qs[tid + half] = __fmaf_rn(q0, sn, __fmul_rn(q1, c));
            const float k0 = __ldcg(a.qkv + D + kh * HD + tid), k1 = __ldcg(a.qkv + D + kh * HD + tid + half);
            const float r0 = __fmaf_rn(k0, c, -__fmul_rn(k1, sn)), r1 = __fmaf_rn(k0, sn, __fmul_rn(k1, c));
            if (kvt == 1) {
                reinterpret_cast<uint16_t*>(knew)[tid] = f32_to_f16_ref(r0);
                reinterpret_cast<uint16_t*>(knew)[tid + half] = f32_to_f16_ref(r1);
            } else {
                reinterpret_cast<float*>(knew)[tid] = r0;
                reinterpret_cast<float*>(knew)[tid + half] = r1;
            }
        }
        {
            const float v = __ldcg(a.qkv + D + kv_dim + kh * HD + tid);
            if (kvt == 1) reinterpret_cast<uint16_t*>(vnew)[tid] = f32_to_f16_ref(v);
            else reinterpret_cast<float*>(vnew)[tid] = v;
        }
        bar_named(kBarAttn, HD);
        if (h % G == 0) {  // the cache rows of this token, once per kv head
            const size_t at = slot_of(p) * row_bytes + head_off;
            uint8_t* kd = L.k_pages + at;
            uint8_t* vd = L.v_pages + at;
            for (int i = tid; i < slice / 4; i += HD) {
                reinterpret_cast<uint32_t*>(kd)[i] = reinterpret_cast<const uint32_t*>(knew)[i];
                reinterpret_cast<uint32_t*>(vd)[i] = reinterpret_cast<const uint32_t*>(vnew)[i];
            }
        }
        if (h == 0 && tid == 0 && a.ctx_out) a.ctx_out[0] = p + 1;

        // 1. scores of the cached tokens (K tiles 0, 1 were issued by prefetch,
        //    tile t+1 after tile t-1: each thread reads only the rows it copied),
        //    then this token's
        for (int tile = 0; tile < nkt; ++tile) {
            if (tile >= 1 || nkt == 1) {
                if (tile >= 1 && tile + 1 < nkt) issue_k(tile + 1, (tile + 1) & 1);
                else cp_async_commit();
            }
            cp_async_wait<1>();
            const int t = tile * KT + tid;
            if (tid < KT && t < p) sc[t] = dot_row(kring + ((size_t)(tile & 1) * KT + tid) * (slice + 16), qs);
        }
        if (tid == (p % KT ? KT - 1 : 0)) sc[p] = dot_row(knew, qs);
        bar_named(kBarAttn, HD);

        // 2. max, exp, double denominator, weights (all p + 1 tokens)
        const int ctx = p + 1;
        float m = -INFINITY;
        for (int t = tid; t < ctx; t += HD) m = fmaxf(m, sc[t]);
        m = warp_max(m);
        if (lane == 0) redf[warp] = m;
        bar_named(kBarAttn, HD);
        m = redf[0];
#pragma unroll
        for (int w = 1; w < HD / 32; ++w) m = fmaxf(m, redf[w]);
        double den = 0.0;
        for (int t = tid; t < ctx; t += HD) {
            const float e = expf_cr(sc[t] - m);
            sc[t] = e;
            den += (double)e;
        }
        den = warp_sum_d(den);
        if (lane == 0) redd[warp] = den;
        bar_named(kBarAttn, HD);
        den = 0.0;
#pragma unroll
        for (int w = 0; w < HD / 32; ++w) den += redd[w];
        const float inv = (float)(1.0 / den);

        // 3. out_d = fma(alpha_t, v_t[d], out_d) over the cached tokens in order, then this token
        float out = 0.0f;
        for (int tile = 0; tile < nvt; ++tile) {
            cp_async_wait<VS - 2>();
            bar_named(kBarAttn, HD);  // the tile is visible to every thread
            const uint8_t* vt = vring + (size_t)(tile % VS) * kVTile * slice;
            const int n = min(kVTile, p - tile * kVTile);
            auto step = [&](int tt, float& v, float& al) {
                al = sc[tile * kVTile + tt] * inv;  // alpha_t = e_t * float(1/den)
                v = kvt == 1 ? half_bits_to_float(reinterpret_cast<const uint16_t*>(vt + tt * slice)[tid])
                             : reinterpret_cast<const float*>(vt + tt * slice)[tid];
            };
            int tt = 0;
            for (; tt + 8 <= n; tt += 8) {
                float v[8], al[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) step(tt + j, v[j], al[j]);
#pragma unroll
                for (int j = 0; j < 8; ++j) out = fmaf(al[j], v[j], out);
            }
            for (; tt < n; ++tt) {
                float v, al;
                step(tt, v, al);
                out = fmaf(al, v, out);
            }
            bar_named(kBarAttn, HD);  // everyone is done with this stage before it is refilled
            issue_v(tile + VS - 1);
        }
        cp_async_wait<0>();
        {
            const float al = sc[p] * inv;
            const float v = kvt == 1 ? half_bits_to_float(reinterpret_cast<const uint16_t*>(vnew)[tid])
                                     : reinterpret_cast<const float*>(vnew)[tid];
            out = fmaf(al, v, out);
        }
        a.att[(size_t)h * HD + tid] = out;
    }
};

// ------------------------------------------------------------- kernel
template <int HD, int VS>
__global__ void __launch_bounds__(kThreads, 1) decode_mk_kernel(const __grid_constant__ MkArgs a) {
    extern __shared__ __align__(128) unsigned char sm[];
    __shared__ double red[kWork / 32];
    __shared__ float redf[HD / 32];
    __shared__ double redd[HD / 32];
    const MkSmem P = mk_plan(HD, a.max_ctx, a.max_pages, a.kv_type, a.stages);
    const int S = a.stages;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int cta = blockIdx.x, G = gridDim.x;
    const uint32_t sbase = tc::smem_u32(sm);
    const uint32_t full0 = sbase + P.bars, empty0 = full0 + 8u * S;
    volatile int* cta_abort = reinterpret_cast<volatile int*>(sm + P.flag);

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            tc::mbar_init(full0 + 8 * s, 1);
            tc::mbar_init(empty0 + 8 * s, kComp);
        }
        *cta_abort = 0;
        tc::mbar_fence_init();
    }
    __syncthreads();

    if (warp == kProdWarp) {
        // ------------------------------------------------------ producer
        uint32_t k = 0, ks = 0, kpar = 0;  // chunks issued; stage and phase parity of chunk k
        bool ok = true;
        int off = 0;
        for (int l = 0; ok && l < a.n_layer; ++l) {
            const MkLayer& L = a.layers[l];
            for (int ph = 0; ok && ph < 4; ++ph) {
                const MkGemv& w = L.w[ph];
                const Seq q = seq_of(w, cta, G, off);
                off = (off + q.T) % G;
                for (int t = q.t0; ok && t < q.T; t += G) {
                    for (int c = 0; c < q.nch; ++c, ++k) {
                        const int s = (int)ks;
                        const uint32_t par = kpar;
                        if (++ks == (uint32_t)S) ks = 0, kpar ^= 1u;
                        ok = tc::mbar_wait(empty0 + 8 * s, par ^ 1u, a.status + 1, a.status, 41);
                        ok = __all_sync(0xffffffffu, ok);
                        if (!ok) break;
                        // one box of nibbles (16 rows x 512 B) and one of scales (16 rows x
                        // 64 B); columns past the row end arrive as zeros and count in full
                        if (lane == 0) {
                            const uint32_t st = sbase + P.ring + (uint32_t)s * kStage;
                            const CUtensorMap* mp = a.maps + 2 * (l * 4 + ph);
                            tc::mbar_expect_tx(full0 + 8 * s, kStage);
                            tc::tma_load_2d(st, mp, c * (kPayRow / 4), t * kTR, full0 + 8 * s);
                            tc::tma_load_2d(st + kTR * kPayRow, mp + 1, c * kTC, t * kTR, full0 + 8 * s);
                        }
                    }
                }
            }
        }
        // drain: the latest load of every stage has landed before the CTA exits
        if (lane == 0)
            for (uint32_t i = k > (uint32_t)S ? k - S : 0; i < k; ++i)
                tc::mbar_wait(full0 + 8 * (i % S), (i / S) & 1u, a.status + 1, a.status, 42, false);
        return;
    }

    // ------------------------------------------------------- work group
    const Act act{reinterpret_cast<int4*>(sm + P.act), reinterpret_cast<int4*>(sm + P.act) + kMaxNb,
                  reinterpret_cast<float2*>(reinterpret_cast<int4*>(sm + P.act) + 2 * kMaxNb)};
    float2* terms = reinterpret_cast<float2*>(sm + P.terms);
    unsigned nbar = 0;
    uint32_t ks = 0, kpar = 0;  // stage and phase parity of the next chunk
    int off = 0;
    const bool attn_cta = cta < a.n_head;

    // One GEMV phase of this CTA: its tiles, chunk by chunk.
    auto gemv = [&](const MkGemv& wg, int epi, float* y) {
        const MkGemv w = wg;  // in registers: the loops below store to global memory
        const Seq q = seq_of(w, cta, G, off);
        off = (off + q.T) % G;
        int it = 0;
        if (warp < kComp) {
            // warp w = row w of the tile, lane = block of the chunk: a warp reads
            // one staged row (512 contiguous bytes) -- no bank conflict
            const int row = warp, cb = lane;
            for (int t = q.t0; t < q.T; t += G) {
                for (int c = 0; c < q.nch; ++c, ++it) {
                    const int s = (int)ks;
                    const uint32_t par = kpar;
                    if (++ks == (uint32_t)S) ks = 0, kpar ^= 1u;
                    bool ok = !*cta_abort;
                    if (ok) ok = tc::mbar_wait(full0 + 8 * s, par, a.status + 1, a.status, 43);
                    ok = __all_sync(0xffffffffu, ok);
                    float2 o2 = make_float2(0.f, 0.f);
                    if (ok) {
                        const unsigned char* st = sm + P.ring + (size_t)s * kStage;
                        const int b = c * kTC + cb;
                        if (b < w.nb) {
                            const int4 alo = act.lo[b], ahi = act.hi[b];
                            const float2 dc = act.dc[b];
                            const uint4 wv = *reinterpret_cast<const uint4*>(st + row * kPayRow + cb * 16);
                            const unsigned short sc =
                                reinterpret_cast<const unsigned short*>(st + kTR * kPayRow + row * kScRow)[cb];
                            const int isum = block_isum(wv, alo, ahi, __float_as_int(dc.y));
                            // float(isum) exactly, without the int->float unit: |isum| < 2^22
                            const float fi = __int_as_float(isum + 0x4B400000) - 12582912.0f;
                            o2 = make_float2(half_bits_to_float(sc) * dc.x, fi);
                        }
                        __syncwarp();
                        if (lane == 0) tc::mbar_arrive(empty0 + 8 * s);
                    } else {
                        *cta_abort = 1;
                    }
                    terms[((it & 1) * kTR + row) * kTT + cb] = o2;
                    bar_named(kBarHand, kWork);  // terms of `it` complete; the chain of it-1 is done
                }
            }
        } else {
            // chain warp: lane = row of the tile
            float sum = 0.0f;
            for (int t = q.t0; t < q.T; t += G) {
                for (int c = 0; c < q.nch; ++c, ++it) {
                    bar_named(kBarHand, kWork);
                    if (lane < kTR) {
                        const float2* tr = terms + ((it & 1) * kTR + lane) * kTT;
                        const int n = min(kTC, w.nb - c * kTC);
                        if (n == kTC) {
#pragma unroll
                            for (int j = 0; j < kTC; j += 2) {
                                const float4 v = *reinterpret_cast<const float4*>(tr + j);
                                sum = fmaf(v.x, v.y, sum);
                                sum = fmaf(v.z, v.w, sum);
                            }
                        } else {
                            for (int j = 0; j < n; ++j) sum = fmaf(tr[j].x, tr[j].y, sum);
                        }
                    }
                    if (c == q.nch - 1) {
                        const int r = t * kTR + lane;
                        if (!*cta_abort) {
                            if (epi == 2) {  // (gate_i, up_i) pairs: ff_i = g/(1+exp(-g)) * u
                                const float u = __shfl_down_sync(0xffffffffu, sum, 1);
                                if (lane < kTR && (lane & 1) == 0 && r + 1 < w.rows)
                                    y[r / 2] = (sum / (1.0f + expf_cr(-sum))) * u;
                            } else if (lane < kTR && r < w.rows) {
                                y[r] = epi == 1 ? __ldcg(y + r) + sum : sum;
                            }
                        }
                        sum = 0.0f;
                    }
                }
            }
        }
    };

    NormPre np;
    for (int l = 0; l < a.n_layer; ++l) {
        const MkLayer& L = a.layers[l];
        // the cached K/V of this CTA's head (tokens of earlier steps) are
        // requested first: they load while the q|k|v phase runs
        Attn<HD, VS> at(a, L, sm, P, cta);
        const bool attn_here = attn_cta && tid < HD && !*cta_abort;
        if (attn_here) at.prefetch();
        // ---- q|k|v (x is complete: the embedding kernel, or layer l-1's down phase)
        norm_fetch(np, L.attn_norm, L.w[0].nb);
        if (l > 0) grid_sync(a, ++nbar, cta_abort);
        if (!*cta_abort) prologue(a.x, &np, a.eps, L.w[0].nb, act, red);
        gemv(L.w[0], 0, a.qkv);
        // ---- attention
        grid_sync(a, ++nbar, cta_abort);
        if (attn_here) {
            if (!*cta_abort) at.run(redf, redd);
            else cp_async_wait<0>();
        }
        // ---- o: att -> x += o rows
        grid_sync(a, ++nbar, cta_abort);
        if (!*cta_abort) prologue(a.att, nullptr, a.eps, L.w[1].nb, act, red);
        gemv(L.w[1], 1, a.x);
        // ---- gate|up: x -> ff
        norm_fetch(np, L.ffn_norm, L.w[2].nb);
        grid_sync(a, ++nbar, cta_abort);
        if (!*cta_abort) prologue(a.x, &np, a.eps, L.w[2].nb, act, red);
        gemv(L.w[2], 2, a.ff);
        // ---- down: ff -> x += down rows
        grid_sync(a, ++nbar, cta_abort);
        if (!*cta_abort) prologue(a.ff, nullptr, a.eps, L.w[3].nb, act, red);
        gemv(L.w[3], 1, a.x);
    }
}

}  // namespace

namespace {
using MkKernel = void (*)(const MkArgs);

MkKernel mk_kernel(int hd, int kv_type) {
    const bool v5 = mk_vstages(hd, kv_type) == 5;
    switch (hd) {
        case 64: return v5 ? decode_mk_kernel<64, 5> : decode_mk_kernel<64, 4>;
        case 128: return v5 ? decode_mk_kernel<128, 5> : decode_mk_kernel<128, 4>;
        case 256: return v5 ? decode_mk_kernel<256, 5> : decode_mk_kernel<256, 4>;
        default: return nullptr;
    }
}

// The kernel's dynamic shared-memory limit raised to the device maximum
// (less its static shared memory) and the carveout set to all-shared, once
// per (kernel, device); *smem_max = that limit.
cudaError_t prepare(MkKernel k, int* smem_max) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    cudaFuncAttributes fa{};
    e = cudaFuncGetAttributes(&fa, k);
    if (e != cudaSuccess) return e;
    *smem_max -= (int)fa.sharedSizeBytes;
    static std::mutex mu;
    static std::set<std::pair<const void*, int>> done;
    std::lock_guard<std::mutex> lock(mu);
    const std::pair<const void*, int> key{reinterpret_cast<const void*>(k), dev};
    if (done.count(key)) return cudaSuccess;
    e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, *smem_max);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e == cudaSuccess) done.insert(key);
    return e;
}
}  // namespace

bool decode_mk_supported(int hd, int kv_type, int max_ctx, int max_pages, uint64_t max_nb, uint64_t norm_cols,
                         int* stages, std::string* why) {
    auto no = [&](const std::string& r) {
        if (why) *why = r;
        return false;
    };
    if (kv_type != 0 && kv_type != 1) return no("KV cache type is not F32/F16");
    if (max_nb > (uint64_t)kMaxNb) return no("a weight is wider than " + std::to_string(kMaxNb * 32));
    if (norm_cols > (uint64_t)kNormKeep * 8 * kWork) return no("n_embd above " + std::to_string(kNormKeep * 8 * kWork));
    const MkKernel k = mk_kernel(hd, kv_type);
    if (!k) return no("head_dim not 64/128/256");
    int smem_max = 0;
    cudaError_t e = prepare(k, &smem_max);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return no(std::string("kernel attributes: ") + cudaGetErrorString(e));
    }
    // the deepest ring with which one CTA still fits on an SM (the launch is
    // cooperative: every CTA must be resident)
    for (int st = 32; st >= 4; --st) {
        const size_t smem = mk_plan(hd, max_ctx, max_pages, kv_type, st).total;
        if (smem > (size_t)smem_max) continue;
        int blocks = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, k, kThreads, smem);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return no(std::string("occupancy query: ") + cudaGetErrorString(e));
        }
        if (blocks >= 1) {
            *stages = st;
            return true;
        }
    }
    return no("no ring depth fits one CTA per SM (shared memory " + std::to_string(smem_max) + ", fixed part " +
              std::to_string(mk_plan(hd, max_ctx, max_pages, kv_type, 0).total) + ")");
}

uint64_t decode_mk_smem(const MkArgs& a) { return mk_plan(a.hd, a.max_ctx, a.max_pages, a.kv_type, a.stages).total; }

cudaError_t decode_mk(const MkArgs& a, cudaStream_t s) {
    const MkKernel k = mk_kernel(a.hd, a.kv_type);
    if (!k) return cudaErrorInvalidValue;
    int smem_max = 0;
    cudaError_t e = prepare(k, &smem_max);
    if (e != cudaSuccess) return e;
    const size_t smem = decode_mk_smem(a);
    if (smem > (size_t)smem_max) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)num_sms());
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaMemsetAsync(a.bar, 0, sizeof(unsigned), s);
    if (e != cudaSuccess) return e;
    return cudaLaunchKernelEx(&cfg, k, a);
}

}  // namespace mvb
