// attention.cu -- paged KV cache append and one-query (decode) attention.
//
// Cache layout (device): K and V each hold n_pages * page token rows; a row
// is kv_dim elements of the cache type (F32 / F16 / int8) and, for the Q8
// types, scales in a separate float array (1 per row for MV_KV_Q8, kv_dim/32
// for MV_KV_Q8_0).  Token t of sequence s lives in page
// block_table[s*max_pages + t/page] at slot t%page.
//
// Reference: PagedKVCache::write / dot_key / add_value
// (src/llama_model.cpp:22-55) and the decode loop (:256).  The reference
// keeps one sequence with an implicit identity page table; the block table
// generalises it to many sequences with scattered pages.
#include "common.cuh"
#include "kernels.cuh"
#include "tp.cuh"

namespace mvb {

uint64_t kv_row_bytes(int kv_type, uint64_t kv_dim) {
    return kv_type == 0 ? kv_dim * 4 : kv_type == 1 ? kv_dim * 2 : kv_dim;
}
uint64_t kv_row_scales(int kv_type, uint64_t kv_dim) { return kv_type == 2 ? 1 : kv_type == 3 ? kv_dim / 32 : 0; }

// ---------------------------------------------------------------- append
// One CTA per (token row, K|V).  F16 uses the reference's fp32_to_fp16; Q8
// takes one scale per token row, s = max|v|/127 (1 if zero), q =
// clamp(round-half-away(v / s)) -- a true division, as the reference writes
// it; Q8_0 applies the activation quantiser per 32-element block.
__global__ void kv_append_kernel(int kv_type, const float* __restrict__ k, const float* __restrict__ v, int kv_dim,
                                 const int32_t* __restrict__ seq, const int32_t* __restrict__ pos,
                                 const int32_t* __restrict__ block_table, int max_pages, int page,
                                 uint8_t* __restrict__ k_pages, uint8_t* __restrict__ v_pages,
                                 float* __restrict__ k_scales, float* __restrict__ v_scales) {
    const int r = blockIdx.x, which = blockIdx.y;
    const float* src = (which ? v : k) + (size_t)r * kv_dim;
    uint8_t* pages = which ? v_pages : k_pages;
    float* scales = which ? v_scales : k_scales;
    const int s = seq ? seq[r] : 0, p = pos[r];
    const size_t slot = (size_t)block_table[(size_t)s * max_pages + p / page] * page + p % page;
    if (kv_type == 0) {
        float* dst = reinterpret_cast<float*>(pages) + slot * kv_dim;
        for (int i = threadIdx.x; i < kv_dim; i += blockDim.x) dst[i] = src[i];
    } else if (kv_type == 1) {
        uint16_t* dst = reinterpret_cast<uint16_t*>(pages) + slot * kv_dim;
        for (int i = threadIdx.x; i < kv_dim; i += blockDim.x) dst[i] = f32_to_f16_ref(src[i]);
    } else if (kv_type == 2) {
        __shared__ float red[32];
        float m = 0.0f;
        for (int i = threadIdx.x; i < kv_dim; i += blockDim.x) m = fmaxf(m, fabsf(src[i]));
        m = warp_max(m);
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
        if (lane == 0) red[warp] = m;
        __syncthreads();
        if (warp == 0) {
            float t = lane < nw ? red[lane] : 0.0f;
            t = warp_max(t);
            if (lane == 0) red[0] = t;
        }
        __syncthreads();
        m = red[0];
        const float sc = m > 0.0f ? m / 127.0f : 1.0f;
        int8_t* dst = reinterpret_cast<int8_t*>(pages) + slot * kv_dim;
        for (int i = threadIdx.x; i < kv_dim; i += blockDim.x) {
            float q = roundf(src[i] / sc);
            q = fminf(fmaxf(q, -127.0f), 127.0f);
            dst[i] = (int8_t)(int)q;
        }
        if (threadIdx.x == 0) scales[slot] = sc;
    } else {
        int8_t* dst = reinterpret_cast<int8_t*>(pages) + slot * kv_dim;
        const int lane = threadIdx.x & 31;
        for (int b = threadIdx.x >> 5; b < kv_dim / 32; b += blockDim.x >> 5) {
            float dd;
            dst[b * 32 + lane] = (int8_t)quant_q8_lane(src[b * 32 + lane], dd);
            if (lane == 0) scales[slot * (kv_dim / 32) + b] = dd;
        }
    }
}

cudaError_t kv_append(int kv_type, const float* k, const float* v, uint64_t rows, uint64_t kv_dim,
                      const int32_t* seq, const int32_t* pos, const int32_t* block_table, uint64_t max_pages,
                      uint64_t page, void* k_pages, void* v_pages, float* k_scales, float* v_scales,
                      cudaStream_t s) {
    if (!rows) return cudaSuccess;
    kv_append_kernel<<<dim3((unsigned)rows, 2), 256, 0, s>>>(
        kv_type, k, v, (int)kv_dim, seq, pos, block_table, (int)max_pages, (int)page,
        static_cast<uint8_t*>(k_pages), static_cast<uint8_t*>(v_pages), k_scales, v_scales);
    return cudaGetLastError();
}

// ------------------------------------------------------- decode attention
// One CTA per (query row, query head), hd threads.  The reference's own
// evaluation order, so the output matches it bit for bit up to the host
// libm's expf (here a correctly rounded exp):
//
//  1. s_t = dot(q, k_t) / sqrt(hd) for every cached token, one thread per
//     token, with the reference's 8 FMA lanes (lane l takes dimensions
//     l, l+8, ...) summed t0+t1+...+t7 (src/llama_model.cpp:23-39;
//     Q8: times the token's K scale);
//  2. m = max s_t; e_t = exp(s_t - m); den = sum of e_t in double;
//     alpha_t = e_t * float(1/den) (src/llama_model.cpp:256);
//  3. thread d owns output dimension d: out_d = fma(alpha_t, v_t[d], out_d)
//     sequentially over t (Q8: alpha_t * v_scale first) -- the FMA chain of
//     PagedKVCache::add_value (src/llama_model.cpp:40-55).
// GQA: query head h reads kv head h / (n_head / n_head_kv).
constexpr int kVTile = 32;    // tokens per V tile
constexpr int kVStages = 4;

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

// Tokens per K tile: one per thread, at most 64, and two tiles of padded
// rows within 128 KB (64-token tiles keep a CTA near 38 KB for hd 128 F16,
// five per SM: these kernels are latency-bound, resident warps count).
__host__ __device__ constexpr int attn_ktile(uint64_t hd, int kv_type) {
    const uint64_t esize = kv_type == 0 ? 4 : kv_type == 1 ? 2 : 1;
    uint64_t kt = 65536 / (hd * esize + 16);
    if (kt > hd) kt = hd;
    if (kt > 64) kt = 64;
    return (int)(kt / 32 * 32);
}

// Shared-memory plan of one CTA (all offsets 16-byte aligned).
struct AttnSmem {
    uint64_t q, table, sc, vsc, ring, total;
};
__host__ __device__ inline AttnSmem attn_plan(uint64_t hd, uint64_t max_ctx, uint64_t max_pages, int kv_type) {
    auto up = [](uint64_t n) { return (n + 15) / 16 * 16; };
    const uint64_t esize = kv_type == 0 ? 4 : kv_type == 1 ? 2 : 1;
    const uint64_t krow = hd * esize + 16;                          // padded K row
    const uint64_t kring = 2 * (uint64_t)attn_ktile(hd, kv_type) * krow;  // double-buffered K tiles
    const uint64_t vring = (uint64_t)kVStages * kVTile * hd * esize; // V stages
    const uint64_t nsc = kv_type == 2 ? 1 : kv_type == 3 ? hd / 32 : 0;  // V scales per token
    AttnSmem p;
    p.q = 0;
    p.table = up(hd * 4);
    p.sc = p.table + up(max_pages * 4);
    p.vsc = p.sc + up(max_ctx * 4);
    p.ring = p.vsc + up(max_ctx * nsc * 4);
    p.total = p.ring + (kring > vring ? kring : vring);
    return p;
}

template <int HD>
__global__ void __launch_bounds__(HD) attn_exact_kernel(AttnArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ float redf[HD / 32];
    __shared__ double redd[HD / 32];
    const int s = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int G = (int)(a.n_head / a.n_head_kv), kh = h / G;
    const int kv_dim = (int)(a.n_head_kv * HD);
    const int kvt = a.kv_type;
    const int esize = kvt == 0 ? 4 : kvt == 1 ? 2 : 1;
    const int page = (int)a.page;
    const AttnSmem P = attn_plan(HD, a.max_ctx, a.max_pages, kvt);
    float* qs = reinterpret_cast<float*>(smem + P.q);
    int* tbl = reinterpret_cast<int*>(smem + P.table);
    float* sc = reinterpret_cast<float*>(smem + P.sc);
    float* vsc = reinterpret_cast<float*>(smem + P.vsc);
    uint8_t* ring = smem + P.ring;
    const uint8_t* kp = static_cast<const uint8_t*>(a.k_pages);
    const uint8_t* vp = static_cast<const uint8_t*>(a.v_pages);
    const size_t row_bytes = (size_t)kv_dim * esize;
    const size_t head_off = (size_t)kh * HD * esize;
    const int slice = HD * esize;  // bytes of one token's head slice

    pdl_trigger();
    pdl_wait();
    const int ctx = a.ctx_len[s];
    const int npg = (ctx + page - 1) / page;
    const size_t trow = a.one_seq ? 0 : (size_t)s;
    for (int i = tid; i < npg; i += HD) tbl[i] = a.block_table[trow * a.max_pages + i];
    qs[tid] = a.q[(size_t)s * a.q_stride + (size_t)h * HD + tid];
    __syncthreads();
    auto slot_of = [&](int t) -> size_t { return (size_t)tbl[t / page] * page + t % page; };

    // 1. scores: thread t of a K tile owns one token; its head slice is staged
    //    by cp.async into its own (padded) shared row, two tiles in flight.
    {
        const int krow = slice + 16;
        const int KT = attn_ktile(HD, kvt);  // threads tid < KT own one token of each tile
        auto issue_k = [&](int tile, int buf) {
            const int t = tile * KT + tid;
            if (tid < KT && t < ctx) {
                const uint8_t* src = kp + slot_of(t) * row_bytes + head_off;
                uint8_t* dst = ring + ((size_t)buf * KT + tid) * krow;
                for (int c = 0; c < slice; c += 16) cp_async16(dst + c, src + c);
            }
            cp_async_commit();
        };
        const int ntile = (ctx + KT - 1) / KT;
        issue_k(0, 0);
        for (int tile = 0; tile < ntile; ++tile) {
            if (tile + 1 < ntile) issue_k(tile + 1, (tile + 1) & 1);
            else cp_async_commit();
            cp_async_wait<1>();  // own row of this tile has landed
            const int t = tile * KT + tid;
            if (tid < KT && t < ctx) {
                const uint8_t* row = ring + ((size_t)(tile & 1) * KT + tid) * krow;
                float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                if (kvt == 1) {
#pragma unroll 4
                    for (int d = 0; d < HD; d += 8) {
                        const uint4 w = *reinterpret_cast<const uint4*>(row + d * 2);
                        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                        for (int l = 0; l < 8; ++l)
                            acc[l] = fmaf(qs[d + l], half_bits_to_float((unsigned short)(ws[l / 2] >> (16 * (l & 1)))),
                                          acc[l]);
                    }
                } else if (kvt == 0) {
#pragma unroll 4
                    for (int d = 0; d < HD; d += 8) {
                        const float4 u = *reinterpret_cast<const float4*>(row + d * 4);
                        const float4 v = *reinterpret_cast<const float4*>(row + d * 4 + 16);
                        const float ks[8] = {u.x, u.y, u.z, u.w, v.x, v.y, v.z, v.w};
#pragma unroll
                        for (int l = 0; l < 8; ++l) acc[l] = fmaf(qs[d + l], ks[l], acc[l]);
                    }
                } else {
                    const size_t slot = slot_of(t);
#pragma unroll 4
                    for (int d = 0; d < HD; d += 8) {
                        const uint2 w = *reinterpret_cast<const uint2*>(row + d);
                        float sc8 = 1.0f;
                        if (kvt == 3) sc8 = a.k_scales[slot * (kv_dim / 32) + (kh * HD + d) / 32];
#pragma unroll
                        for (int l = 0; l < 8; ++l)
                            acc[l] = fmaf(qs[d + l], s8_to_f32(l < 4 ? w.x : w.y, l & 3) * sc8, acc[l]);
                    }
                }
                float dot = acc[0];
#pragma unroll
                for (int l = 1; l < 8; ++l) dot += acc[l];
                if (kvt == 2) dot = dot * a.k_scales[slot_of(t)];
                sc[t] = dot / sqrtf((float)HD);
            }
        }
        cp_async_wait<0>();
    }
    // per-token V scales (Q8 types), gathered while the softmax runs
    if (kvt == 2) {
        for (int t = tid; t < ctx; t += HD) vsc[t] = a.v_scales[slot_of(t)];
    } else if (kvt == 3) {
        for (int i = tid; i < ctx * (HD / 32); i += HD) {
            const int t = i / (HD / 32), b = i % (HD / 32);
            vsc[i] = a.v_scales[slot_of(t) * (kv_dim / 32) + kh * (HD / 32) + b];
        }
    }
    __syncthreads();  // every K tile is consumed: the ring is free for V

    // 2. max, exp, double denominator, weights
    float m = -INFINITY;
    for (int t = tid; t < ctx; t += HD) m = fmaxf(m, sc[t]);
    m = warp_max(m);
    if (lane == 0) redf[warp] = m;
    __syncthreads();
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
    __syncthreads();
    den = 0.0;
#pragma unroll
    for (int w = 0; w < HD / 32; ++w) den += redd[w];
    const float inv = (float)(1.0 / den);

    // 3. thread d: out_d = fma(alpha_t, v_t[d], out_d) over t in order; V
    //    tiles of kVTile tokens staged by all threads through a kVStages ring.
    const int chunks = kVTile * slice / 16;  // 16-byte copies per tile
    const int ntile = (ctx + kVTile - 1) / kVTile;
    auto issue_v = [&](int tile) {
        if (tile < ntile) {
            uint8_t* dst = ring + (size_t)(tile % kVStages) * kVTile * slice;
            for (int c = tid; c < chunks; c += HD) {
                const int tt = c / (slice / 16), off = (c % (slice / 16)) * 16;
                const int t = tile * kVTile + tt;
                if (t < ctx) cp_async16(dst + tt * slice + off, vp + slot_of(t) * row_bytes + head_off + off);
            }
        }
        cp_async_commit();
    };
    for (int k = 0; k < kVStages - 1; ++k) issue_v(k);
    float out = 0.0f;
    for (int tile = 0; tile < ntile; ++tile) {
        cp_async_wait<kVStages - 2>();
        __syncthreads();  // the tile is visible to every thread
        const uint8_t* vt = ring + (size_t)(tile % kVStages) * kVTile * slice;
        const int n = min(kVTile, ctx - tile * kVTile);
        // alpha_t = e_t * float(1/den) (times the V scale for Q8); the loads
        // of 8 tokens go out before their 8 chain steps
        auto step = [&](int tt, float& v, float& al) {
            const int t = tile * kVTile + tt;
            al = sc[t] * inv;
            if (kvt == 1) v = half_bits_to_float(reinterpret_cast<const uint16_t*>(vt + tt * slice)[tid]);
            else if (kvt == 0) v = reinterpret_cast<const float*>(vt + tt * slice)[tid];
            else {
                v = (float)reinterpret_cast<const int8_t*>(vt + tt * slice)[tid];
                al = al * (kvt == 2 ? vsc[t] : vsc[t * (HD / 32) + tid / 32]);
            }
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
        __syncthreads();  // everyone is done with this stage before it is refilled
        issue_v(tile + kVStages - 1);
    }
    cp_async_wait<0>();
    a.out[((size_t)s * a.n_head + h) * HD + tid] = out;
}

// ------------------------------------------ prefill attention (query groups)
// The prefill form of attn_exact_kernel: QG consecutive query rows of ONE
// sequence (they share the block-table row of the group's first query) and one
// query head per CTA, hd threads (with one_seq every row reads block-table
// row 0).  Every K tile and V tile is staged once and
// used by all QG queries (a prefill chunk's queries attend to the same cached
// tokens), and the V loop carries QG independent FMA chains per thread.  Each
// query keeps attn_exact_kernel's evaluation order exactly -- the same 8-lane
// dot per token, the same per-thread strided max / double sums combined warp
// by warp, alpha_t = e_t * float(1/den), the same per-dimension FMA chain over
// its own tokens in order -- so the outputs are identical to it bit for bit.
// Query q of the group sees tokens t < ctx_len[s0 + q] (causal prefill).
// One K tile and two V stages, the block table read through L1 (37,888 bytes
// for hd 128, F16, 8 queries over 512 tokens: six CTAs per SM)
constexpr int kGroupVStages = 2;
struct AttnGroupSmem {
    uint64_t q, sc, vsc, ring, total;
};
__host__ __device__ inline AttnGroupSmem attn_group_plan(uint64_t hd, uint64_t max_ctx, uint64_t max_pages,
                                                         int kv_type, int qg) {
    auto up = [](uint64_t n) { return (n + 15) / 16 * 16; };
    const uint64_t esize = kv_type == 0 ? 4 : kv_type == 1 ? 2 : 1;
    const uint64_t krow = hd * esize + 16;
    const uint64_t kring = (uint64_t)attn_ktile(hd, kv_type) * krow;  // one K tile
    const uint64_t vring = (uint64_t)kGroupVStages * kVTile * hd * esize;
    const uint64_t nsc = kv_type == 2 ? 1 : kv_type == 3 ? hd / 32 : 0;
    AttnGroupSmem p;
    p.q = 0;
    p.sc = up((uint64_t)qg * hd * 4);
    p.vsc = p.sc + up((uint64_t)qg * max_ctx * 4);
    p.ring = p.vsc + up(max_ctx * nsc * 4);
    p.total = p.ring + (kring > vring ? kring : vring);
    return p;
}

// Page of token t by a multiply: t / page = umulhi(t, ceil(2^32 / page)) is
// exact while t * page < 2^32 (paged_attn_prefill checks max_ctx * page).
struct PageDiv {
    uint32_t page, mul;
    __device__ explicit PageDiv(uint64_t p) : page((uint32_t)p), mul((uint32_t)((0x100000000ull + p - 1) / p)) {}
    __device__ __forceinline__ uint32_t index(uint32_t t) const { return page == 1 ? t : __umulhi(t, mul); }
};

// Two fp32 values in one 64-bit register pair (element 0 in the low half) and
// fma.rn.f32x2: two IEEE round-to-nearest FMAs, each bit-identical to fmaf.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
// The QG weights of one token (token-major rows, 8-byte aligned for QG = 2,
// 16-byte aligned from QG = 4) as QG/2 pairs of queries (2p, 2p+1).
template <int QG>
__device__ __forceinline__ void ld_pairs(const float* p, uint64_t (&w)[QG / 2]) {
    if constexpr (QG == 2) {
        w[0] = *reinterpret_cast<const uint64_t*>(p);
    } else {
#pragma unroll
        for (int k = 0; k < QG / 4; ++k) {
            const ulonglong2 u = reinterpret_cast<const ulonglong2*>(p)[k];
            w[2 * k] = u.x;
            w[2 * k + 1] = u.y;
        }
    }
}
template <int QG>
__device__ __forceinline__ void ld_row(const float* p, float (&w)[QG]) {
#pragma unroll
    for (int k = 0; k < QG / 2; ++k) {
        const float2 u = reinterpret_cast<const float2*>(p)[k];
        w[2 * k] = u.x;
        w[2 * k + 1] = u.y;
    }
}
template <int QG>
__device__ __forceinline__ void st_row(float* p, const float (&w)[QG]) {
    if constexpr (QG == 2) {
        *reinterpret_cast<float2*>(p) = make_float2(w[0], w[1]);
    } else {
#pragma unroll
        for (int k = 0; k < QG / 4; ++k)
            reinterpret_cast<float4*>(p)[k] = make_float4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
    }
}

template <int HD, int QG, int KVT>
__global__ void __launch_bounds__(HD) attn_group_kernel(AttnArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    constexpr int kEs = KVT == 0 ? 4 : KVT == 1 ? 2 : 1;
    constexpr int kSlice = HD * kEs;  // bytes of one head's K or V row
    constexpr int kKT = attn_ktile(HD, KVT);
    // blockIdx.x is the query head; blockIdx.y counts groups from the last, so
    // the groups with the longest causal context are dispatched first
    const int grp = (int)(gridDim.y - 1 - blockIdx.y);
    const int s0 = grp * QG, h = blockIdx.x, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int G = (int)(a.n_head / a.n_head_kv), kh = h / G;
    const int kv_dim = (int)(a.n_head_kv * HD);
    const PageDiv pdiv(a.page);
    const AttnGroupSmem P = attn_group_plan(HD, a.max_ctx, a.max_pages, KVT, QG);
    float* qs = reinterpret_cast<float*>(smem + P.q);  // [QG][HD]
    float* sc = reinterpret_cast<float*>(smem + P.sc);  // [max_ctx][QG]: token-major
    float* vsc = reinterpret_cast<float*>(smem + P.vsc);
    uint8_t* ring = smem + P.ring;
    // the softmax's cross-warp reductions live in the ring while no K or V
    // tile is staged (between the last K tile and the first V copy)
    auto redd = reinterpret_cast<double(*)[HD / 32]>(ring);
    auto redf = reinterpret_cast<float(*)[HD / 32]>(ring + QG * (HD / 32) * sizeof(double));
    const uint8_t* kp = static_cast<const uint8_t*>(a.k_pages);
    const uint8_t* vp = static_cast<const uint8_t*>(a.v_pages);
    const size_t row_bytes = (size_t)kv_dim * kEs;
    const size_t head_off = (size_t)kh * kSlice;

    pdl_trigger();
    pdl_wait();
    int cq[QG];
    int cmax = 0, cmin = INT_MAX;
#pragma unroll
    for (int i = 0; i < QG; ++i) {
        cq[i] = s0 + i < (int)a.n_seq ? a.ctx_len[s0 + i] : 0;
        cmax = max(cmax, cq[i]);
        cmin = min(cmin, cq[i]);
    }
    const int32_t* tbl = a.block_table + (a.one_seq ? 0 : (size_t)s0) * a.max_pages;
#pragma unroll
    for (int i = 0; i < QG; ++i)
        qs[i * HD + tid] = cq[i] > 0 ? a.q[(size_t)(s0 + i) * a.q_stride + (size_t)h * HD + tid] : 0.0f;
    __syncthreads();
    auto slot_of = [&](int t) -> size_t {
        const uint32_t pi = pdiv.index((uint32_t)t);
        return (size_t)__ldg(tbl + pi) * pdiv.page + ((uint32_t)t - pi * pdiv.page);
    };

    // 1. raw dot products of every query with tokens 0..cmax-1: a K tile's rows
    // are copied by thread t (token t of the tile) and scored by a pair of lanes
    {
        constexpr int kRow = kSlice + 16;
        auto issue_k = [&](int tile, int buf) {
            const int t = tile * kKT + tid;
            if (tid < kKT && t < cmax) {
                const uint8_t* src = kp + slot_of(t) * row_bytes + head_off;
                uint8_t* dst = ring + ((size_t)buf * kKT + tid) * kRow;
#pragma unroll
                for (int c = 0; c < kSlice; c += 16) cp_async16(dst + c, src + c);
            }
            cp_async_commit();
        };
        const int ntile = (cmax + kKT - 1) / kKT;
        for (int tile = 0; tile < ntile; ++tile) {
            if (tile) __syncthreads();  // tile-1's rows are no longer read
            issue_k(tile, 0);
            cp_async_wait<0>();  // this thread's copies of the tile have landed
            __syncthreads();     // ... every thread's
            // a pair of lanes per token: the even lane accumulates the reference's
            // lanes 0..3 (elements d..d+3 of every 8), the odd lane lanes 4..7,
            // as two packed pairs (lanes 0,1 and 2,3); the odd lane's four sums
            // then join the even lane's in lane order
            const int half = lane & 1;
            for (int tk = warp * 16 + (lane >> 1); tk < kKT; tk += (HD / 32) * 16) {  // warp-uniform trips
                const int t = tile * kKT + tk;
                const bool valid = t < cmax;
                const uint8_t* row = ring + (size_t)tk * kRow + 4 * half * kEs;
                const float* qh = qs + 4 * half;
                uint64_t acc[QG][2];
#pragma unroll
                for (int i = 0; i < QG; ++i) acc[i][0] = acc[i][1] = 0ull;  // +0.0f, +0.0f
                const size_t slot = KVT >= 2 && valid ? slot_of(t) : 0;
                if (valid) {
#pragma unroll
                    for (int d = 0; d < HD; d += 8) {
                        uint64_t k01, k23;
                        if constexpr (KVT == 1) {
                            const uint2 w = *reinterpret_cast<const uint2*>(row + d * 2);
                            k01 = f2_pack(half_bits_to_float((unsigned short)(w.x & 0xffff)),
                                          half_bits_to_float((unsigned short)(w.x >> 16)));
                            k23 = f2_pack(half_bits_to_float((unsigned short)(w.y & 0xffff)),
                                          half_bits_to_float((unsigned short)(w.y >> 16)));
                        } else if constexpr (KVT == 0) {
                            const ulonglong2 u = *reinterpret_cast<const ulonglong2*>(row + d * 4);
                            k01 = u.x, k23 = u.y;
                        } else {
                            const uint32_t w = *reinterpret_cast<const uint32_t*>(row + d);
                            const float sc8 = KVT == 3 ? a.k_scales[slot * (kv_dim / 32) + (kh * HD + d) / 32] : 1.0f;
                            k01 = f2_pack(s8_to_f32(w, 0) * sc8, s8_to_f32(w, 1) * sc8);
                            k23 = f2_pack(s8_to_f32(w, 2) * sc8, s8_to_f32(w, 3) * sc8);
                        }
#pragma unroll
                        for (int i = 0; i < QG; ++i) {
                            const ulonglong2 qv = *reinterpret_cast<const ulonglong2*>(qh + i * HD + d);
                            acc[i][0] = f2_fma(qv.x, k01, acc[i][0]);
                            acc[i][1] = f2_fma(qv.y, k23, acc[i][1]);
                        }
                    }
                }
                const float ksc = KVT == 2 && valid ? a.k_scales[slot] : 1.0f;
                float dots[QG];
#pragma unroll
                for (int i = 0; i < QG; ++i) {
                    const float2 a01 = f2_unpack(acc[i][0]), a23 = f2_unpack(acc[i][1]);
                    const float hi0 = __shfl_xor_sync(0xffffffffu, a01.x, 1);
                    const float hi1 = __shfl_xor_sync(0xffffffffu, a01.y, 1);
                    const float hi2 = __shfl_xor_sync(0xffffffffu, a23.x, 1);
                    const float hi3 = __shfl_xor_sync(0xffffffffu, a23.y, 1);
                    float dot = a01.x;
                    dot += a01.y;
                    dot += a23.x;
                    dot += a23.y;
                    dot += hi0;
                    dot += hi1;
                    dot += hi2;
                    dot += hi3;
                    if (KVT == 2) dot = dot * ksc;
                    dots[i] = dot;  // divided by sqrt(hd) in the max pass below
                }
                if (valid && half == 0) st_row<QG>(sc + (size_t)t * QG, dots);
            }
        }
        cp_async_wait<0>();
    }
    if constexpr (KVT == 2) {
        for (int t = tid; t < cmax; t += HD) vsc[t] = a.v_scales[slot_of(t)];
    } else if constexpr (KVT == 3) {
        for (int i = tid; i < cmax * (HD / 32); i += HD) {
            const int t = i / (HD / 32), b = i % (HD / 32);
            vsc[i] = a.v_scales[slot_of(t) * (kv_dim / 32) + kh * (HD / 32) + b];
        }
    }
    __syncthreads();  // every K tile is consumed: the ring is free for V

    // 2. per query: s_t = dot_t / sqrt(hd), max, exp, double denominator,
    // alpha_t = e_t * float(1/den); thread tid visits tokens tid, tid + hd, ...
    // for every query (each query's own sums in that order, as the one-query
    // kernel's)
    float m[QG];
#pragma unroll
    for (int i = 0; i < QG; ++i) m[i] = -INFINITY;
    for (int t = tid; t < cmax; t += HD) {
        float w[QG];
        ld_row<QG>(sc + (size_t)t * QG, w);
#pragma unroll
        for (int i = 0; i < QG; ++i) {
            w[i] = w[i] / sqrtf((float)HD);
            if (t < cq[i]) m[i] = fmaxf(m[i], w[i]);
        }
        st_row<QG>(sc + (size_t)t * QG, w);
    }
#pragma unroll
    for (int i = 0; i < QG; ++i) {
        const float v = warp_max(m[i]);
        if (lane == 0) redf[i][warp] = v;
    }
    __syncthreads();
    double den[QG];
#pragma unroll
    for (int i = 0; i < QG; ++i) {
        m[i] = redf[i][0];
#pragma unroll
        for (int w = 1; w < HD / 32; ++w) m[i] = fmaxf(m[i], redf[i][w]);
        den[i] = 0.0;
    }
    for (int t = tid; t < cmax; t += HD) {
        float w[QG];
        ld_row<QG>(sc + (size_t)t * QG, w);
#pragma unroll
        for (int i = 0; i < QG; ++i) {
            if (t < cq[i]) {
                w[i] = expf_cr(w[i] - m[i]);
                den[i] += (double)w[i];
            }
        }
        st_row<QG>(sc + (size_t)t * QG, w);
    }
#pragma unroll
    for (int i = 0; i < QG; ++i) {
        const double d = warp_sum_d(den[i]);
        if (lane == 0) redd[i][warp] = d;
    }
    __syncthreads();
    float inv[QG];
#pragma unroll
    for (int i = 0; i < QG; ++i) {
        double d = 0.0;
#pragma unroll
        for (int w = 0; w < HD / 32; ++w) d += redd[i][w];
        inv[i] = (float)(1.0 / d);
    }
    for (int t = tid; t < cmax; t += HD) {
        float w[QG];
        ld_row<QG>(sc + (size_t)t * QG, w);
#pragma unroll
        for (int i = 0; i < QG; ++i) w[i] = w[i] * inv[i];
        st_row<QG>(sc + (size_t)t * QG, w);
    }
    __syncthreads();  // redd is read: the ring takes V tiles

    // 3. thread d: out_q,d = fma(alpha_q,t, v_t[d], out_q,d) over t < ctx_q in
    // order, queries (2p, 2p+1) in one packed FMA
    constexpr int kChunks = kVTile * kSlice / 16;
    const int ntile = (cmax + kVTile - 1) / kVTile;
    auto issue_v = [&](int tile) {
        if (tile < ntile) {
            uint8_t* dst = ring + (size_t)(tile % kGroupVStages) * kVTile * kSlice;
#pragma unroll
            for (int c0 = 0; c0 < kChunks; c0 += HD) {
                const int c = c0 + tid;
                const int tt = c / (kSlice / 16), off = (c % (kSlice / 16)) * 16;
                const int t = tile * kVTile + tt;
                if ((kChunks % HD == 0 || c < kChunks) && t < cmax)
                    cp_async16(dst + tt * kSlice + off, vp + slot_of(t) * row_bytes + head_off + off);
            }
        }
        cp_async_commit();
    };
    issue_v(0);
    uint64_t out[QG / 2];
#pragma unroll
    for (int p = 0; p < QG / 2; ++p) out[p] = 0ull;
    for (int tile = 0; tile < ntile; ++tile) {
        cp_async_wait<0>();
        __syncthreads();    // the tile (and, first time round, every alpha) is visible, and
        issue_v(tile + 1);  // the other stage (tile - 1) is read by no one: it takes tile + 1
        const uint8_t* vt = ring + (size_t)(tile % kGroupVStages) * kVTile * kSlice;
        const int n = min(kVTile, cmax - tile * kVTile);
        auto vload = [&](int tt, float& v, float& vs) {
            const int t = tile * kVTile + tt;
            vs = 1.0f;
            if constexpr (KVT == 1) v = half_bits_to_float(reinterpret_cast<const uint16_t*>(vt + tt * kSlice)[tid]);
            else if constexpr (KVT == 0) v = reinterpret_cast<const float*>(vt + tt * kSlice)[tid];
            else {
                v = (float)reinterpret_cast<const int8_t*>(vt + tt * kSlice)[tid];
                vs = KVT == 2 ? vsc[t] : vsc[t * (HD / 32) + tid / 32];
            }
        };
        // tokens every query of the group sees, 8 at a time: all their loads
        // go out before the chain steps (each query's steps stay in token order)
        const int nall = max(0, min(n, cmin - tile * kVTile));
        const float* wt = sc + (size_t)tile * kVTile * QG;
        int tt = 0;
        for (; tt + 8 <= nall; tt += 8) {
            float v[8], vs[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) vload(tt + j, v[j], vs[j]);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                uint64_t w[QG / 2];
                ld_pairs<QG>(wt + (tt + j) * QG, w);
                const uint64_t vv = f2_pack(v[j], v[j]);
                if constexpr (KVT >= 2) {
                    const uint64_t ss = f2_pack(vs[j], vs[j]);
#pragma unroll
                    for (int p = 0; p < QG / 2; ++p) w[p] = f2_mul(w[p], ss);
                }
#pragma unroll
                for (int p = 0; p < QG / 2; ++p) out[p] = f2_fma(w[p], vv, out[p]);
            }
        }
        for (; tt < n; ++tt) {
            float v, vs;
            vload(tt, v, vs);
            const int t = tile * kVTile + tt;
            float w[QG];
            ld_row<QG>(wt + tt * QG, w);
#pragma unroll
            for (int p = 0; p < QG / 2; ++p) {
                float2 o = f2_unpack(out[p]);
                if (t < cq[2 * p]) o.x = fmaf(KVT >= 2 ? w[2 * p] * vs : w[2 * p], v, o.x);
                if (t < cq[2 * p + 1]) o.y = fmaf(KVT >= 2 ? w[2 * p + 1] * vs : w[2 * p + 1], v, o.y);
                out[p] = f2_pack(o.x, o.y);
            }
        }
    }
    cp_async_wait<0>();
    float res[QG];
#pragma unroll
    for (int p = 0; p < QG / 2; ++p) {
        const float2 o = f2_unpack(out[p]);
        res[2 * p] = o.x;
        res[2 * p + 1] = o.y;
    }
#pragma unroll
    for (int i = 0; i < QG; ++i)
        if (s0 + i < (int)a.n_seq) a.out[((size_t)(s0 + i) * a.n_head + h) * HD + tid] = res[i];
    if (a.xq) {
        // the o projection's Q8 input, as quantize_q8_t_kernel lays it out:
        // warp w holds 32-element block (h*HD + 32w)/32 of every query row
        const uint64_t D = a.n_head * HD, nb = D / 32, ldb = a.xq_ldb;
        const uint64_t blk = ((uint64_t)h * HD + 32 * warp) / 32;
        float* cT = a.xdT + nb * ldb;
#pragma unroll
        for (int i = 0; i < QG; ++i) {
            if (s0 + i < (int)a.n_seq) {  // warp-uniform
                float dd;
                const int v = quant_q8_lane(res[i], dd);
                const size_t at = (size_t)(s0 + i) * D + (size_t)h * HD + tid;
                if (a.xq_f16) reinterpret_cast<uint16_t*>(a.xq)[at] = __half_as_ushort(__int2half_rn(v));
                else a.xq[at] = (int8_t)v;
                const int sum = warp_sum_i(v);
                if (lane == 0) {
                    a.xdT[blk * ldb + s0 + i] = dd;
                    cT[blk * ldb + s0 + i] = 12582912.0f + (float)(8 * sum);
                }
            }
        }
        if (grp == 0) {  // token rows n_seq..ldb-1 of this block: zero
            for (uint64_t r = a.n_seq + lane; r < ldb; r += 32) {
                a.xdT[blk * ldb + r] = 0.0f;
                cT[blk * ldb + r] = 0.0f;
            }
        }
    }
}

// ------------------------------------------- fused decode step (F16/F32 KV)
// One decode token: RoPE of the query and key heads, the append of this
// token's K and V to the paged cache and the attention above, in one kernel
// (grid n_head, hd threads).  The math is that of rope_append_heads_kernel
// followed by attn_exact_kernel:
//   * q and k rotate by the reference's half-split RoPE (fma(x0,c,-(x1*s)),
//     fma(x0,s,x1*c)); the cache stores k and v as the reference's KV cache
//     does (fp32, or fp16 rounded half-up), and this token's score and value
//     use those stored values;
//   * the cached tokens 0..p-1 are scored tile by tile as before, this token
//     (t = p, last in order) after them; its value is the last FMA of every
//     output chain -- the reference's order.
// Before waiting on the previous kernel (the q|k|v GEMV) it only reads what
// earlier decode steps wrote -- the position, the block table, the cached
// K/V rows of tokens 0..p-1 -- so the first K tile and the first V tiles are
// in flight while the GEMV finishes.  One CTA per kv head (h % group == 0)
// writes the cache rows of this token.
struct FusedSmem {
    uint64_t q, table, sc, knew, vnew, kring, vring, total;
};
// Sizes of the decode kernel's K and V staging.  The kernel follows the
// q|k|v GEMV, whose CTAs fill the SMs: the GEMV leaves one CTA slot free on
// some SMs (GemvQ4Args::reserve) and the attention is kept small enough to
// start there early (K tiles of 64 tokens, a 5-tile V ring: ~78 KB for hd 128
// F16) and issue its cached K/V loads while the GEMV still runs -- measured
// faster than a deeper ring that has to wait for two GEMV CTAs to leave.
__host__ __device__ inline int fused_ktile(uint64_t hd, int kv_type) {
    const int kt = attn_ktile(hd, kv_type);
    return kt < 64 ? kt : 64;
}
__host__ __device__ inline int fused_vstages(uint64_t hd, int kv_type) {
    return hd * (kv_type == 0 ? 4 : 2) <= 256 ? 5 : 4;
}
__host__ __device__ inline FusedSmem fused_plan(uint64_t hd, uint64_t max_ctx, uint64_t max_pages, int kv_type) {
    auto up = [](uint64_t n) { return (n + 15) / 16 * 16; };
    const uint64_t esize = kv_type == 0 ? 4 : 2;
    const uint64_t krow = hd * esize + 16;
    FusedSmem p;
    p.q = 0;
    p.table = up(hd * 4);
    p.sc = p.table + up(max_pages * 4);
    p.knew = p.sc + up(max_ctx * 4);
    p.vnew = p.knew + up(hd * esize);
    p.kring = p.vnew + up(hd * esize);
    p.vring = p.kring + 2 * (uint64_t)fused_ktile(hd, kv_type) * krow;
    p.total = p.vring + (uint64_t)fused_vstages(hd, kv_type) * kVTile * hd * esize;
    return p;
}

// TP: tensor parallel, the output goes to every rank's LL buffer (a separate
// instantiation, so the one-GPU kernel carries none of it).
template <int HD, bool TP, int VS>
__global__ void __launch_bounds__(HD) attn_decode_fused_kernel(AttnFusedArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ float redf[HD / 32];
    __shared__ double redd[HD / 32];
    const int h = blockIdx.x, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int G = (int)(a.n_head / a.n_head_kv), kh = h / G;
    const int D = (int)(a.n_head * HD), kv_dim = (int)(a.n_head_kv * HD);
    const int kvt = a.kv_type, esize = kvt == 0 ? 4 : 2;
    const int page = (int)a.page, half = HD / 2;
    const FusedSmem P = fused_plan(HD, a.max_ctx, a.max_pages, kvt);
    float* qs = reinterpret_cast<float*>(smem + P.q);
    int* tbl = reinterpret_cast<int*>(smem + P.table);
    float* sc = reinterpret_cast<float*>(smem + P.sc);
    uint8_t* knew = smem + P.knew;
    uint8_t* vnew = smem + P.vnew;
    uint8_t* kring = smem + P.kring;
    uint8_t* vring = smem + P.vring;
    const uint8_t* kp = static_cast<const uint8_t*>(a.k_pages);
    const uint8_t* vp = static_cast<const uint8_t*>(a.v_pages);
    const size_t row_bytes = (size_t)kv_dim * esize;
    const size_t head_off = (size_t)kh * HD * esize;
    const int slice = HD * esize;  // bytes of one token's head slice

    pdl_trigger();
    const int p = a.pos[0];  // this token; tokens 0..p-1 are cached
    const int npg = (p + page) / page;
    for (int i = tid; i < npg; i += HD) tbl[i] = a.block_table[i];
    __syncthreads();
    auto slot_of = [&](int t) -> size_t { return (size_t)tbl[t / page] * page + t % page; };

    const int krow = slice + 16;
    const int KT = fused_ktile(HD, kvt);
    const int nkt = (p + KT - 1) / KT;
    auto issue_k = [&](int tile, int buf) {
        const int t = tile * KT + tid;
        if (tid < KT && t < p) {
            const uint8_t* src = kp + slot_of(t) * row_bytes + head_off;
            uint8_t* dst = kring + ((size_t)buf * KT + tid) * krow;
            for (int c = 0; c < slice; c += 16) cp_async16(dst + c, src + c);
        }
        cp_async_commit();
    };
    const int chunks = kVTile * slice / 16;
    const int nvt = (p + kVTile - 1) / kVTile;
    auto issue_v = [&](int tile) {
        if (tile < nvt) {
            uint8_t* dst = vring + (size_t)(tile % VS) * kVTile * slice;
            for (int c = tid; c < chunks; c += HD) {
                const int tt = c / (slice / 16), off = (c % (slice / 16)) * 16;
                const int t = tile * kVTile + tt;
                if (t < p) cp_async16(dst + tt * slice + off, vp + slot_of(t) * row_bytes + head_off + off);
            }
        }
        cp_async_commit();
    };
    // groups in flight: V tiles 0..VS-2, then K tiles 0 and 1
    for (int k = 0; k < VS - 1; ++k) issue_v(k);
    issue_k(0, 0);
    if (nkt > 1) issue_k(1, 1);
    // this token's rotation (the tables are immutable)
    float c = 0.0f, sn = 0.0f;
    if (tid < half) {
        c = a.cos_t[(size_t)p * half + tid];
        sn = a.sin_t[(size_t)p * half + tid];
    }

    pdl_wait();
    // this token: RoPE of q (head h) and k (kv head kh), k and v in cache form
    {
        const float* row = a.qkv;
        if (tid < half) {
            const float q0 = row[h * HD + tid], q1 = row[h * HD + tid + half];
            qs[tid] = __fmaf_rn(q0, c, -__fmul_rn(q1, sn));
            qs[tid + half] = __fmaf_rn(q0, sn, __fmul_rn(q1, c));
            const float k0 = row[D + kh * HD + tid], k1 = row[D + kh * HD + tid + half];
            const float r0 = __fmaf_rn(k0, c, -__fmul_rn(k1, sn)), r1 = __fmaf_rn(k0, sn, __fmul_rn(k1, c));
            if (kvt == 1) {
                reinterpret_cast<uint16_t*>(knew)[tid] = f32_to_f16_ref(r0);
                reinterpret_cast<uint16_t*>(knew)[tid + half] = f32_to_f16_ref(r1);
            } else {
                reinterpret_cast<float*>(knew)[tid] = r0;
                reinterpret_cast<float*>(knew)[tid + half] = r1;
            }
        }
        const float v = row[D + kv_dim + kh * HD + tid];
        if (kvt == 1) reinterpret_cast<uint16_t*>(vnew)[tid] = f32_to_f16_ref(v);
        else reinterpret_cast<float*>(vnew)[tid] = v;
    }
    __syncthreads();
    if (h % G == 0) {  // the cache rows of this token, once per kv head
        const size_t at = slot_of(p) * row_bytes + head_off;
        uint8_t* kd = static_cast<uint8_t*>(a.k_pages) + at;
        uint8_t* vd = static_cast<uint8_t*>(a.v_pages) + at;
        for (int i = tid; i < slice / 4; i += HD) {
            reinterpret_cast<uint32_t*>(kd)[i] = reinterpret_cast<const uint32_t*>(knew)[i];
            reinterpret_cast<uint32_t*>(vd)[i] = reinterpret_cast<const uint32_t*>(vnew)[i];
        }
    }
    if (h == 0 && tid == 0 && a.ctx_out) a.ctx_out[0] = p + 1;

    // 1. scores of the cached tokens, then this token's
    auto dot_row = [&](const uint8_t* krw) -> float {
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
    };
    // K groups: tiles 0 and 1 before the wait, tile t+1 after tile t-1 (own
    // rows: each thread reads only the rows it copied)
    for (int tile = 0; tile < nkt; ++tile) {
        if (tile >= 1 || nkt == 1) {
            if (tile >= 1 && tile + 1 < nkt) issue_k(tile + 1, (tile + 1) & 1);
            else cp_async_commit();
        }
        cp_async_wait<1>();  // own row of this tile has landed (and, before it, the V tiles)
        const int t = tile * KT + tid;
        if (tid < KT && t < p) sc[t] = dot_row(kring + ((size_t)(tile & 1) * KT + tid) * krow);
    }
    // this token's score: by a thread without a token in the last tile
    if (tid == (p % KT ? KT - 1 : 0)) sc[p] = dot_row(knew);
    __syncthreads();

    // 2. max, exp, double denominator, weights (all p + 1 tokens)
    const int ctx = p + 1;
    float m = -INFINITY;
    for (int t = tid; t < ctx; t += HD) m = fmaxf(m, sc[t]);
    m = warp_max(m);
    if (lane == 0) redf[warp] = m;
    __syncthreads();
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
    __syncthreads();
    den = 0.0;
#pragma unroll
    for (int w = 0; w < HD / 32; ++w) den += redd[w];
    const float inv = (float)(1.0 / den);

    // 3. out_d = fma(alpha_t, v_t[d], out_d) over the cached tokens in order, then this token
    float out = 0.0f;
    for (int tile = 0; tile < nvt; ++tile) {
        cp_async_wait<VS - 2>();
        __syncthreads();  // the tile is visible to every thread
        const uint8_t* vt = vring + (size_t)(tile % VS) * kVTile * slice;
        const int n = min(kVTile, p - tile * kVTile);
        auto step = [&](int tt, float& v, float& al) {
            al = sc[tile * kVTile + tt] * inv;  // alpha_t = e_t * float(1/den)
            v = kvt == 1 ? half_bits_to_float(reinterpret_cast<const uint16_t*>(vt + tt * slice)[tid])
                         : reinterpret_cast<const float*>(vt + tt * slice)[tid];
        };
        // the loads of 8 tokens go out before their 8 chain steps
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
        __syncthreads();  // everyone is done with this stage before it is refilled
        issue_v(tile + VS - 1);
    }
    cp_async_wait<0>();
    {
        const float al = sc[p] * inv;
        const float v = kvt == 1 ? half_bits_to_float(reinterpret_cast<const uint16_t*>(vnew)[tid])
                                 : reinterpret_cast<const float*>(vnew)[tid];
        out = fmaf(al, v, out);
    }
    if constexpr (TP) ll_put_all(a.tp, a.out_shared, (uint64_t)(a.head_off + h) * HD + tid, out,
                                 tp_uepoch(a.tp, a.out_point));
    else a.out[(size_t)h * HD + tid] = out;
}

uint64_t attn_fused_smem_bytes(uint64_t hd, uint64_t max_ctx, uint64_t max_pages, int kv_type) {
    return fused_plan(hd, max_ctx, max_pages, kv_type).total;
}

cudaError_t attn_decode_fused(const AttnFusedArgs& a, cudaStream_t s) {
    if (a.kv_type != 0 && a.kv_type != 1) return cudaErrorInvalidValue;
    if (a.n_head % a.n_head_kv || a.hd % 32) return cudaErrorInvalidValue;
    const size_t smem = attn_fused_smem_bytes(a.hd, a.max_ctx ? a.max_ctx : 1, a.max_pages, a.kv_type);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    const dim3 grid((unsigned)a.n_head);
    auto go = [&](auto kernel, int hd) {
        ensure_smem_attr(kernel, 200 * 1024);
        return launch_pdl(kernel, grid, dim3(hd), smem, s, a);
    };
    const bool tp = a.tp.world > 1, v5 = fused_vstages(a.hd, a.kv_type) == 5;
#define MV_FUSED(H)                                                                                  \
    (tp ? (v5 ? go(attn_decode_fused_kernel<H, true, 5>, H) : go(attn_decode_fused_kernel<H, true, 4>, H)) \
        : (v5 ? go(attn_decode_fused_kernel<H, false, 5>, H) : go(attn_decode_fused_kernel<H, false, 4>, H)))
    switch (a.hd) {
        case 64: return MV_FUSED(64);
        case 128: return MV_FUSED(128);
        case 256: return MV_FUSED(256);
        default: return cudaErrorInvalidValue;
    }
#undef MV_FUSED
}

uint64_t attn_smem_bytes(uint64_t hd, uint64_t max_ctx, uint64_t max_pages, int kv_type) {
    return attn_plan(hd, max_ctx, max_pages, kv_type).total;
}

cudaError_t paged_attn_decode(const AttnArgs& a, cudaStream_t s) {
    if (!a.n_seq) return cudaSuccess;
    if (a.n_head % a.n_head_kv) return cudaErrorInvalidValue;
    const size_t smem = attn_smem_bytes(a.hd, a.max_ctx ? a.max_ctx : 1, a.max_pages, a.kv_type);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    dim3 grid((unsigned)a.n_seq, (unsigned)a.n_head);
    switch (a.hd) {
        case 64:
            ensure_smem_attr(attn_exact_kernel<64>, 200 * 1024);
            return launch_pdl(attn_exact_kernel<64>, grid, dim3(64), smem, s, a);
        case 128:
            ensure_smem_attr(attn_exact_kernel<128>, 200 * 1024);
            return launch_pdl(attn_exact_kernel<128>, grid, dim3(128), smem, s, a);
        case 256:
            ensure_smem_attr(attn_exact_kernel<256>, 200 * 1024);
            return launch_pdl(attn_exact_kernel<256>, grid, dim3(256), smem, s, a);
        default:
            return cudaErrorInvalidValue;
    }
}

namespace {
template <int HD, int QG, int KVT>
cudaError_t launch_group(const AttnArgs& a, size_t smem, cudaStream_t s) {
    dim3 grid((unsigned)a.n_head, (unsigned)((a.n_seq + QG - 1) / QG));
    ensure_smem_attr(attn_group_kernel<HD, QG, KVT>, 200 * 1024);
    return launch_pdl(attn_group_kernel<HD, QG, KVT>, grid, dim3(HD), smem, s, a);
}
template <int HD, int QG>
cudaError_t launch_group_kv(const AttnArgs& a, size_t smem, cudaStream_t s) {
    switch (a.kv_type) {
        case 0: return launch_group<HD, QG, 0>(a, smem, s);
        case 1: return launch_group<HD, QG, 1>(a, smem, s);
        case 2: return launch_group<HD, QG, 2>(a, smem, s);
        case 3: return launch_group<HD, QG, 3>(a, smem, s);
        default: return cudaErrorInvalidValue;
    }
}
template <int QG>
cudaError_t launch_group_hd(const AttnArgs& a, size_t smem, cudaStream_t s) {
    switch (a.hd) {
        case 64: return launch_group_kv<64, QG>(a, smem, s);
        case 128: return launch_group_kv<128, QG>(a, smem, s);
        case 256: return launch_group_kv<256, QG>(a, smem, s);
        default: return cudaErrorInvalidValue;
    }
}
}  // namespace

cudaError_t paged_attn_prefill(const AttnArgs& a, cudaStream_t s) {
    if (!a.n_seq) return cudaSuccess;
    if (a.n_head % a.n_head_kv) return cudaErrorInvalidValue;
    // groups of 8 when that still gives every SM two CTAs (merged prefill
    // batches: twice the reuse of every staged K/V tile, eight independent
    // chains per thread), of 4 when it gives every SM a CTA, else pairs
    const uint64_t sms = (uint64_t)num_sms();
    // (pp512, 7B: groups of 8 12,640 tok/s against 12,350 with groups of 4)
    const int qg = (a.n_seq + 7) / 8 * a.n_head >= 2 * sms ? 8
                   : (a.n_seq + 3) / 4 * a.n_head >= sms   ? 4
                   : a.n_seq >= 2                          ? 2
                                                           : 1;
    const size_t smem = qg > 1 ? attn_group_plan(a.hd, a.max_ctx ? a.max_ctx : 1, a.max_pages, a.kv_type, qg).total : 0;
    // the group kernel finds a token's page by a 32-bit multiply (exact while
    // (max_ctx + page) * page < 2^32) and numbers its groups in grid.y
    const bool fits = (a.max_ctx + a.page) * a.page < (1ull << 32) && (a.n_seq + qg - 1) / qg <= 65535;
    if (qg == 1 || smem > 200 * 1024 || !fits) {
        cudaError_t e = paged_attn_decode(a, s);
        if (e == cudaSuccess && a.xq)
            e = quantize_q8_rows_t(a.out, a.n_seq, a.n_head * a.hd, a.xq, a.xdT, a.xq_ldb, s,
                                   a.xq_f16 ? reinterpret_cast<uint16_t*>(a.xq) : nullptr);
        return e;
    }
    if (a.xq && a.xq_ldb < a.n_seq) return cudaErrorInvalidValue;
    return qg == 8 ? launch_group_hd<8>(a, smem, s) : qg == 4 ? launch_group_hd<4>(a, smem, s)
                                                     : launch_group_hd<2>(a, smem, s);
}

}  // namespace mvb
