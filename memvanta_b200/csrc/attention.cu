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
__host__ __device__ inline int attn_ktile(uint64_t hd, int kv_type) {
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
struct AttnGroupSmem {
    uint64_t q, table, sc, vsc, ring, total;
};
__host__ __device__ inline AttnGroupSmem attn_group_plan(uint64_t hd, uint64_t max_ctx, uint64_t max_pages,
                                                         int kv_type, int qg) {
    auto up = [](uint64_t n) { return (n + 15) / 16 * 16; };
    const uint64_t esize = kv_type == 0 ? 4 : kv_type == 1 ? 2 : 1;
    const uint64_t krow = hd * esize + 16;
    const uint64_t kring = 2 * (uint64_t)attn_ktile(hd, kv_type) * krow;
    const uint64_t vring = (uint64_t)kVStages * kVTile * hd * esize;
    const uint64_t nsc = kv_type == 2 ? 1 : kv_type == 3 ? hd / 32 : 0;
    AttnGroupSmem p;
    p.q = 0;
    p.table = up((uint64_t)qg * hd * 4);
    p.sc = p.table + up(max_pages * 4);
    p.vsc = p.sc + up((uint64_t)qg * max_ctx * 4);
    p.ring = p.vsc + up(max_ctx * nsc * 4);
    p.total = p.ring + (kring > vring ? kring : vring);
    return p;
}

template <int HD, int QG>
__global__ void __launch_bounds__(HD) attn_group_kernel(AttnArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ float redf[QG][HD / 32];
    __shared__ double redd[QG][HD / 32];
    const int s0 = blockIdx.x * QG, h = blockIdx.y, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int G = (int)(a.n_head / a.n_head_kv), kh = h / G;
    const int kv_dim = (int)(a.n_head_kv * HD);
    const int kvt = a.kv_type;
    const int esize = kvt == 0 ? 4 : kvt == 1 ? 2 : 1;
    const int page = (int)a.page;
    const int mctx = (int)a.max_ctx;
    const AttnGroupSmem P = attn_group_plan(HD, a.max_ctx, a.max_pages, kvt, QG);
    float* qs = reinterpret_cast<float*>(smem + P.q);  // [QG][HD]
    int* tbl = reinterpret_cast<int*>(smem + P.table);
    float* sc = reinterpret_cast<float*>(smem + P.sc);  // [QG][max_ctx]
    float* vsc = reinterpret_cast<float*>(smem + P.vsc);
    uint8_t* ring = smem + P.ring;
    const uint8_t* kp = static_cast<const uint8_t*>(a.k_pages);
    const uint8_t* vp = static_cast<const uint8_t*>(a.v_pages);
    const size_t row_bytes = (size_t)kv_dim * esize;
    const size_t head_off = (size_t)kh * HD * esize;
    const int slice = HD * esize;

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
    const int npg = (cmax + page - 1) / page;
    const size_t trow = a.one_seq ? 0 : (size_t)s0;
    for (int i = tid; i < npg; i += HD) tbl[i] = a.block_table[trow * a.max_pages + i];
#pragma unroll
    for (int i = 0; i < QG; ++i)
        qs[i * HD + tid] = cq[i] > 0 ? a.q[(size_t)(s0 + i) * a.q_stride + (size_t)h * HD + tid] : 0.0f;
    __syncthreads();
    auto slot_of = [&](int t) -> size_t { return (size_t)tbl[t / page] * page + t % page; };

    // 1. scores: a K tile's rows are copied by thread t (token t of the tile) and
    // scored by a pair of lanes, for all QG queries
    {
        const int krow = slice + 16;
        const int KT = attn_ktile(HD, kvt);
        auto issue_k = [&](int tile, int buf) {
            const int t = tile * KT + tid;
            if (tid < KT && t < cmax) {
                const uint8_t* src = kp + slot_of(t) * row_bytes + head_off;
                uint8_t* dst = ring + ((size_t)buf * KT + tid) * krow;
                for (int c = 0; c < slice; c += 16) cp_async16(dst + c, src + c);
            }
            cp_async_commit();
        };
        const int ntile = (cmax + KT - 1) / KT;
        issue_k(0, 0);
        for (int tile = 0; tile < ntile; ++tile) {
            cp_async_wait<0>();  // this thread's copies of the tile have landed
            __syncthreads();     // ... every thread's; and tile-1's rows are no longer read
            if (tile + 1 < ntile) issue_k(tile + 1, (tile + 1) & 1);
            else cp_async_commit();
            // a pair of lanes per token: the even lane accumulates the reference's
            // lanes 0..3 (elements d..d+3 of every 8), the odd lane lanes 4..7;
            // the odd lane's four sums then join the even lane's in lane order
            const int half = lane & 1;
            for (int tk = warp * 16 + (lane >> 1); tk < KT; tk += (HD / 32) * 16) {  // warp-uniform trips
                const int t = tile * KT + tk;
                const bool valid = t < cmax;
                const uint8_t* row = ring + ((size_t)(tile & 1) * KT + tk) * krow;
                float acc[QG][4];
#pragma unroll
                for (int i = 0; i < QG; ++i)
#pragma unroll
                    for (int l = 0; l < 4; ++l) acc[i][l] = 0.f;
                const size_t slot = kvt >= 2 && valid ? slot_of(t) : 0;
                if (valid) {
#pragma unroll 2
                    for (int d = 0; d < HD; d += 8) {
                        const int e = d + 4 * half;  // this lane's four elements of the group
                        float kf[4];
                        if (kvt == 1) {
                            const uint2 w = *reinterpret_cast<const uint2*>(row + e * 2);
                            kf[0] = half_bits_to_float((unsigned short)(w.x & 0xffff));
                            kf[1] = half_bits_to_float((unsigned short)(w.x >> 16));
                            kf[2] = half_bits_to_float((unsigned short)(w.y & 0xffff));
                            kf[3] = half_bits_to_float((unsigned short)(w.y >> 16));
                        } else if (kvt == 0) {
                            const float4 u = *reinterpret_cast<const float4*>(row + e * 4);
                            kf[0] = u.x, kf[1] = u.y, kf[2] = u.z, kf[3] = u.w;
                        } else {
                            const uint32_t w = *reinterpret_cast<const uint32_t*>(row + e);
                            const float sc8 = kvt == 3 ? a.k_scales[slot * (kv_dim / 32) + (kh * HD + d) / 32] : 1.0f;
#pragma unroll
                            for (int l = 0; l < 4; ++l) kf[l] = s8_to_f32(w, l) * sc8;
                        }
#pragma unroll
                        for (int i = 0; i < QG; ++i) {
                            const float4 qv = *reinterpret_cast<const float4*>(qs + i * HD + e);
                            acc[i][0] = fmaf(qv.x, kf[0], acc[i][0]);
                            acc[i][1] = fmaf(qv.y, kf[1], acc[i][1]);
                            acc[i][2] = fmaf(qv.z, kf[2], acc[i][2]);
                            acc[i][3] = fmaf(qv.w, kf[3], acc[i][3]);
                        }
                    }
                }
                const float ksc = kvt == 2 && valid ? a.k_scales[slot] : 1.0f;
#pragma unroll
                for (int i = 0; i < QG; ++i) {
                    float hi[4];
#pragma unroll
                    for (int l = 0; l < 4; ++l) hi[l] = __shfl_xor_sync(0xffffffffu, acc[i][l], 1);
                    if (valid && half == 0 && t < cq[i]) {
                        float dot = acc[i][0];
                        dot += acc[i][1];
                        dot += acc[i][2];
                        dot += acc[i][3];
#pragma unroll
                        for (int l = 0; l < 4; ++l) dot += hi[l];
                        if (kvt == 2) dot = dot * ksc;
                        sc[i * mctx + t] = dot / sqrtf((float)HD);
                    }
                }
            }
        }
        cp_async_wait<0>();
    }
    if (kvt == 2) {
        for (int t = tid; t < cmax; t += HD) vsc[t] = a.v_scales[slot_of(t)];
    } else if (kvt == 3) {
        for (int i = tid; i < cmax * (HD / 32); i += HD) {
            const int t = i / (HD / 32), b = i % (HD / 32);
            vsc[i] = a.v_scales[slot_of(t) * (kv_dim / 32) + kh * (HD / 32) + b];
        }
    }
    __syncthreads();  // every K tile is consumed: the ring is free for V

    // 2. per query: max, exp, double denominator, alpha_t = e_t * float(1/den)
    float m[QG];
#pragma unroll
    for (int i = 0; i < QG; ++i) {
        float v = -INFINITY;
        for (int t = tid; t < cq[i]; t += HD) v = fmaxf(v, sc[i * mctx + t]);
        v = warp_max(v);
        if (lane == 0) redf[i][warp] = v;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < QG; ++i) {
        m[i] = redf[i][0];
#pragma unroll
        for (int w = 1; w < HD / 32; ++w) m[i] = fmaxf(m[i], redf[i][w]);
        double den = 0.0;
        for (int t = tid; t < cq[i]; t += HD) {
            const float e = expf_cr(sc[i * mctx + t] - m[i]);
            sc[i * mctx + t] = e;
            den += (double)e;
        }
        den = warp_sum_d(den);
        if (lane == 0) redd[i][warp] = den;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < QG; ++i) {
        double den = 0.0;
#pragma unroll
        for (int w = 0; w < HD / 32; ++w) den += redd[i][w];
        const float inv = (float)(1.0 / den);
        for (int t = tid; t < cq[i]; t += HD) sc[i * mctx + t] = sc[i * mctx + t] * inv;
    }

    // 3. thread d: out_q,d = fma(alpha_q,t, v_t[d], out_q,d) over t < ctx_q in order
    const int chunks = kVTile * slice / 16;
    const int ntile = (cmax + kVTile - 1) / kVTile;
    auto issue_v = [&](int tile) {
        if (tile < ntile) {
            uint8_t* dst = ring + (size_t)(tile % kVStages) * kVTile * slice;
            for (int c = tid; c < chunks; c += HD) {
                const int tt = c / (slice / 16), off = (c % (slice / 16)) * 16;
                const int t = tile * kVTile + tt;
                if (t < cmax) cp_async16(dst + tt * slice + off, vp + slot_of(t) * row_bytes + head_off + off);
            }
        }
        cp_async_commit();
    };
    for (int k = 0; k < kVStages - 1; ++k) issue_v(k);
    float out[QG];
#pragma unroll
    for (int i = 0; i < QG; ++i) out[i] = 0.0f;
    for (int tile = 0; tile < ntile; ++tile) {
        cp_async_wait<kVStages - 2>();
        __syncthreads();  // the tile (and, first time round, every alpha) is visible
        const uint8_t* vt = ring + (size_t)(tile % kVStages) * kVTile * slice;
        const int n = min(kVTile, cmax - tile * kVTile);
        auto vload = [&](int tt, float& v, float& vs) {
            const int t = tile * kVTile + tt;
            vs = 1.0f;
            if (kvt == 1) v = half_bits_to_float(reinterpret_cast<const uint16_t*>(vt + tt * slice)[tid]);
            else if (kvt == 0) v = reinterpret_cast<const float*>(vt + tt * slice)[tid];
            else {
                v = (float)reinterpret_cast<const int8_t*>(vt + tt * slice)[tid];
                vs = kvt == 2 ? vsc[t] : vsc[t * (HD / 32) + tid / 32];
            }
        };
        auto vstep = [&](int tt, float v, float vs) {
            const int t = tile * kVTile + tt;
#pragma unroll
            for (int i = 0; i < QG; ++i) {
                if (t < cq[i]) {
                    float al = sc[i * mctx + t];
                    if (kvt >= 2) al = al * vs;
                    out[i] = fmaf(al, v, out[i]);
                }
            }
        };
        // tokens every query of the group sees, 8 at a time: all their loads
        // go out before the chain steps (each query's steps stay in token order)
        const int nall = max(0, min(n, cmin - tile * kVTile));
        int tt = 0;
        if (kvt < 2 && (mctx & 3) == 0) {  // weights as float4 runs (16-byte aligned rows)
            for (; tt + 8 <= nall; tt += 8) {
                float v[8], vs;
#pragma unroll
                for (int j = 0; j < 8; ++j) vload(tt + j, v[j], vs);
#pragma unroll
                for (int i = 0; i < QG; ++i) {
                    const float* al = sc + i * mctx + tile * kVTile + tt;
                    const float4 a0 = *reinterpret_cast<const float4*>(al);
                    const float4 a1 = *reinterpret_cast<const float4*>(al + 4);
                    const float aj[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
                    for (int j = 0; j < 8; ++j) out[i] = fmaf(aj[j], v[j], out[i]);
                }
            }
        }
        for (; tt + 8 <= nall; tt += 8) {
            float v[8], vs[8], al[QG][8];
#pragma unroll
            for (int j = 0; j < 8; ++j) vload(tt + j, v[j], vs[j]);
#pragma unroll
            for (int i = 0; i < QG; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    al[i][j] = sc[i * mctx + tile * kVTile + tt + j];
                    if (kvt >= 2) al[i][j] = al[i][j] * vs[j];
                }
#pragma unroll
            for (int j = 0; j < 8; ++j)
#pragma unroll
                for (int i = 0; i < QG; ++i) out[i] = fmaf(al[i][j], v[j], out[i]);
        }
        for (; tt < n; ++tt) {
            float v, vs;
            vload(tt, v, vs);
            vstep(tt, v, vs);
        }
        __syncthreads();
        issue_v(tile + kVStages - 1);
    }
    cp_async_wait<0>();
#pragma unroll
    for (int i = 0; i < QG; ++i)
        if (s0 + i < (int)a.n_seq) a.out[((size_t)(s0 + i) * a.n_head + h) * HD + tid] = out[i];
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
                const int v = quant_q8_lane(out[i], dd);
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
        if (blockIdx.x == 0) {  // token rows n_seq..ldb-1 of this block: zero
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
template <int HD, int QG>
cudaError_t launch_group(const AttnArgs& a, size_t smem, cudaStream_t s) {
    dim3 grid((unsigned)((a.n_seq + QG - 1) / QG), (unsigned)a.n_head);
    ensure_smem_attr(attn_group_kernel<HD, QG>, 200 * 1024);
    return launch_pdl(attn_group_kernel<HD, QG>, grid, dim3(HD), smem, s, a);
}
template <int QG>
cudaError_t launch_group_hd(const AttnArgs& a, size_t smem, cudaStream_t s) {
    switch (a.hd) {
        case 64: return launch_group<64, QG>(a, smem, s);
        case 128: return launch_group<128, QG>(a, smem, s);
        case 256: return launch_group<256, QG>(a, smem, s);
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
    if (qg == 1 || smem > 200 * 1024) {
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
