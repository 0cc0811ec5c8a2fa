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
// Grid (n_seq, n_head_kv, n_split).  A CTA owns one kv head of one sequence
// and one contiguous slice of its context, and serves all G = n_head /
// n_head_kv query heads that share that kv head.  Lane l owns head
// dimensions [l*E, l*E+E) (E = hd/32), so every K or V row is one coalesced
// warp-wide read.
//
//  1. scores s_t = (q . k_t) / sqrt(hd) for the slice's tokens (warps stride
//     over tokens), kept in shared memory;
//  2. per query head: m = max s_t, e_t = exp(s_t - m), l = sum e_t;
//  3. o = sum_t e_t v_t (warps stride over tokens, then a cross-warp sum);
//  4. (m, l, o) of the slice go to scratch; attn_merge combines the slices:
//     M = max m_j, L = sum l_j e^(m_j - M), out = sum o_j e^(m_j - M) / L.
// For one slice this is the reference's softmax(q k / sqrt(hd)) v with its
// exact max subtraction; the reference sums the denominator in double and
// scales each weight by float(1/den) before accumulating v, which changes
// only the rounding.
constexpr int kAttnWarps = 4;
constexpr int kAttnMaxG = 8;

template <int E>
__device__ __forceinline__ void load_row(int kv_type, const uint8_t* pages, const float* scales, size_t slot,
                                         int kv_dim, int off, float out[E]) {
    if (kv_type == 1) {
        const uint16_t* r = reinterpret_cast<const uint16_t*>(pages) + slot * kv_dim + off;
        if constexpr (E == 4) {
            const uint2 h = *reinterpret_cast<const uint2*>(r);
            out[0] = half_bits_to_float(h.x & 0xffff);
            out[1] = half_bits_to_float(h.x >> 16);
            out[2] = half_bits_to_float(h.y & 0xffff);
            out[3] = half_bits_to_float(h.y >> 16);
        } else {
#pragma unroll
            for (int i = 0; i < E; ++i) out[i] = half_bits_to_float(r[i]);
        }
    } else if (kv_type == 0) {
        const float* r = reinterpret_cast<const float*>(pages) + slot * kv_dim + off;
#pragma unroll
        for (int i = 0; i < E; ++i) out[i] = r[i];
    } else {
        const int8_t* r = reinterpret_cast<const int8_t*>(pages) + slot * kv_dim + off;
        float sc;
        if (kv_type == 2) sc = 1.0f;  // per-token scale applied by the caller
        else sc = scales[slot * (kv_dim / 32) + off / 32];
#pragma unroll
        for (int i = 0; i < E; ++i) out[i] = (float)r[i] * sc;
    }
}

template <int E, int G>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_split_kernel(AttnArgs a, int split_len, int n_split) {
    extern __shared__ float sm[];  // [G][split_len] scores, then [kAttnWarps][G][hd] partial o
    const int s = blockIdx.x, kh = blockIdx.y, j = blockIdx.z;
    const int hd = (int)a.hd, kv_dim = (int)(a.n_head_kv * a.hd);
    const int ctx = a.ctx_len[s];
    const int t0 = j * split_len, t1 = min(ctx, t0 + split_len);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const size_t n_splits = (size_t)n_split;
    // scratch layout: per (s, head, split): [hd] o, then m, l
    auto slot_of = [&](int t) -> size_t {
        return (size_t)a.block_table[(size_t)s * a.max_pages + t / (int)a.page] * a.page + t % (int)a.page;
    };
    const uint8_t* kp = static_cast<const uint8_t*>(a.k_pages);
    const uint8_t* vp = static_cast<const uint8_t*>(a.v_pages);
    const int off = kh * hd + lane * E;
    float qv[G][E];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const float* qh = a.q + (size_t)s * a.q_stride + (size_t)(kh * G + g) * hd + lane * E;
#pragma unroll
        for (int i = 0; i < E; ++i) qv[g][i] = qh[i];
    }
    const float root = sqrtf((float)hd);
    float* sc = sm;
    if (t0 < t1) {
        // 1. scores
        for (int t = t0 + warp; t < t1; t += kAttnWarps) {
            const size_t sl = slot_of(t);
            float kvv[E];
            load_row<E>(a.kv_type, kp, a.k_scales, sl, kv_dim, off, kvv);
            const float ks = a.kv_type == 2 ? a.k_scales[sl] : 1.0f;
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float p = 0.0f;
#pragma unroll
                for (int i = 0; i < E; ++i) p = fmaf(qv[g][i], kvv[i], p);
                p = warp_sum(p);
                if (lane == 0) sc[g * split_len + (t - t0)] = (p * ks) / root;
            }
        }
    }
    __syncthreads();
    // 2. per-head max / exp / sum over the slice (warp g handles head g, ...)
    __shared__ float mh[kAttnMaxG], lh[kAttnMaxG];
    for (int g = warp; g < G; g += kAttnWarps) {
        float m = -INFINITY;
        for (int t = lane; t < t1 - t0; t += 32) m = fmaxf(m, sc[g * split_len + t]);
        m = warp_max(m);
        float l = 0.0f;
        for (int t = lane; t < t1 - t0; t += 32) {
            const float e = expf(sc[g * split_len + t] - m);
            sc[g * split_len + t] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) {
            mh[g] = m;
            lh[g] = l;
        }
    }
    __syncthreads();
    // 3. o = sum e_t v_t
    float acc[G][E];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int i = 0; i < E; ++i) acc[g][i] = 0.0f;
    for (int t = t0 + warp; t < t1; t += kAttnWarps) {
        const size_t sl = slot_of(t);
        float vv[E];
        load_row<E>(a.kv_type, vp, a.v_scales, sl, kv_dim, off, vv);
        const float vs = a.kv_type == 2 ? a.v_scales[sl] : 1.0f;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float p = sc[g * split_len + (t - t0)] * vs;
#pragma unroll
            for (int i = 0; i < E; ++i) acc[g][i] = fmaf(p, vv[i], acc[g][i]);
        }
    }
    float* po = sm + (size_t)G * split_len;  // [kAttnWarps][G][hd]
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int i = 0; i < E; ++i) po[((size_t)warp * G + g) * hd + lane * E + i] = acc[g][i];
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * hd; idx += blockDim.x) {
        const int g = idx / hd, dcol = idx % hd;
        float o = 0.0f;
        for (int w = 0; w < kAttnWarps; ++w) o += po[((size_t)w * G + g) * hd + dcol];
        float* dst = a.scratch + (((size_t)s * a.n_head + (size_t)kh * G + g) * n_splits + j) * (hd + 2);
        dst[dcol] = o;
        if (dcol == 0) {
            dst[hd] = t0 < t1 ? mh[g] : -INFINITY;
            dst[hd + 1] = t0 < t1 ? lh[g] : 0.0f;
        }
    }
}

__global__ void attn_merge_kernel(AttnArgs a, int n_split) {
    const int s = blockIdx.x, h = blockIdx.y, hd = (int)a.hd;
    const float* base = a.scratch + ((size_t)s * a.n_head + h) * n_split * (hd + 2);
    float M = -INFINITY;
    for (int j = 0; j < n_split; ++j) M = fmaxf(M, base[(size_t)j * (hd + 2) + hd]);
    float L = 0.0f;
    for (int j = 0; j < n_split; ++j) {
        const float m = base[(size_t)j * (hd + 2) + hd];
        if (m != -INFINITY) L += base[(size_t)j * (hd + 2) + hd + 1] * expf(m - M);
    }
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
    for (int dcol = threadIdx.x; dcol < hd; dcol += blockDim.x) {
        float o = 0.0f;
        for (int j = 0; j < n_split; ++j) {
            const float m = base[(size_t)j * (hd + 2) + hd];
            if (m != -INFINITY) o = fmaf(base[(size_t)j * (hd + 2) + dcol], expf(m - M), o);
        }
        a.out[((size_t)s * a.n_head + h) * hd + dcol] = o * inv;
    }
}

template <int E, int G>
static cudaError_t launch_attn(dim3 grid, size_t smem, cudaStream_t s, const AttnArgs& a, int split_len, int n_split) {
    ensure_smem_attr(attn_split_kernel<E, G>, 200 * 1024);
    attn_split_kernel<E, G><<<grid, kAttnWarps * 32, smem, s>>>(a, split_len, n_split);
    return cudaSuccess;
}
template <int E>
static cudaError_t launch_attn_g(int G, dim3 grid, size_t smem, cudaStream_t s, const AttnArgs& a, int split_len,
                                 int n_split) {
    switch (G) {
        case 1: return launch_attn<E, 1>(grid, smem, s, a, split_len, n_split);
        case 2: return launch_attn<E, 2>(grid, smem, s, a, split_len, n_split);
        case 4: return launch_attn<E, 4>(grid, smem, s, a, split_len, n_split);
        case 8: return launch_attn<E, 8>(grid, smem, s, a, split_len, n_split);
    }
    return cudaErrorInvalidValue;
}
static cudaError_t launch_attn_e(uint64_t hd, int G, dim3 grid, size_t smem, cudaStream_t s, const AttnArgs& a,
                                 int split_len, int n_split) {
    switch (hd) {
        case 64: return launch_attn_g<2>(G, grid, smem, s, a, split_len, n_split);
        case 128: return launch_attn_g<4>(G, grid, smem, s, a, split_len, n_split);
        case 256: return launch_attn_g<8>(G, grid, smem, s, a, split_len, n_split);
    }
    return cudaErrorInvalidValue;
}

static void split_plan(uint64_t n_seq, uint64_t n_head_kv, uint64_t G, uint64_t hd, uint64_t max_ctx, int& split_len,
                       int& n_split) {
    const uint64_t units = n_seq * n_head_kv;
    const uint64_t target = (uint64_t)num_sms() * 4;
    uint64_t ns = units >= target ? 1 : (target + units - 1) / units;
    const uint64_t max_ns = (max_ctx + 31) / 32;  // keep >= 32 tokens per slice
    if (ns > max_ns) ns = max_ns ? max_ns : 1;
    uint64_t len = (max_ctx + ns - 1) / ns;
    len = (len + 15) / 16 * 16;
    if (len == 0) len = 16;
    // the slice's scores and the per-warp partial outputs must fit in shared memory
    const uint64_t cap = ((200 * 1024 / 4) - (uint64_t)kAttnWarps * G * hd) / G / 16 * 16;
    if (len > cap) len = cap;
    split_len = (int)len;
    n_split = (int)((max_ctx + len - 1) / len);
    if (n_split < 1) n_split = 1;
}

uint64_t attn_scratch_floats(uint64_t n_seq, uint64_t n_head, uint64_t hd, uint64_t max_ctx) {
    // upper bound over every plan split_plan can choose for this shape
    // (slices are at least 16 tokens long)
    const uint64_t max_ns = max_ctx / 16 + 1;
    return n_seq * n_head * max_ns * (hd + 2);
}

cudaError_t paged_attn_decode(const AttnArgs& a, cudaStream_t s) {
    if (!a.n_seq) return cudaSuccess;
    const int G = (int)(a.n_head / a.n_head_kv);
    if (G > kAttnMaxG || a.n_head % a.n_head_kv) return cudaErrorInvalidValue;
    int split_len, n_split;
    split_plan(a.n_seq, a.n_head_kv, (uint64_t)G, a.hd, a.max_ctx ? a.max_ctx : 1, split_len, n_split);
    const size_t smem = ((size_t)G * split_len + (size_t)kAttnWarps * G * a.hd) * sizeof(float);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    dim3 grid((unsigned)a.n_seq, (unsigned)a.n_head_kv, (unsigned)n_split);
    cudaError_t e = launch_attn_e(a.hd, G, grid, smem, s, a, split_len, n_split);
    if (e != cudaSuccess) return e;
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    attn_merge_kernel<<<dim3((unsigned)a.n_seq, (unsigned)a.n_head), 128, 0, s>>>(a, n_split);
    return cudaGetLastError();
}

}  // namespace mvb
