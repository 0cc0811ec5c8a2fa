// attn_split.cu -- one-query paged attention for many sequences (BASELINE
// config 4: ragged contexts, scattered pages) split over the context.
//
// The reference's decode loop (src/llama_model.cpp:256 over
// PagedKVCache::dot_key / add_value, :23-55) walks one head's tokens in
// order: scores, their max, exp and a double denominator, then one FMA chain
// per output dimension over all tokens.  That last chain is sequential in
// the context, so a kernel that keeps it (attention.cu) gets one CTA's worth
// of parallelism per (sequence, head).  Here every warp of the CTA owns one
// contiguous quarter of the context (split-K) and keeps its own running
// softmax state, merged once at the end in a fixed order:
//
//   warp w, tokens [t0_w, t1_w):
//     s_t  = dot(q, k_t) / sqrt(hd)       lane partials summed in a warp tree
//     m_w  = max s_t,  e_t = exp(s_t - m_w),  den_w = sum e_t (double)
//     o_w[d] = sum_t e_t * v_t[d]          (fp32 FMA chain per dimension)
//   merge:  M = max_w m_w,  c_w = exp(m_w - M)
//     den = sum_w den_w * c_w (double),  out[d] = (sum_w o_w[d] * c_w) * float(1/den)
//
// The dot products, the weights e_t * c_w (against the reference's
// exp(s_t - M)) and the output sums each round in another order than the
// reference's, so outputs agree with it to ~1e-6 of their scale (the tests
// hold it to 1e-5); attention.cu's kernel stays the exact path.
//
// Memory: each warp streams its tokens through its own ring of shared-memory
// stages (16 tokens' key and value head slices per stage, 16-byte cp.async
// copies spread over the lanes, two stages in flight while one is used), so
// no warp waits for another before the merge.  Scores: two lanes per token,
// each over half of the head's dimensions; values: lane = hd/32 consecutive
// dimensions.  One CTA per (sequence, head), 4 warps.
#include "common.cuh"
#include "kernels.cuh"

namespace mvb {

namespace {

constexpr int kSW = 4;  // warps per (sequence, head)

__device__ __forceinline__ float expf_cr(float x) { return (float)exp((double)x); }

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gsrc) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

constexpr int kTok = 16;  // tokens per stage

// Shared-memory plan of one CTA: the query, the block-table row, and per warp
// a ring of S stages of kTok tokens' key and value head slices (rows padded
// by 16 bytes) plus their scales (Q8: one per token, Q8_0: hd/32 per token).
template <int HD, int KVT>
struct SplitPlan {
    static constexpr int ES = KVT == 0 ? 4 : KVT == 1 ? 2 : 1;
    static constexpr int SL = HD * ES;        // bytes of one head slice
    static constexpr int SLP = SL + 16;       // padded row
    static constexpr int NSC = KVT == 2 ? 1 : KVT == 3 ? HD / 32 : 0;  // scales per token
    static constexpr int S = KVT == 0 ? 2 : 3;                         // ring stages
    static constexpr int STAGE = 2 * kTok * SLP + 2 * kTok * NSC * 4;
    static constexpr int WARP = S * STAGE;
};

template <int HD, int KVT>
__global__ void __launch_bounds__(kSW * 32) attn_split_kernel(AttnArgs a) {
    using P = SplitPlan<HD, KVT>;
    constexpr int DPL = HD / 32;  // value dimensions per lane
    constexpr int ES = P::ES, SL = P::SL, SLP = P::SLP, NSC = P::NSC, S = P::S;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ __align__(16) float qs[HD];
    __shared__ float mw[kSW];
    __shared__ double dw[kSW];
    __shared__ float ow[kSW][HD];
    const int s = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = (int)(a.n_head / a.n_head_kv), kh = h / G;
    const int kv_dim = (int)(a.n_head_kv * HD), page = (int)a.page;
    const size_t row_bytes = (size_t)kv_dim * ES;
    const size_t head_off = (size_t)kh * HD * ES;
    const uint8_t* kp = static_cast<const uint8_t*>(a.k_pages);
    const uint8_t* vp = static_cast<const uint8_t*>(a.v_pages);
    int* tbl = reinterpret_cast<int*>(smem + kSW * P::WARP);
    unsigned char* ring = smem + warp * P::WARP;
    const int ctx = a.ctx_len[s];
    const int npg = (ctx + page - 1) / page;
    const int32_t* trow = a.block_table + (a.one_seq ? 0 : (size_t)s) * a.max_pages;
    for (int i = tid; i < npg; i += kSW * 32) tbl[i] = trow[i];
    for (int i = tid; i < HD; i += kSW * 32) qs[i] = a.q[(size_t)s * a.q_stride + (size_t)h * HD + i];
    __syncthreads();
    auto slot_of = [&](int t) -> size_t { return (size_t)tbl[t / page] * page + t % page; };
    // this warp's tokens: a contiguous quarter of the context, in stages of kTok
    const int per = (ctx + kSW - 1) / kSW;
    const int t0 = min(ctx, warp * per), t1 = min(ctx, t0 + per);
    const int ng = (t1 - t0 + kTok - 1) / kTok;
    // stage g of this warp into ring slot g % S: kTok tokens' key and value
    // slices (16-byte copies spread over the lanes) and their scales
    auto issue = [&](int g) {
        if (g < ng) {
            unsigned char* base = ring + (g % S) * P::STAGE;
            constexpr int CPT = SL / 16;  // 16-byte chunks per slice
            const int tb = t0 + g * kTok;
            // lane u < kTok: the cache slot of token tb + u, once per stage
            const int tu = tb + (lane & (kTok - 1));
            const size_t myslot = tu < t1 ? slot_of(tu) : 0;
#pragma unroll
            for (int i = 0; i < 2 * kTok * CPT / 32; ++i) {
                const int c = lane + 32 * i;  // chunk: (K|V, token u, 16-byte offset)
                const int kv = c / (kTok * CPT), rem = c % (kTok * CPT), u = rem / CPT, off = (rem % CPT) * 16;
                const size_t su = __shfl_sync(0xffffffffu, myslot, u);
                if (tb + u < t1)
                    cp_async16(base + (kv * kTok + u) * SLP + off, (kv ? vp : kp) + su * row_bytes + head_off + off);
            }
            if constexpr (NSC > 0) {
                const int u = lane & 15, kv = lane >> 4, t = tb + u;
                if (t < t1) {
                    const float* src = (kv ? a.v_scales : a.k_scales) +
                                       (KVT == 2 ? myslot : myslot * (kv_dim / 32) + kh * NSC);
                    float* dst = reinterpret_cast<float*>(base + 2 * kTok * SLP) + (kv * kTok + u) * NSC;
#pragma unroll
                    for (int i = 0; i < NSC; ++i) cp_async4(dst + i, src + i);
                }
            }
        }
        cp_async_commit();
    };
    float m = -INFINITY;
    double den = 0.0;
    float o[DPL];
#pragma unroll
    for (int j = 0; j < DPL; ++j) o[j] = 0.0f;
    const float root = sqrtf((float)HD);
    const int u = lane & 15, half = lane >> 4;  // scores: token u of the stage, half of its dimensions
#pragma unroll
    for (int k = 0; k < S - 1; ++k) issue(k);
    for (int g = 0; g < ng; ++g) {
        issue(g + S - 1);        // into the slot stage g-1 used (consumed before the last __syncwarp)
        cp_async_wait<S - 1>();  // this lane's copies of stage g have landed
        __syncwarp();            // ... and every lane's
        const unsigned char* base = ring + (g % S) * P::STAGE;
        const float* ksc = reinterpret_cast<const float*>(base + 2 * kTok * SLP);
        const float* vsc = ksc + kTok * NSC;
        const int n = min(kTok, t1 - (t0 + g * kTok));
        // scores: two lanes per token, each over half of the dimensions
        float part = 0.0f;
        {
            const unsigned char* kr = base + u * SLP + half * (SL / 2);
            const float* qh = qs + half * (HD / 2);
            if constexpr (KVT == 0) {
#pragma unroll
                for (int d = 0; d < HD / 2; d += 4) {
                    const float4 k4 = *reinterpret_cast<const float4*>(kr + d * 4);
                    part = fmaf(qh[d], k4.x, part);
                    part = fmaf(qh[d + 1], k4.y, part);
                    part = fmaf(qh[d + 2], k4.z, part);
                    part = fmaf(qh[d + 3], k4.w, part);
                }
            } else if constexpr (KVT == 1) {
#pragma unroll
                for (int d = 0; d < HD / 2; d += 8) {
                    const uint4 w = *reinterpret_cast<const uint4*>(kr + d * 2);
                    const float4 qa = *reinterpret_cast<const float4*>(qh + d);
                    const float4 qb = *reinterpret_cast<const float4*>(qh + d + 4);
                    const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int l = 0; l < 8; ++l)
                        part = fmaf(qv[l], half_bits_to_float((unsigned short)(ws[l / 2] >> (16 * (l & 1)))), part);
                }
            } else {
#pragma unroll
                for (int bb = 0; bb < HD / 64; ++bb) {  // the 32-element blocks of this half
                    float bs = 0.0f;
#pragma unroll
                    for (int d = 0; d < 32; d += 16) {
                        const uint4 w = *reinterpret_cast<const uint4*>(kr + bb * 32 + d);
                        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                        for (int l = 0; l < 16; ++l) bs = fmaf(qh[bb * 32 + d + l], s8_to_f32(ws[l / 4], l & 3), bs);
                    }
                    part += KVT == 3 ? bs * ksc[u * NSC + half * (HD / 64) + bb] : bs;
                }
            }
        }
        float dot = part + __shfl_xor_sync(0xffffffffu, part, 16);
        if constexpr (KVT == 2) dot = dot * ksc[u];
        const float sc = u < n ? dot / root : -INFINITY;
        // the running max, the sums rescaled when it rises
        const float nm = fmaxf(m, warp_max(sc));
        if (nm != m && m != -INFINITY) {
            const float c = expf_cr(m - nm);
            den *= (double)c;
#pragma unroll
            for (int j = 0; j < DPL; ++j) o[j] *= c;
        }
        m = nm;
        const float e = u < n ? expf_cr(sc - m) : 0.0f;
        den += warp_sum_d(half == 0 ? (double)e : 0.0);
        // values: lane = DPL consecutive dimensions, tokens in order
        const unsigned char* vr = base + kTok * SLP + lane * DPL * ES;
        for (int uu = 0; uu < n; ++uu) {
            float al = __shfl_sync(0xffffffffu, e, uu);
            if constexpr (KVT == 2) al = al * vsc[uu];
            if constexpr (KVT == 3) al = al * vsc[uu * NSC + lane * DPL / 32];
            const unsigned char* vv = vr + uu * SLP;
            float v[DPL];
            if constexpr (KVT == 0) {
#pragma unroll
                for (int j = 0; j < DPL; j += 2) {
                    const float2 f = *reinterpret_cast<const float2*>(vv + j * 4);
                    v[j] = f.x, v[j + 1] = f.y;
                }
            } else if constexpr (KVT == 1) {
#pragma unroll
                for (int j = 0; j < DPL; j += 2) {
                    const uint32_t w = *reinterpret_cast<const uint32_t*>(vv + j * 2);
                    v[j] = half_bits_to_float((unsigned short)(w & 0xffff));
                    v[j + 1] = half_bits_to_float((unsigned short)(w >> 16));
                }
            } else {
#pragma unroll
                for (int j = 0; j < DPL; j += 2) {
                    const uint32_t w = *reinterpret_cast<const unsigned short*>(vv + j);
                    v[j] = s8_to_f32(w, 0);
                    v[j + 1] = s8_to_f32(w, 1);
                }
            }
#pragma unroll
            for (int j = 0; j < DPL; ++j) o[j] = fmaf(al, v[j], o[j]);
        }
        __syncwarp();  // every lane is done with this slot before it is refilled
    }
    cp_async_wait<0>();
    // merge the warps' states in warp order
    if (lane == 0) {
        mw[warp] = m;
        dw[warp] = den;
    }
#pragma unroll
    for (int j = 0; j < DPL; ++j) ow[warp][lane * DPL + j] = o[j];
    __syncthreads();
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kSW; ++w) M = fmaxf(M, mw[w]);
    float cw[kSW];
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < kSW; ++w) {
        cw[w] = mw[w] == -INFINITY ? 0.0f : expf_cr(mw[w] - M);
        tot += dw[w] * (double)cw[w];
    }
    const float inv = (float)(1.0 / tot);
    for (int d = tid; d < HD; d += kSW * 32) {
        float acc = 0.0f;
#pragma unroll
        for (int w = 0; w < kSW; ++w) acc = fmaf(ow[w][d], cw[w], acc);
        a.out[((size_t)s * a.n_head + h) * HD + d] = acc * inv;
    }
}

template <int HD, int KVT>
size_t split_smem(const AttnArgs& a) {
    return (size_t)kSW * SplitPlan<HD, KVT>::WARP + ((a.max_ctx + a.page - 1) / a.page) * 4;
}

template <int HD, int KVT>
cudaError_t launch_split(const AttnArgs& a, cudaStream_t s) {
    const size_t smem = split_smem<HD, KVT>(a);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    ensure_smem_attr(attn_split_kernel<HD, KVT>, 200 * 1024);
    return launch_opt(false, attn_split_kernel<HD, KVT>, dim3((unsigned)a.n_seq, (unsigned)a.n_head),
                      dim3(kSW * 32), smem, s, a);
}

template <int HD>
cudaError_t launch_split_hd(const AttnArgs& a, cudaStream_t s) {
    switch (a.kv_type) {
        case 0: return launch_split<HD, 0>(a, s);
        case 1: return launch_split<HD, 1>(a, s);
        case 2: return launch_split<HD, 2>(a, s);
        case 3: return launch_split<HD, 3>(a, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t paged_attn_decode_split(const AttnArgs& a, cudaStream_t s) {
    if (!a.n_seq) return cudaSuccess;
    if (a.n_head % a.n_head_kv) return cudaErrorInvalidValue;
    switch (a.hd) {
        case 64: return launch_split_hd<64>(a, s);
        case 128: return launch_split_hd<128>(a, s);
        case 256: return launch_split_hd<256>(a, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace mvb
