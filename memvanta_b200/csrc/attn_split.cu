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
// Memory: a warp takes its tokens 32 at a time; for keys and values alike
// lane l holds dimensions [l*hd/32, (l+1)*hd/32) of a token, so a token's
// head slice is one coalesced row for the warp, and the 32 tokens' slices
// are requested at once before they are used.  One CTA per (sequence, head), 4
// warps, a few KB of shared memory: many CTAs per SM keep enough bytes in
// flight for HBM.
#include "common.cuh"
#include "kernels.cuh"

namespace mvb {

namespace {

constexpr int kSW = 4;  // warps per (sequence, head)

__device__ __forceinline__ float expf_cr(float x) { return (float)exp((double)x); }

// DPL consecutive value elements of one token (lane's dimensions), as floats
// (Q8 types: raw int8 values).
template <int KVT, int DPL>
struct VSlice {
    static constexpr int ES = KVT == 0 ? 4 : KVT == 1 ? 2 : 1;
    static constexpr int W = DPL * ES / 4 > 0 ? DPL * ES / 4 : 1;  // 32-bit words
    uint32_t w[W];
    __device__ __forceinline__ void load(const uint8_t* src) {
        if constexpr (DPL * ES >= 16) {
#pragma unroll
            for (int i = 0; i < W; i += 4) {
                const uint4 u = __ldg(reinterpret_cast<const uint4*>(src) + i / 4);
                w[i] = u.x, w[i + 1] = u.y, w[i + 2] = u.z, w[i + 3] = u.w;
            }
        } else if constexpr (DPL * ES == 8) {
            const uint2 u = __ldg(reinterpret_cast<const uint2*>(src));
            w[0] = u.x, w[1] = u.y;
        } else if constexpr (DPL * ES == 4) {
            w[0] = __ldg(reinterpret_cast<const uint32_t*>(src));
        } else {  // 2 bytes (hd 64, int8)
            w[0] = __ldg(reinterpret_cast<const unsigned short*>(src));
        }
    }
    __device__ __forceinline__ float at(int j) const {
        if constexpr (KVT == 0) return __uint_as_float(w[j]);
        else if constexpr (KVT == 1) return half_bits_to_float((unsigned short)(w[j / 2] >> (16 * (j & 1))));
        else return s8_to_f32(w[j / 4], j & 3);
    }
};

template <int HD, int KVT>
__global__ void __launch_bounds__(kSW * 32) attn_split_kernel(AttnArgs a) {
    constexpr int DPL = HD / 32;                        // dimensions per lane (values)
    constexpr int ES = KVT == 0 ? 4 : KVT == 1 ? 2 : 1;  // bytes per element
    __shared__ float qs[HD];
    __shared__ float mw[kSW];
    __shared__ double dw[kSW];
    __shared__ float ow[kSW][HD];
    const int s = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = (int)(a.n_head / a.n_head_kv), kh = h / G;
    const int kv_dim = (int)(a.n_head_kv * HD), page = (int)a.page;
    const size_t row_bytes = (size_t)kv_dim * ES;
    const size_t head_off = (size_t)kh * HD * ES;
    const int32_t* tbl = a.block_table + (a.one_seq ? 0 : (size_t)s) * a.max_pages;
    const uint8_t* kp = static_cast<const uint8_t*>(a.k_pages);
    const uint8_t* vp = static_cast<const uint8_t*>(a.v_pages);
    pdl_trigger();
    pdl_wait();
    const int ctx = a.ctx_len[s];
    for (int i = tid; i < HD; i += kSW * 32) qs[i] = a.q[(size_t)s * a.q_stride + (size_t)h * HD + i];
    __syncthreads();
    auto slot_of = [&](int t) -> size_t { return (size_t)__ldg(tbl + t / page) * page + t % page; };
    // this warp's tokens: a contiguous quarter of the context, in groups of 32
    const int per = (ctx + kSW - 1) / kSW;
    const int t0 = min(ctx, warp * per), t1 = min(ctx, t0 + per);
    float m = -INFINITY;
    double den = 0.0;
    float o[DPL];
#pragma unroll
    for (int j = 0; j < DPL; ++j) o[j] = 0.0f;
    const float root = sqrtf((float)HD);
    float qr[DPL];  // the query elements this lane multiplies
#pragma unroll
    for (int j = 0; j < DPL; ++j) qr[j] = qs[lane * DPL + j];
    for (int g0 = t0; g0 < t1; g0 += 32) {
        const int n = min(32, t1 - g0);
        // scores: the warp reads one token's key slice as one coalesced row
        // (lane = hd/32 consecutive elements), the 32 tokens' rows requested
        // at once, then one dot per token (lane partials summed by shuffles)
        const int t = g0 + lane;
        const bool live = lane < n;
        const size_t slot = live ? slot_of(t) : 0;
        const size_t koff = head_off + (size_t)lane * DPL * ES;
        float sc = -INFINITY;
        {
            VSlice<KVT, DPL> kk[32];
#pragma unroll
            for (int u = 0; u < 32; ++u) {
                const size_t su = __shfl_sync(0xffffffffu, slot, u);
                if (u < n) kk[u].load(kp + su * row_bytes + koff);
            }
#pragma unroll
            for (int u = 0; u < 32; ++u) {
                if (u < n) {  // warp-uniform
                    float part = 0.0f;
#pragma unroll
                    for (int j = 0; j < DPL; ++j) part = fmaf(qr[j], kk[u].at(j), part);
                    if constexpr (KVT == 3) {
                        const size_t su = __shfl_sync(0xffffffffu, slot, u);
                        part *= __ldg(a.k_scales + su * (kv_dim / 32) + (kh * HD + lane * DPL) / 32);
                    }
                    part = warp_sum(part);
                    if (lane == u) sc = part;
                }
            }
            if constexpr (KVT == 2) sc = sc * (live ? __ldg(a.k_scales + slot) : 0.f);
            if (live) sc = sc / root;
            else sc = -INFINITY;
        }
        // the running max, the sums rescaled when it rises
        const float nm = fmaxf(m, warp_max(sc));
        if (nm != m && m != -INFINITY) {
            const float c = expf_cr(m - nm);
            den *= (double)c;
#pragma unroll
            for (int j = 0; j < DPL; ++j) o[j] *= c;
        }
        m = nm;
        float e = live ? expf_cr(sc - m) : 0.0f;
        den += warp_sum_d((double)e);
        // values: lane = DPL dimensions, the group's slices requested at once
        const size_t voff = head_off + (size_t)lane * DPL * ES;
        VSlice<KVT, DPL> v[32];
        float vs = 1.0f;  // this lane's token's value scale (Q8 types)
#pragma unroll
        for (int u = 0; u < 32; ++u) {
            const size_t su = __shfl_sync(0xffffffffu, slot, u);
            if (u < n) v[u].load(vp + su * row_bytes + voff);
        }
        if constexpr (KVT == 2) vs = live ? __ldg(a.v_scales + slot) : 0.f;
        (void)vs;
#pragma unroll
        for (int u = 0; u < 32; ++u) {
            if (u < n) {
                float al = __shfl_sync(0xffffffffu, e, u);
                if constexpr (KVT == 2) al = al * __shfl_sync(0xffffffffu, vs, u);
                if constexpr (KVT == 3) {
                    const size_t su = __shfl_sync(0xffffffffu, slot, u);
                    al = al * __ldg(a.v_scales + su * (kv_dim / 32) + (kh * HD + lane * DPL) / 32);
                }
#pragma unroll
                for (int j = 0; j < DPL; ++j) o[j] = fmaf(al, v[u].at(j), o[j]);
            }
        }
    }
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

template <int HD>
cudaError_t launch_split_hd(const AttnArgs& a, cudaStream_t s) {
    const dim3 grid((unsigned)a.n_seq, (unsigned)a.n_head);
    switch (a.kv_type) {
        case 0: return launch_opt(false, attn_split_kernel<HD, 0>, grid, dim3(kSW * 32), 0, s, a);
        case 1: return launch_opt(false, attn_split_kernel<HD, 1>, grid, dim3(kSW * 32), 0, s, a);
        case 2: return launch_opt(false, attn_split_kernel<HD, 2>, grid, dim3(kSW * 32), 0, s, a);
        case 3: return launch_opt(false, attn_split_kernel<HD, 3>, grid, dim3(kSW * 32), 0, s, a);
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
