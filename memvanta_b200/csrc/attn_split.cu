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
//     s_t  = dot(q, k_t) / sqrt(hd)       the reference's 8-lane FMA dot and
//                                         left-to-right sum (bit-identical)
//     m_w  = max s_t,  e_t = exp(s_t - m_w),  den_w = sum e_t (double)
//     o_w[d] = sum_t e_t * v_t[d]          (fp32 FMA chain per dimension)
//   merge:  M = max_w m_w,  c_w = exp(m_w - M)
//     den = sum_w den_w * c_w (double),  out[d] = (sum_w o_w[d] * c_w) * float(1/den)
//
// Scores are exact; the weights e_t * c_w differ from the reference's
// exp(s_t - M) by a rounding or two and the output is summed in another
// order, so outputs agree with the reference to ~1e-6 of their scale (the
// tests hold it to 1e-5).  attention.cu's kernel stays the exact path.
//
// Memory: lane = token for the keys (one lane reads its token's head slice,
// 16-byte loads, 32 rows in flight per warp), lane = 4 (8 for hd 256)
// consecutive dimensions for the values (a warp reads a token's slice as one
// coalesced row), the loads of 8 tokens issued before their FMA steps.  One
// CTA per (sequence, head), 4 warps, a few KB of shared memory: many CTAs
// per SM keep enough loads in flight for HBM.
#include "common.cuh"
#include "kernels.cuh"

namespace mvb {

namespace {

constexpr int kSW = 4;  // warps per (sequence, head)

__device__ __forceinline__ float expf_cr(float x) { return (float)exp((double)x); }

// 8 consecutive cache elements of one token's row as floats (Q8 types: raw
// int8 values; the scale is applied by the caller).
template <int KVT>
__device__ __forceinline__ void load8(const uint8_t* row, int d, float (&v)[8]) {
    if constexpr (KVT == 0) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(row + d * 4));
        const float4 b = __ldg(reinterpret_cast<const float4*>(row + d * 4 + 16));
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else if constexpr (KVT == 1) {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(row + d * 2));
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int l = 0; l < 8; ++l) v[l] = half_bits_to_float((unsigned short)(ws[l / 2] >> (16 * (l & 1))));
    } else {
        const uint2 w = __ldg(reinterpret_cast<const uint2*>(row + d));
#pragma unroll
        for (int l = 0; l < 8; ++l) v[l] = s8_to_f32(l < 4 ? w.x : w.y, l & 3);
    }
}

template <int HD, int KVT>
__global__ void __launch_bounds__(kSW * 32) attn_split_kernel(AttnArgs a) {
    constexpr int DPL = HD / 32;                        // dimensions per lane (values)
    constexpr int ES = KVT == 0 ? 4 : KVT == 1 ? 2 : 1;  // bytes per element
    __shared__ float qs[HD];
    __shared__ float ew[kSW][32 * 8];                   // e_t of the tokens a warp is on (one 256-token pass)
    __shared__ float mw[kSW];
    __shared__ double dw[kSW];
    __shared__ float ow[kSW][HD];
    const int s = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = (int)(a.n_head / a.n_head_kv), kh = h / G;
    const int kv_dim = (int)(a.n_head_kv * HD), page = (int)a.page;
    const size_t row_bytes = (size_t)kv_dim * ES;
    const size_t head_off = (size_t)kh * HD * ES;
    const int32_t* tbl = a.block_table + (a.one_seq ? 0 : (size_t)s) * a.max_pages;
    pdl_trigger();
    pdl_wait();
    const int ctx = a.ctx_len[s];
    for (int i = tid; i < HD; i += kSW * 32) qs[i] = a.q[(size_t)s * a.q_stride + (size_t)h * HD + i];
    __syncthreads();
    auto slot_of = [&](int t) -> size_t { return (size_t)__ldg(tbl + t / page) * page + t % page; };
    // this warp's tokens
    const int per = (ctx + kSW - 1) / kSW;
    const int t0 = min(ctx, warp * per), t1 = min(ctx, t0 + per);
    float m = -INFINITY;
    double den = 0.0;
    float o[DPL];
#pragma unroll
    for (int j = 0; j < DPL; ++j) o[j] = 0.0f;
    const float root = sqrtf((float)HD);
    // passes of up to 256 tokens: scores (lane = token, 8 per lane), then the
    // running max is raised and the partial sums rescaled once per pass
    for (int p0 = t0; p0 < t1; p0 += 256) {
        const int np = min(256, t1 - p0);
        float sc[8];
        float pm = -INFINITY;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int tt = i * 32 + lane;
            sc[i] = -INFINITY;
            if (tt < np) {
                const int t = p0 + tt;
                const size_t slot = slot_of(t);
                const uint8_t* row = static_cast<const uint8_t*>(a.k_pages) + slot * row_bytes + head_off;
                float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
                for (int d = 0; d < HD; d += 8) {
                    float kv[8];
                    load8<KVT>(row, d, kv);
                    float sc8 = 1.0f;
                    if constexpr (KVT == 3) sc8 = __ldg(a.k_scales + slot * (kv_dim / 32) + (kh * HD + d) / 32);
#pragma unroll
                    for (int l = 0; l < 8; ++l)
                        acc[l] = fmaf(qs[d + l], KVT == 3 ? kv[l] * sc8 : kv[l], acc[l]);
                }
                float dot = acc[0];
#pragma unroll
                for (int l = 1; l < 8; ++l) dot += acc[l];
                if constexpr (KVT == 2) dot = dot * __ldg(a.k_scales + slot);
                sc[i] = dot / root;
                pm = fmaxf(pm, sc[i]);
            }
        }
        pm = warp_max(pm);
        const float nm = fmaxf(m, pm);
        // rescale what this warp summed so far to the new max
        if (m != nm && m != -INFINITY) {
            const float c = expf_cr(m - nm);
            den *= (double)c;
#pragma unroll
            for (int j = 0; j < DPL; ++j) o[j] *= c;
        }
        m = nm;
        double pden = 0.0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int tt = i * 32 + lane;
            const float e = tt < np ? expf_cr(sc[i] - m) : 0.0f;
            if (tt < np) ew[warp][tt] = e;
            pden += (double)e;
        }
        den += warp_sum_d(pden);
        __syncwarp();
        // values: lane owns dimensions lane*DPL .. +DPL-1, tokens in order,
        // the loads of 8 tokens before their FMA steps
        const size_t voff = head_off + (size_t)lane * DPL * ES;
        for (int tt = 0; tt < np; tt += 8) {
            const int n8 = min(8, np - tt);
            float v[8][DPL];
            float al[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                al[u] = 0.0f;
#pragma unroll
                for (int j = 0; j < DPL; ++j) v[u][j] = 0.0f;
                if (u < n8) {
                    const int t = p0 + tt + u;
                    const size_t slot = slot_of(t);
                    const uint8_t* src = static_cast<const uint8_t*>(a.v_pages) + slot * row_bytes + voff;
                    al[u] = ew[warp][tt + u];
                    // DPL consecutive elements: two per load (hd 64 gives lanes two)
                    if constexpr (KVT == 0) {
#pragma unroll
                        for (int j = 0; j < DPL; j += 2) {
                            const float2 f = __ldg(reinterpret_cast<const float2*>(src) + j / 2);
                            v[u][j] = f.x, v[u][j + 1] = f.y;
                        }
                    } else if constexpr (KVT == 1) {
#pragma unroll
                        for (int j = 0; j < DPL; j += 2) {
                            const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(src) + j / 2);
                            v[u][j] = half_bits_to_float(w & 0xffff);
                            v[u][j + 1] = half_bits_to_float(w >> 16);
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < DPL; j += 2) {
                            const uint32_t w = __ldg(reinterpret_cast<const unsigned short*>(src) + j / 2);
                            v[u][j] = s8_to_f32(w, 0);
                            v[u][j + 1] = s8_to_f32(w, 1);
                        }
                        // one scale per token (Q8) or per 32-element block (Q8_0)
                        al[u] *= KVT == 2 ? __ldg(a.v_scales + slot)
                                          : __ldg(a.v_scales + slot * (kv_dim / 32) + (kh * HD + lane * DPL) / 32);
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < 8; ++u)
#pragma unroll
                for (int j = 0; j < DPL; ++j) o[j] = fmaf(al[u], v[u][j], o[j]);
        }
        __syncwarp();
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
        case 0: return launch_pdl(attn_split_kernel<HD, 0>, grid, dim3(kSW * 32), 0, s, a);
        case 1: return launch_pdl(attn_split_kernel<HD, 1>, grid, dim3(kSW * 32), 0, s, a);
        case 2: return launch_pdl(attn_split_kernel<HD, 2>, grid, dim3(kSW * 32), 0, s, a);
        case 3: return launch_pdl(attn_split_kernel<HD, 3>, grid, dim3(kSW * 32), 0, s, a);
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
