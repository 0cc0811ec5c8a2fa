// attn_split.cu -- one-query paged attention split over the context: for
// many sequences (ragged contexts, scattered pages;
// attn_split_kernel) and, opt-in, for the model's decode step with RoPE and
// the KV append fused in (attn_fused_split_kernel, MV_ATTN_SPLIT=1).
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
// copies spread over the lanes, one stage in flight while one is used), so
// no warp waits for another before the merge.  Two stages keep a CTA at
// ~70 KB (F16, hd 128): three CTAs share an SM, which measured faster than
// deeper rings at two CTAs per SM (config 4 F16: 96.5 against 121.8 us).  Scores: two lanes per token,
// each over half of the head's dimensions; values: lane = hd/32 consecutive
// dimensions.  One CTA per (sequence, head), 4 warps.
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.cuh"
#include "tp.cuh"

namespace mvb {

namespace cg = cooperative_groups;

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

// Shared-memory plan of one warp's ring: S stages of kTok tokens' key and
// value head slices (rows padded by 16 bytes) plus their scales (Q8: one per
// token, Q8_0: hd/32 per token).
template <int HD, int KVT, int S_>
struct SplitPlan {
    static constexpr int ES = KVT == 0 ? 4 : KVT == 1 ? 2 : 1;
    static constexpr int SL = HD * ES;        // bytes of one head slice
    static constexpr int SLP = SL + 16;       // padded row
    static constexpr int NSC = KVT == 2 ? 1 : KVT == 3 ? HD / 32 : 0;  // scales per token
    static constexpr int S = S_;                                       // ring stages
    static constexpr int STAGE = 2 * kTok * SLP + 2 * kTok * NSC * 4;
    static constexpr int WARP = S * STAGE;
};

// Where one head's cached rows live.
struct KvSrc {
    const uint8_t* kp;
    const uint8_t* vp;
    const float* ksc;
    const float* vsc;
    size_t row_bytes, head_off;
    int kv_dim, kh, page;
};

// Stage g of a warp's tokens [t0, t1) into ring slot g % S: kTok tokens' key
// and value slices (16-byte copies spread over the lanes) and their scales.
// Always commits one cp.async group (empty past the last stage).
template <class P, int KVT>
__device__ __forceinline__ void stage_issue(unsigned char* ring, int g, int ng, int t0, int t1, const int* tbl,
                                            const KvSrc& src, int lane) {
    if (g < ng) {
        unsigned char* base = ring + (g % P::S) * P::STAGE;
        constexpr int CPT = P::SL / 16;  // 16-byte chunks per slice
        const int tb = t0 + g * kTok;
        // lane u < kTok: the cache slot of token tb + u, once per stage
        const int tu = tb + (lane & (kTok - 1));
        const size_t myslot = tu < t1 ? (size_t)tbl[tu / src.page] * src.page + tu % src.page : 0;
#pragma unroll
        for (int i = 0; i < 2 * kTok * CPT / 32; ++i) {
            const int c = lane + 32 * i;  // chunk: (K|V, token u, 16-byte offset)
            const int kv = c / (kTok * CPT), rem = c % (kTok * CPT), u = rem / CPT, off = (rem % CPT) * 16;
            const size_t su = __shfl_sync(0xffffffffu, myslot, u);
            if (tb + u < t1)
                cp_async16(base + (kv * kTok + u) * P::SLP + off,
                           (kv ? src.vp : src.kp) + su * src.row_bytes + src.head_off + off);
        }
        if constexpr (P::NSC > 0) {
            const int u = lane & 15, kv = lane >> 4, t = tb + u;
            if (t < t1) {
                const float* sp = (kv ? src.vsc : src.ksc) +
                                  (KVT == 2 ? myslot : myslot * (src.kv_dim / 32) + src.kh * P::NSC);
                float* dst = reinterpret_cast<float*>(base + 2 * kTok * P::SLP) + (kv * kTok + u) * P::NSC;
#pragma unroll
                for (int i = 0; i < P::NSC; ++i) cp_async4(dst + i, sp + i);
            }
        }
    }
    cp_async_commit();
}

// One warp's running softmax state over its tokens (max m, double
// denominator, unnormalised output: lane = HD/32 consecutive dimensions).
template <int HD, int KVT>
struct WarpSoftmax {
    static constexpr int DPL = HD / 32;
    float m = -INFINITY;
    double den = 0.0;
    float o[DPL];
    __device__ __forceinline__ WarpSoftmax() {
#pragma unroll
        for (int j = 0; j < DPL; ++j) o[j] = 0.0f;
    }

    // Folds in the n (<= kTok) tokens of a landed stage.
    template <class P>
    __device__ __forceinline__ void consume(const unsigned char* base, int n, const float* qs, int lane) {
        constexpr int ES = P::ES, SL = P::SL, SLP = P::SLP, NSC = P::NSC;
        const float* ksc = reinterpret_cast<const float*>(base + 2 * kTok * SLP);
        const float* vsc = ksc + kTok * NSC;
        const int u = lane & 15, half = lane >> 4;  // scores: token u of the stage, half of its dimensions
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
        const float sc = u < n ? dot / sqrtf((float)HD) : -INFINITY;
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
    }

    // Streams tokens [t0, t1) through this warp's ring (the first S-1 stages
    // were issued by the caller with stage_issue).
    template <class P>
    __device__ __forceinline__ void run(unsigned char* ring, int t0, int t1, const int* tbl, const KvSrc& src,
                                        const float* qs, int lane) {
        const int ng = (t1 - t0 + kTok - 1) / kTok;
        for (int g = 0; g < ng; ++g) {
            stage_issue<P, KVT>(ring, g + P::S - 1, ng, t0, t1, tbl, src, lane);  // the slot stage g-1 used
            cp_async_wait<P::S - 1>();  // this lane's copies of stage g have landed
            __syncwarp();               // ... and every lane's
            consume<P>(ring + (g % P::S) * P::STAGE, min(kTok, t1 - (t0 + g * kTok)), qs, lane);
            __syncwarp();  // every lane is done with this slot before it is refilled
        }
        cp_async_wait<0>();
    }
};

template <int HD, int KVT>
using SplitPlanOf = SplitPlan<HD, KVT, 2>;  // two stages: three CTAs fit an SM

template <int HD, int KVT>
__global__ void __launch_bounds__(kSW * 32) attn_split_kernel(AttnArgs a) {
    using P = SplitPlanOf<HD, KVT>;
    constexpr int DPL = HD / 32;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ __align__(16) float qs[HD];
    __shared__ float mw[kSW];
    __shared__ double dw[kSW];
    __shared__ float ow[kSW][HD];
    const int s = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = (int)(a.n_head / a.n_head_kv), kh = h / G;
    const int kv_dim = (int)(a.n_head_kv * HD);
    const KvSrc src{static_cast<const uint8_t*>(a.k_pages), static_cast<const uint8_t*>(a.v_pages), a.k_scales,
                    a.v_scales, (size_t)kv_dim * P::ES, (size_t)kh * HD * P::ES, kv_dim, kh, (int)a.page};
    int* tbl = reinterpret_cast<int*>(smem + kSW * P::WARP);
    unsigned char* ring = smem + warp * P::WARP;
    const int ctx = a.ctx_len[s];
    const int npg = (ctx + src.page - 1) / src.page;
    const int32_t* trow = a.block_table + (a.one_seq ? 0 : (size_t)s) * a.max_pages;
    for (int i = tid; i < npg; i += kSW * 32) tbl[i] = trow[i];
    for (int i = tid; i < HD; i += kSW * 32) qs[i] = a.q[(size_t)s * a.q_stride + (size_t)h * HD + i];
    __syncthreads();
    // this warp's tokens: a contiguous quarter of the context, in stages of kTok
    const int per = (ctx + kSW - 1) / kSW;
    const int t0 = min(ctx, warp * per), t1 = min(ctx, t0 + per);
    const int ng = (t1 - t0 + kTok - 1) / kTok;
#pragma unroll
    for (int k = 0; k < P::S - 1; ++k) stage_issue<P, KVT>(ring, k, ng, t0, t1, tbl, src, lane);
    WarpSoftmax<HD, KVT> st;
    st.template run<P>(ring, t0, t1, tbl, src, qs, lane);
    // merge the warps' states in warp order
    if (lane == 0) {
        mw[warp] = st.m;
        dw[warp] = st.den;
    }
#pragma unroll
    for (int j = 0; j < DPL; ++j) ow[warp][lane * DPL + j] = st.o[j];
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

// ------------------------------------------------ fused decode (one sequence)
// One decode token of the model (F32/F16 cache): RoPE of the query and key
// heads, the append of this token's K and V to the paged cache, and the
// attention over tokens 0..p split over the context.  The rotation and the
// cache rows are the exact ones of the reference (half-split RoPE as
// fma(x0,c,-(x1*s)), fma(x0,s,x1*c); fp16 rounded half-up); the attention
// merges partial softmax states as attn_split_kernel does.
//
// A head is a cluster of kFC CTAs of kSW warps: the kFC*kSW warps each own a
// contiguous share of the cached tokens 0..p-1 and stream it through their own
// ring (kFS stages, small enough that a CTA fits the slot the q|k|v GEMV
// leaves free, so the first stage of every warp is in flight before the GEMV
// finishes).  Each warp's state goes to rank 0's shared memory (DSMEM), which
// merges them in warp order and adds this token (score from the stored k,
// value from the stored v) last.
constexpr int kFC = 2;  // CTAs per head
constexpr int kFS = 2;  // ring stages per warp

template <int HD, int KVT>
using FusedPlan = SplitPlan<HD, KVT, kFS>;

template <int HD, int KVT, bool TP>
__global__ void __launch_bounds__(kSW * 32) attn_fused_split_kernel(AttnFusedArgs a) {
    using P = FusedPlan<HD, KVT>;
    constexpr int DPL = HD / 32, NW = kFC * kSW, NT = kSW * 32, half = HD / 2;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ __align__(16) float qs[HD];
    __shared__ __align__(16) unsigned char knew[P::SL];  // this token's k and v in cache form
    __shared__ __align__(16) unsigned char vnew[P::SL];
    __shared__ float mw[NW];
    __shared__ double dw[NW];
    __shared__ float snew;
    __shared__ __align__(16) float ow[NW][HD];  // rank 0's copy receives every warp's output
    cg::cluster_group cl = cg::this_cluster();
    const int rank = (int)cl.block_rank(), h = blockIdx.x / kFC;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = (int)(a.n_head / a.n_head_kv), kh = h / G;
    const int D = (int)(a.n_head * HD), kv_dim = (int)(a.n_head_kv * HD);
    const KvSrc src{static_cast<const uint8_t*>(a.k_pages), static_cast<const uint8_t*>(a.v_pages), nullptr, nullptr,
                    (size_t)kv_dim * P::ES, (size_t)kh * HD * P::ES, kv_dim, kh, (int)a.page};
    int* tbl = reinterpret_cast<int*>(smem + kSW * P::WARP);
    unsigned char* ring = smem + warp * P::WARP;
    // every CTA of the cluster has started before any writes another's memory
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

    pdl_trigger();
    // before the wait: only what earlier steps wrote (the position, the block
    // table, the cached rows of tokens 0..p-1) and the immutable tables
    const int p = a.pos[0];
    const int npg = (p + src.page) / src.page;  // pages of tokens 0..p
    for (int i = tid; i < npg; i += NT) tbl[i] = a.block_table[i];
    __syncthreads();
    const int gw = rank * kSW + warp;
    const int per = (p + NW - 1) / NW;
    const int t0 = min(p, gw * per), t1 = min(p, t0 + per);
    const int ng = (t1 - t0 + kTok - 1) / kTok;
#pragma unroll
    for (int k = 0; k < P::S - 1; ++k) stage_issue<P, KVT>(ring, k, ng, t0, t1, tbl, src, lane);
    float cs[(half + NT - 1) / NT], sn[(half + NT - 1) / NT];
#pragma unroll
    for (int j = 0; j < (half + NT - 1) / NT; ++j) {
        const int i = tid + j * NT;
        cs[j] = i < half ? a.cos_t[(size_t)p * half + i] : 0.0f;
        sn[j] = i < half ? a.sin_t[(size_t)p * half + i] : 0.0f;
    }

    pdl_wait();
    {
        const float* row = a.qkv;
#pragma unroll
        for (int j = 0; j < (half + NT - 1) / NT; ++j) {
            const int i = tid + j * NT;
            if (i < half) {
                const float c = cs[j], s = sn[j];
                const float q0 = row[h * HD + i], q1 = row[h * HD + i + half];
                qs[i] = __fmaf_rn(q0, c, -__fmul_rn(q1, s));
                qs[i + half] = __fmaf_rn(q0, s, __fmul_rn(q1, c));
                if (rank == 0) {
                    const float k0 = row[D + kh * HD + i], k1 = row[D + kh * HD + i + half];
                    const float r0 = __fmaf_rn(k0, c, -__fmul_rn(k1, s)), r1 = __fmaf_rn(k0, s, __fmul_rn(k1, c));
                    if constexpr (KVT == 1) {
                        reinterpret_cast<uint16_t*>(knew)[i] = f32_to_f16_ref(r0);
                        reinterpret_cast<uint16_t*>(knew)[i + half] = f32_to_f16_ref(r1);
                    } else {
                        reinterpret_cast<float*>(knew)[i] = r0;
                        reinterpret_cast<float*>(knew)[i + half] = r1;
                    }
                }
            }
        }
        if (rank == 0) {
            for (int i = tid; i < HD; i += NT) {
                const float v = row[D + kv_dim + kh * HD + i];
                if constexpr (KVT == 1) reinterpret_cast<uint16_t*>(vnew)[i] = f32_to_f16_ref(v);
                else reinterpret_cast<float*>(vnew)[i] = v;
            }
        }
    }
    __syncthreads();
    if (rank == 0) {
        if (h % G == 0) {  // the cache rows of this token, once per kv head
            const size_t at = ((size_t)tbl[p / src.page] * src.page + p % src.page) * src.row_bytes + src.head_off;
            uint8_t* kd = static_cast<uint8_t*>(a.k_pages) + at;
            uint8_t* vd = static_cast<uint8_t*>(a.v_pages) + at;
            for (int i = tid; i < P::SL / 4; i += NT) {
                reinterpret_cast<uint32_t*>(kd)[i] = reinterpret_cast<const uint32_t*>(knew)[i];
                reinterpret_cast<uint32_t*>(vd)[i] = reinterpret_cast<const uint32_t*>(vnew)[i];
            }
        }
        if (h == 0 && tid == 0 && a.ctx_out) a.ctx_out[0] = p + 1;
        if (warp == 0) {  // this token's score
            float part = 0.0f;
#pragma unroll
            for (int j = 0; j < DPL; ++j) {
                const int d = lane * DPL + j;
                const float k = KVT == 1 ? half_bits_to_float(reinterpret_cast<const uint16_t*>(knew)[d])
                                         : reinterpret_cast<const float*>(knew)[d];
                part = fmaf(qs[d], k, part);
            }
            part = warp_sum(part);
            if (lane == 0) snew = part / sqrtf((float)HD);
        }
    }
    WarpSoftmax<HD, KVT> st;
    st.template run<P>(ring, t0, t1, tbl, src, qs, lane);
    // every warp's state into rank 0's memory, then rank 0 merges
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
    float* ow0 = cl.map_shared_rank(&ow[0][0], 0);
    if (lane == 0) {
        cl.map_shared_rank(mw, 0)[gw] = st.m;
        cl.map_shared_rank(dw, 0)[gw] = st.den;
    }
#pragma unroll
    for (int j = 0; j < DPL; ++j) ow0[gw * HD + lane * DPL + j] = st.o[j];
    cl.sync();
    if (rank != 0) return;
    float M = snew;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, mw[w]);
    float cw[NW];
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        cw[w] = mw[w] == -INFINITY ? 0.0f : expf_cr(mw[w] - M);
        tot += dw[w] * (double)cw[w];
    }
    const float cn = expf_cr(snew - M);
    tot += (double)cn;
    const float inv = (float)(1.0 / tot);
    for (int d = tid; d < HD; d += NT) {
        float acc = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; ++w) acc = fmaf(ow[w][d], cw[w], acc);
        const float v = KVT == 1 ? half_bits_to_float(reinterpret_cast<const uint16_t*>(vnew)[d])
                                 : reinterpret_cast<const float*>(vnew)[d];
        acc = fmaf(v, cn, acc);
        if constexpr (TP) ll_put_all(a.tp, a.out_shared, (uint64_t)(a.head_off + h) * HD + d, acc * inv,
                                     tp_uepoch(a.tp, a.out_point));
        else a.out[(size_t)h * HD + d] = acc * inv;
    }
}

template <int HD, int KVT>
size_t split_smem(const AttnArgs& a) {
    return (size_t)kSW * SplitPlanOf<HD, KVT>::WARP + ((a.max_ctx + a.page - 1) / a.page) * 4;
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

template <int HD, int KVT>
size_t fused_split_smem(uint64_t max_pages) {
    return (size_t)kSW * FusedPlan<HD, KVT>::WARP + max_pages * 4;
}

template <int HD, int KVT>
cudaError_t launch_fused_split(const AttnFusedArgs& a, cudaStream_t s) {
    const size_t smem = fused_split_smem<HD, KVT>(a.max_pages);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    const dim3 grid((unsigned)(a.n_head * kFC)), block(kSW * 32);
    if (a.tp.world > 1) {
        ensure_smem_attr(attn_fused_split_kernel<HD, KVT, true>, 200 * 1024);
        return launch_pdl_cluster(attn_fused_split_kernel<HD, KVT, true>, grid, block, smem, s, kFC, a);
    }
    ensure_smem_attr(attn_fused_split_kernel<HD, KVT, false>, 200 * 1024);
    return launch_pdl_cluster(attn_fused_split_kernel<HD, KVT, false>, grid, block, smem, s, kFC, a);
}

template <int HD>
cudaError_t launch_fused_split_hd(const AttnFusedArgs& a, cudaStream_t s) {
    return a.kv_type == 1 ? launch_fused_split<HD, 1>(a, s) : launch_fused_split<HD, 0>(a, s);
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

uint64_t attn_fused_split_smem_bytes(uint64_t hd, uint64_t max_pages, int kv_type) {
    if (kv_type != 0 && kv_type != 1) return 0;
    const bool f16 = kv_type == 1;
    switch (hd) {
        case 64: return f16 ? fused_split_smem<64, 1>(max_pages) : fused_split_smem<64, 0>(max_pages);
        case 128: return f16 ? fused_split_smem<128, 1>(max_pages) : fused_split_smem<128, 0>(max_pages);
        case 256: return f16 ? fused_split_smem<256, 1>(max_pages) : fused_split_smem<256, 0>(max_pages);
        default: return 0;
    }
}

cudaError_t attn_decode_fused_split(const AttnFusedArgs& a, cudaStream_t s) {
    if (a.kv_type != 0 && a.kv_type != 1) return cudaErrorInvalidValue;
    if (a.n_head % a.n_head_kv) return cudaErrorInvalidValue;
    switch (a.hd) {
        case 64: return launch_fused_split_hd<64>(a, s);
        case 128: return launch_fused_split_hd<128>(a, s);
        case 256: return launch_fused_split_hd<256>(a, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace mvb
