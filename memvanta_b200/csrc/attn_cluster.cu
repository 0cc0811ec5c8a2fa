// attn_cluster.cu -- the model's fused decode step (F32/F16 cache) in the
// reference's order, spread over a cluster of CTAs per head.
//
// The reference's decode attention (src/llama_model.cpp:256 over
// PagedKVCache::dot_key / add_value, :23-55) for one head and token p:
//   s_t   = dot(q, k_t) / sqrt(hd)        8-lane FMA order, lanes summed in order
//   m     = max_t s_t,  e_t = exp(s_t - m),  den = sum_t e_t (double)
//   out_d = fma(e_t * float(1/den), v_t[d], out_d)  over t = 0..p in order
// The scores are independent per token and the output chains independent
// per dimension; only each chain is sequential.  So a head is a cluster of
// kCC CTAs:
//   * CTA r scores its contiguous share of the cached tokens 0..p-1 (one
//     thread per token, the K rows in its shared memory); the last CTA also
//     rotates and scores this token p;
//   * the cluster combines the per-CTA maxima through distributed shared
//     memory (st.async stores that complete bytes on the receiving CTA's
//     mbarrier: no cluster-wide fence), then in one more exchange every CTA
//     broadcasts its tokens'
//     exponentials e_t into every CTA's weight array and its double
//     denominator into every CTA (each adds them in rank order, so all hold
//     the same den and form alpha_t = e_t * float(1/den) themselves);
//   * CTA r then runs the chains of dimensions [r*hd/kCC, (r+1)*hd/kCC) over
//     all tokens in order, from the V columns of those dimensions, which it
//     staged for every token.
// Each score and each chain is computed exactly as the reference does; the
// denominator's double sum is grouped per CTA (a rounding difference there
// needs partial sums beyond 53 bits, below 2^-44 of the total).  The cache
// rows of token p are the reference's (RoPE as fma(x0,c,-(x1*s)),
// fma(x0,s,x1*c); fp16 rounded half-up).
//
// Before waiting on the q|k|v GEMV the CTAs stage everything the previous
// steps wrote: the block table, their K rows and their V columns of tokens
// 0..p-1.
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.cuh"
#include "tc.cuh"
#include "tp.cuh"

namespace mvb {

namespace cg = cooperative_groups;

__device__ int g_attn_status = 0;  // site of a cluster-attention wait that ran out (0: none)

// Adds this file's status to *status (first site wins) and clears it.
cudaError_t attn_status_take(int* status) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_attn_status, sizeof(int));
    if (e == cudaSuccess && v) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_attn_status, &zero, sizeof(int));
        if (!*status) *status = v;
    }
    return e;
}

namespace {

constexpr int kCC = 8;            // CTAs per head (a cluster)
constexpr int kCT = 128;          // threads per CTA

__device__ __forceinline__ float expf_cr(float x) { return (float)exp((double)x); }

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Remote 4- / 8-byte stores into a peer CTA's shared memory that complete
// bytes on the peer's mbarrier (no fence, no cluster barrier on the data path).
__device__ __forceinline__ uint32_t mapa_u32(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_async_b32(uint32_t raddr, uint32_t v, uint32_t rbar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(raddr), "r"(v),
                 "r"(rbar)
                 : "memory");
}
__device__ __forceinline__ void st_async_b64(uint32_t raddr, uint64_t v, uint32_t rbar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b64 [%0], %1, [%2];" ::"r"(raddr), "l"(v),
                 "r"(rbar)
                 : "memory");
}

__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// Shared-memory plan (bytes) of one CTA for a cache of max_ctx tokens.
struct ClusterPlan {
    uint64_t krow, per, vcol, k, v, w, sc, table, total;
};
__host__ __device__ inline ClusterPlan cluster_plan(uint64_t hd, uint64_t max_ctx, uint64_t max_pages, int kv_type) {
    auto up = [](uint64_t n) { return (n + 15) / 16 * 16; };
    const uint64_t es = kv_type == 0 ? 4 : 2;
    ClusterPlan p;
    p.krow = hd * es + 16;                         // padded: thread-per-row reads spread over the banks
    p.per = (max_ctx + kCC - 1) / kCC;             // cached tokens of one CTA at most
    p.vcol = hd / kCC * es;                        // bytes of this CTA's V columns per token
    p.k = 0;
    p.v = p.k + up(p.per * p.krow);
    p.w = p.v + up((max_ctx + 1) * p.vcol);        // + this token's
    p.sc = p.w + up((max_ctx + 1) * 4);            // weights of every token
    p.table = p.sc + up(p.per * 4);                // this CTA's scores / exponentials
    p.total = p.table + up(max_pages * 4);
    return p;
}

template <int HD, int KVT, bool TP>
__global__ void __launch_bounds__(kCT) attn_decode_cluster_kernel(AttnFusedArgs a) {
    constexpr int ES = KVT == 0 ? 4 : 2, SL = HD * ES, DPC = HD / kCC, half = HD / 2;
    static_assert(DPC * ES % 16 == 0, "V columns of a CTA are whole 16-byte chunks");
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ __align__(16) float qs[HD];
    __shared__ __align__(16) unsigned char knew[SL];
    __shared__ float vnew[DPC];
    __shared__ float red[kCT / 32];
    __shared__ double redd[kCT / 32];
    __shared__ float mx[kCC];
    __shared__ double dn[kCC];
    __shared__ float snew;
    __shared__ float qv[32];  // xq: the 32 outputs of one Q8 block (its first CTA)
    __shared__ __align__(8) uint64_t xbar[2];  // [0]: the maxima landed, [1]: exponentials + denominators
    __shared__ int xabort;
    cg::cluster_group cl = cg::this_cluster();
    const int r = (int)cl.block_rank(), h = blockIdx.x / kCC;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = (int)(a.n_head / a.n_head_kv), kh = h / G;
    const int D = (int)(a.n_head * HD), kv_dim = (int)(a.n_head_kv * HD);
    const int page = (int)a.page;
    const ClusterPlan P = cluster_plan(HD, a.max_ctx, a.max_pages, KVT);
    unsigned char* ks = smem + P.k;
    unsigned char* vs = smem + P.v;
    float* wt = reinterpret_cast<float*>(smem + P.w);
    float* sc = reinterpret_cast<float*>(smem + P.sc);
    int* tbl = reinterpret_cast<int*>(smem + P.table);
    const uint8_t* kp = static_cast<const uint8_t*>(a.k_pages);
    const uint8_t* vp = static_cast<const uint8_t*>(a.v_pages);
    const size_t row_bytes = (size_t)kv_dim * ES, head_off = (size_t)kh * HD * ES;
    const uint32_t xb0 = tc::smem_u32(&xbar[0]), xb1 = xb0 + 8;
    const int p = a.pos[0];  // this token; tokens 0..p-1 are cached
    if (tid == 0) {
        // the exchanges' receive barriers, armed for what every CTA will send
        xabort = 0;
        tc::mbar_init(xb0, 1);
        tc::mbar_init(xb1, 1);
        tc::mbar_fence_init();
        tc::mbar_expect_tx(xb0, kCC * 4);
        tc::mbar_expect_tx(xb1, (uint32_t)(p + 1) * 4 + kCC * 8);
    }
    // every CTA of the cluster has started (and armed its barriers) before
    // any writes another's memory
    cluster_arrive();

    pdl_trigger();
    const int npg = (p + page) / page;
    for (int i = tid; i < npg; i += kCT) tbl[i] = a.block_table[i];
    __syncthreads();
    auto slot_of = [&](int t) -> size_t { return (size_t)tbl[t / page] * page + t % page; };
    const int per = (p + kCC - 1) / kCC;
    const int t0 = min(p, r * per), t1 = min(p, t0 + per), nt = t1 - t0;
    // K rows of this CTA's tokens; V columns [r*DPC, (r+1)*DPC) of every token
    {
        constexpr int KC = SL / 16, VC = DPC * ES / 16;
        for (int c = tid; c < nt * KC; c += kCT) {
            const int i = c / KC, off = (c % KC) * 16;
            cp_async16(ks + (size_t)i * P.krow + off, kp + slot_of(t0 + i) * row_bytes + head_off + off);
        }
        for (int c = tid; c < p * VC; c += kCT) {
            const int t = c / VC, off = (c % VC) * 16;
            cp_async16(vs + (size_t)t * P.vcol + off,
                       vp + slot_of(t) * row_bytes + head_off + (size_t)r * DPC * ES + off);
        }
        cp_async_commit();
    }
    float cs = 0.0f, sn = 0.0f;
    if (tid < half) {
        cs = a.cos_t[(size_t)p * half + tid];
        sn = a.sin_t[(size_t)p * half + tid];
    }

    pdl_wait();
    const bool last = r == kCC - 1;
    {
        const float* row = a.qkv;
        for (int i = tid; i < half; i += kCT) {
            const float q0 = row[h * HD + i], q1 = row[h * HD + i + half];
            qs[i] = __fmaf_rn(q0, cs, -__fmul_rn(q1, sn));
            qs[i + half] = __fmaf_rn(q0, sn, __fmul_rn(q1, cs));
            if (last) {  // this token's key, in cache form
                const float k0 = row[D + kh * HD + i], k1 = row[D + kh * HD + i + half];
                const float r0 = __fmaf_rn(k0, cs, -__fmul_rn(k1, sn)), r1 = __fmaf_rn(k0, sn, __fmul_rn(k1, cs));
                if constexpr (KVT == 1) {
                    reinterpret_cast<uint16_t*>(knew)[i] = f32_to_f16_ref(r0);
                    reinterpret_cast<uint16_t*>(knew)[i + half] = f32_to_f16_ref(r1);
                } else {
                    reinterpret_cast<float*>(knew)[i] = r0;
                    reinterpret_cast<float*>(knew)[i + half] = r1;
                }
            }
        }
        // this token's value in cache form: this CTA's columns
        if (tid < DPC) {
            const float v = row[D + kv_dim + kh * HD + r * DPC + tid];
            if constexpr (KVT == 1) {
                const uint16_t b = f32_to_f16_ref(v);
                vnew[tid] = half_bits_to_float(b);
                if (h % G == 0)
                    reinterpret_cast<uint16_t*>(static_cast<uint8_t*>(a.v_pages) + slot_of(p) * row_bytes +
                                                head_off)[r * DPC + tid] = b;
            } else {
                vnew[tid] = v;
                if (h % G == 0)
                    reinterpret_cast<float*>(static_cast<uint8_t*>(a.v_pages) + slot_of(p) * row_bytes +
                                             head_off)[r * DPC + tid] = v;
            }
        }
    }
    cp_async_wait_all();
    __syncthreads();
    if (last && h % G == 0) {  // this token's key row, once per kv head
        uint8_t* kd = static_cast<uint8_t*>(a.k_pages) + slot_of(p) * row_bytes + head_off;
        for (int i = tid; i < SL / 4; i += kCT)
            reinterpret_cast<uint32_t*>(kd)[i] = reinterpret_cast<const uint32_t*>(knew)[i];
    }
    if (h == 0 && r == 0 && tid == 0 && a.ctx_out) a.ctx_out[0] = p + 1;

    // 1. scores (the reference's 8-lane order); the last CTA also this token's
    auto dot_row = [&](const unsigned char* krw) -> float {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if constexpr (KVT == 1) {
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
                const float kv8[8] = {u.x, u.y, u.z, u.w, v.x, v.y, v.z, v.w};
#pragma unroll
                for (int l = 0; l < 8; ++l) acc[l] = fmaf(qs[d + l], kv8[l], acc[l]);
            }
        }
        float dot = acc[0];
#pragma unroll
        for (int l = 1; l < 8; ++l) dot += acc[l];
        return dot / sqrtf((float)HD);
    };
    float m = -INFINITY;
    for (int i = tid; i < nt; i += kCT) {
        const float s = dot_row(ks + (size_t)i * P.krow);
        sc[i] = s;
        m = fmaxf(m, s);
    }
    if (last && tid == kCT - 1) {
        snew = dot_row(knew);
        m = fmaxf(m, snew);
    }
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    cluster_wait();  // the phase armed at the top: every peer has started
    if (tid == 0) {
        float cm = red[0];
#pragma unroll
        for (int w = 1; w < kCT / 32; ++w) cm = fmaxf(cm, red[w]);
        const uint32_t dst = tc::smem_u32(&mx[r]);
        for (int q = 0; q < kCC; ++q) st_async_b32(mapa_u32(dst, q), __float_as_uint(cm), mapa_u32(xb0, q));
    }
    tc::mbar_wait(xb0, 0, &xabort, &g_attn_status, 51);  // every CTA's maximum has landed
    float M = mx[0];
#pragma unroll
    for (int q = 1; q < kCC; ++q) M = fmaxf(M, mx[q]);

    // 2. exponentials into every CTA's weight array and the double denominator
    //    into every CTA (one exchange); every CTA then adds the denominators in
    //    rank order and forms alpha_t = e_t * float(1/den) itself
    double den = 0.0;
    const uint32_t wt0 = tc::smem_u32(wt);
    for (int i = tid; i < nt; i += kCT) {
        const float e = expf_cr(sc[i] - M);
        den += (double)e;
        for (int q = 0; q < kCC; ++q)
            st_async_b32(mapa_u32(wt0 + (uint32_t)(t0 + i) * 4, q), __float_as_uint(e), mapa_u32(xb1, q));
    }
    if (last && tid == kCT - 1) {
        const float enew = expf_cr(snew - M);
        den += (double)enew;
        for (int q = 0; q < kCC; ++q) st_async_b32(mapa_u32(wt0 + (uint32_t)p * 4, q), __float_as_uint(enew), mapa_u32(xb1, q));
    }
    den = warp_sum_d(den);
    if (lane == 0) redd[warp] = den;
    __syncthreads();
    if (tid == 0) {
        double cd = 0.0;
#pragma unroll
        for (int w = 0; w < kCT / 32; ++w) cd += redd[w];
        const uint32_t dst = tc::smem_u32(&dn[r]);
        for (int q = 0; q < kCC; ++q)
            st_async_b64(mapa_u32(dst, q), (uint64_t)__double_as_longlong(cd), mapa_u32(xb1, q));
    }
    tc::mbar_wait(xb1, 0, &xabort, &g_attn_status, 52);  // every exponential and denominator has landed
    double tot = 0.0;
#pragma unroll
    for (int q = 0; q < kCC; ++q) tot += dn[q];
    const float inv = (float)(1.0 / tot);

    // 4. this CTA's output dimensions: one chain per dimension over t = 0..p
    float out = 0.0f;
    if (tid < DPC) {
        auto v_at = [&](int t) -> float {
            const unsigned char* vr = vs + (size_t)t * P.vcol;
            if constexpr (KVT == 1) return half_bits_to_float(reinterpret_cast<const uint16_t*>(vr)[tid]);
            else return reinterpret_cast<const float*>(vr)[tid];
        };
        int t = 0;
        for (; t + 8 <= p; t += 8) {  // the loads of 8 tokens go out before their 8 chain steps
            float v[8], al[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                al[j] = wt[t + j] * inv;
                v[j] = v_at(t + j);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) out = fmaf(al[j], v[j], out);
        }
        for (; t < p; ++t) out = fmaf(wt[t] * inv, v_at(t), out);
        out = fmaf(wt[p] * inv, vnew[tid], out);
        const int d = r * DPC + tid;
        if constexpr (TP) ll_put_all(a.tp, a.out_shared, (uint64_t)(a.head_off + h) * HD + d, out,
                                     tp_uepoch(a.tp, a.out_point));
        else a.out[(size_t)h * HD + d] = out;
    }
    // 5. one GPU, xq: the o projection's input quantised here (as the GEMV's
    // own prologue would: d = max|v|/127, q = clamp(round(v/d))), the 32
    // outputs of a block gathered in the first of its CTAs
    if constexpr (!TP) {
        if (a.xq) {
            constexpr int CPB = 32 / DPC;  // CTAs per Q8 block
            if (tid < DPC) cl.map_shared_rank(qv, r - r % CPB)[(r % CPB) * DPC + tid] = out;
            cluster_arrive();
            cluster_wait();
            if (r % CPB == 0 && warp == 0) {
                const float v = qv[lane];
                const float mxa = warp_max(fabsf(v));
                const float d = mxa > 0.0f ? mxa / 127.0f : 1.0f;
                const float id = 1.0f / d;
                const int q = (int)fminf(fmaxf(roundf(v * id), -127.0f), 127.0f);
                const int qsum = warp_sum_i(q);
                uint32_t word = (uint32_t)(q & 0xff);
#pragma unroll
                for (int k = 1; k < 4; ++k) word |= (uint32_t)(__shfl_down_sync(0xffffffffu, q, k) & 0xff) << (8 * k);
                const int b = (h * HD + r * DPC) / 32, nbo = (int)(a.n_head * HD / 32);
                uint8_t* base = static_cast<uint8_t*>(a.xq);
                if ((lane & 3) == 0)
                    *reinterpret_cast<uint32_t*>(base + (size_t)(lane < 16 ? b : nbo + b) * 16 + (lane & 15)) = word;
                if (lane == 0)
                    reinterpret_cast<float2*>(base + (size_t)nbo * 32)[b] = make_float2(d, __int_as_float(8 * qsum));
            }
        }
    }
}

template <int HD, int KVT>
cudaError_t launch_cluster(const AttnFusedArgs& a, size_t smem, cudaStream_t s) {
    const dim3 grid((unsigned)(a.n_head * kCC)), block(kCT);
    if (a.tp.world > 1) {
        ensure_smem_attr(attn_decode_cluster_kernel<HD, KVT, true>, 200 * 1024);
        return launch_pdl_cluster(attn_decode_cluster_kernel<HD, KVT, true>, grid, block, smem, s, kCC, a);
    }
    ensure_smem_attr(attn_decode_cluster_kernel<HD, KVT, false>, 200 * 1024);
    return launch_pdl_cluster(attn_decode_cluster_kernel<HD, KVT, false>, grid, block, smem, s, kCC, a);
}

}  // namespace

uint64_t attn_cluster_smem_bytes(uint64_t hd, uint64_t max_ctx, uint64_t max_pages, int kv_type) {
    if ((kv_type != 0 && kv_type != 1) || (hd != 64 && hd != 128 && hd != 256)) return 0;
    return cluster_plan(hd, max_ctx, max_pages, kv_type).total;
}

cudaError_t attn_decode_cluster(const AttnFusedArgs& a, cudaStream_t s) {
    if (a.kv_type != 0 && a.kv_type != 1) return cudaErrorInvalidValue;
    if (a.n_head % a.n_head_kv) return cudaErrorInvalidValue;
    const uint64_t smem = attn_cluster_smem_bytes(a.hd, a.max_ctx, a.max_pages, a.kv_type);
    if (!smem || smem > 200 * 1024) return cudaErrorInvalidValue;
    const bool f16 = a.kv_type == 1;
    switch (a.hd) {
        case 64: return f16 ? launch_cluster<64, 1>(a, smem, s) : launch_cluster<64, 0>(a, smem, s);
        case 128: return f16 ? launch_cluster<128, 1>(a, smem, s) : launch_cluster<128, 0>(a, smem, s);
        case 256: return f16 ? launch_cluster<256, 1>(a, smem, s) : launch_cluster<256, 0>(a, smem, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace mvb
