// gemv_q4.cu -- decode GEMV y = W x for a Q4_0 weight with Q8 activations,
// bit-exact with the reference's decode path (tensor_matvec Q4_0 branch,
// src/gguf_kernels.cpp:246 -> quantize_q8 :161-172 -> dot_q4_q8 :189 ->
// dot_q4_q8_block :180-188).
//
// Exactness.  The reference accumulates a row as a sequential chain over the
// 32-element blocks, b = 0, 1, ..., nb-1:
//     sum = fma(fp16(d_w[b]) * d_a[b], float(isum[b]), sum)
// (its multi-threaded build; GCC contracts the update into one FMA).  Here
// the lanes of a warp compute the per-block terms (t_b = d_w*d_a, isum_b) in
// parallel -- isum with dp4a, bit-exact -- write them to shared memory, and
// one lane per row then runs the same FMA chain in block order.  Rows come
// out identical to the reference's to the last bit, so the Q8 quantisation of
// the next layer's input sees exactly the reference's values.
//
// Bandwidth.  HBM-bound: each weight byte is read once, staged through a
// per-warp shared-memory ring by 16-byte cp.async copies (one nibble payload
// per lane per block; the fp16 scales 8 per copy), several items deep so
// about 110 KB per SM are in flight.  A warp owns RPW rows at a time; the
// ring's first items are requested before the activation prologue (and
// before waiting on the previous kernel), hiding both under the weight fetch.
//
// Prologue (every CTA): optional RMSNorm (double sum of squares,
// src/llama_model.cpp:237) and the per-32 Q8 quantisation of x into shared
// memory, one vectorised pass: a thread owns 8 consecutive elements, four
// neighbouring lanes make one 32-element block.
//
// Block dot: element i<16 is the low nibble of payload byte i, element 16+i
// the high nibble, so with the payload as four words w,
//   sum (nib-8)*a = sum dp4a(w & 0x0F0F0F0F, a_lo) + dp4a((w>>4) & 0x0F0F0F0F, a_hi)
//                   - 8*sum(a)
// (nibbles 0..15 are non-negative bytes for the signed dp4a).
#include <cooperative_groups.h>

#include <map>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"
#include "tc.cuh"
#include "tp.cuh"

namespace cg = cooperative_groups;

namespace mvb {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kCbStride = 34;    // float2 per chain-buffer row (16-byte aligned, conflict-free)
constexpr uint32_t kLoNib = 0x0F0F0F0Fu;

// dp4a with unsigned bytes in a, signed bytes in b
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// sum_k (nib_k - 8) * a_k of one block: low nibbles against elements 0..15,
// the high nibbles kept in place (16 x nib, bytes up to 240, an unsigned dot)
// against elements 16..31 and shifted back, minus c8 = 8 * sum(a).
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

struct Act {
    int4* lo;    // [nb] elements 0..15 of each block
    int4* hi;    // [nb] elements 16..31
    float2* dc;  // [nb] (d_a, 8*sum(q) as int bits)
    float2* cb;  // [kWarps][RPW][kCbStride] chain buffers
};

__device__ __forceinline__ Act act_smem(int nb) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Act a;
    a.lo = reinterpret_cast<int4*>(smem_raw);
    a.hi = a.lo + nb;
    a.dc = reinterpret_cast<float2*>(a.hi + nb);
    a.cb = a.dc + ((nb + 1) & ~1);
    return a;
}

size_t act_smem_bytes(uint64_t nb, int rpw) {
    return nb * 32 + ((nb + 1) & ~1ull) * 8 + (size_t)kWarps * rpw * kCbStride * 8;
}

// Double-precision block reduction (all threads); result broadcast.
__device__ __forceinline__ double block_sum_d(double v) {
    __shared__ double red[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum_d(v);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        double t = lane < nw ? red[lane] : 0.0;
        t = warp_sum_d(t);
        if (lane == 0) red[0] = t;
    }
    __syncthreads();
    const double r = red[0];
    __syncthreads();
    return r;
}

// Where a quantised group goes: this CTA's shared memory.
struct LocalSink {
    const Act& a;
    __device__ __forceinline__ void put(int b, int sub, uint2 pk, bool first, float2 dc) const {
        *(reinterpret_cast<uint2*>(sub < 2 ? &a.lo[b] : &a.hi[b]) + (sub & 1)) = pk;
        if (first) a.dc[b] = dc;
    }
};

// One 8-element group of the quantisation: 4 neighbouring lanes hold one
// 32-element block.  All 32 lanes of the warp must call it (shuffles).
// n0/n1: the group's RMSNorm weights (used when rms).
template <class Sink = LocalSink>
__device__ __forceinline__ void quant_group(int g, bool active, float4 u, float4 w, float4 n0, float4 n1, bool rms,
                                            float inv, const Sink& out) {
    float v[8] = {u.x, u.y, u.z, u.w, w.x, w.y, w.z, w.w};
    if (active && rms) {
        const float nw[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = v[i] * inv * nw[i];  // (x*inv)*w as the reference
    }
    if (!active) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.0f;
    }
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(v[i]));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    const float d = m > 0.0f ? m / 127.0f : 1.0f;  // quantize_q8: d = mx/127, inv = 1/d
    const float id = 1.0f / d;
    uint32_t pk[2] = {0u, 0u};
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int q = (int)fminf(fmaxf(roundf(v[i] * id), -127.0f), 127.0f);  // lround: half away from 0
        sum += q;
        pk[i >> 2] |= (uint32_t)(q & 0xff) << (8 * (i & 3));
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if (active) out.put(g >> 2, g & 3, make_uint2(pk[0], pk[1]), (g & 3) == 0, make_float2(d, __int_as_float(8 * sum)));
}

// Group loaders: 8 consecutive elements of x, from a float vector or (tensor
// parallel decode) from an LL buffer once they carry the expected epoch.
struct XFloat {
    const float4* x4;
    __device__ __forceinline__ void operator()(int g, float4& lo, float4& hi) const {
        lo = x4[2 * g];
        hi = x4[2 * g + 1];
    }
};
struct XLL {
    const TpCtx& tp;
    const uint2* x;
    unsigned ep;
    int site;
    __device__ __forceinline__ void operator()(int g, float4& lo, float4& hi) const {
        ll_load8(tp, x + 8 * g, ep, site, lo, hi);
    }
};

// Quantised activations of (optionally RMS-normalised) x into shared memory.
// A thread owns groups g = tid, tid + blockDim, ...  The prologue sits on the
// critical path between two kernels, so every load is issued at once: the
// first KEEP groups of x go to registers together (KEEP = 2 covers K = 4096,
// 6 covers K up to 12288 at 256 threads), and the RMSNorm weights of the
// first kNormKeep groups are fetched before the kernel waits on its
// predecessor (norm_preload).
constexpr int kNormKeep = 2;

struct NormPre {
    float4 w[kNormKeep][2];
};

__device__ __forceinline__ void norm_preload(NormPre& np, const float* __restrict__ norm_w, bool rms, int nb) {
    const int G = nb * 4, tid = (int)threadIdx.x, bd = (int)blockDim.x;
#pragma unroll
    for (int it = 0; it < kNormKeep; ++it) {
        const int g = tid + it * bd;
        np.w[it][0] = np.w[it][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (rms && g < G) {
            np.w[it][0] = reinterpret_cast<const float4*>(norm_w)[2 * g];
            np.w[it][1] = reinterpret_cast<const float4*>(norm_w)[2 * g + 1];
        }
    }
}

template <int KEEP, class Ld>
__device__ __forceinline__ void prologue(const Ld& ld, const NormPre& np, const float* __restrict__ norm_w, float eps,
                                         bool rms, int nb, const Act& a) {
    constexpr int kKeep = KEEP;
    const int G = nb * 4;  // groups of 8 elements
    const int bd = (int)blockDim.x, tid = (int)threadIdx.x;
    const int iters = (G + bd - 1) / bd;
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 keep[kKeep][2];
#pragma unroll
    for (int it = 0; it < kKeep; ++it) {
        const int g = tid + it * bd;
        keep[it][0] = keep[it][1] = z;
        if (g < G) ld(g, keep[it][0], keep[it][1]);
    }
    auto norm_of = [&](int it, int g, float4& n0, float4& n1) {
        n0 = n1 = z;
        if (!rms || g >= G) return;
        if (it < kNormKeep) {
            n0 = np.w[it < kNormKeep ? it : 0][0];
            n1 = np.w[it < kNormKeep ? it : 0][1];
        } else {
            n0 = reinterpret_cast<const float4*>(norm_w)[2 * g];
            n1 = reinterpret_cast<const float4*>(norm_w)[2 * g + 1];
        }
    };
    float inv = 1.0f;
    if (rms) {
        double ss = 0.0;
        auto acc = [&](float4 u, float4 v) {
            ss += (double)u.x * u.x + (double)u.y * u.y + (double)u.z * u.z + (double)u.w * u.w;
            ss += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
        };
#pragma unroll
        for (int it = 0; it < kKeep; ++it) acc(keep[it][0], keep[it][1]);
        for (int g = tid + kKeep * bd; g < G; g += bd) {
            float4 u, v;
            ld(g, u, v);
            acc(u, v);
        }
        const double tot = block_sum_d(ss);
        inv = 1.0f / sqrtf((float)(tot / (double)(nb * 32)) + eps);
    }
#pragma unroll
    for (int it = 0; it < kKeep; ++it) {
        if (it < iters) {  // uniform across the CTA
            const int g = tid + it * bd;
            float4 n0, n1;
            norm_of(it, g, n0, n1);
            quant_group(g, g < G, keep[it][0], keep[it][1], n0, n1, rms, inv, LocalSink{a});
        }
    }
    for (int it = kKeep; it < iters; ++it) {
        const int g = tid + it * bd;
        const bool active = g < G;  // uniform over the 4 lanes of a block
        float4 u = z, w = z, n0, n1;
        if (active) ld(g, u, w);
        norm_of(it, g, n0, n1);
        quant_group(g, active, u, w, n0, n1, rms, inv, LocalSink{a});
    }
    __syncthreads();
}

// Correctly rounded expf through double precision, the closest portable
// match to the host libm's expf the reference calls.
__device__ __forceinline__ float expf_cr(float x) { return (float)exp((double)x); }

// ---------------------------------------------------------- staging ring
// Each warp streams its rows through a ring of S shared-memory stages filled
// by cp.async (16-byte asynchronous copies, completion tracked per thread by
// commit/wait groups -- no software spin).  One stage holds one work item:
// RPW rows x 32 blocks of payload (16 B per block, lane-contiguous) followed
// by the same blocks' fp16 scales.  S-1 items are in flight while one is
// consumed: about 7 KB per warp, 110 KB per SM with 16 warps.
template <int RPW>
struct Ring {
    static constexpr int S = 16 / RPW;
    static constexpr int PAY = RPW * 32 * 16;
    static constexpr int STAGE = PAY + RPW * 64;
    static constexpr int BYTES = S * STAGE;  // 9216 per warp
};

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Copies work item (row group rg, chunk c) into a stage.  Lane l copies block
// c*32+l of every row; lanes 0..3 copy the chunk's 32 scales (8 per copy --
// the d plane's rows are padded to a multiple of 8, so these are aligned and
// stay inside the row).
template <int RPW>
__device__ __forceinline__ void issue_item(uint8_t* st, const uint4* __restrict__ qs,
                                           const unsigned short* __restrict__ dsc, int rows, int nb, int dstride,
                                           int rg, int c, int lane) {
    const int b = c * 32 + lane;
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
        const int r = rg * RPW + j;
        if (r < rows) {
            if (b < nb) cp_async16(st + (j * 32 + lane) * 16, qs + (size_t)r * nb + b);
            if (lane < 4 && c * 32 + lane * 8 < nb)
                cp_async16(st + Ring<RPW>::PAY + j * 64 + lane * 16, dsc + (size_t)r * dstride + c * 32 + lane * 8);
        }
    }
}

// Per-block terms of one item, then each row's FMA chain over them in block
// order.  `sum` is live in lanes 0..RPW-1 (lane j = row j of the group).
template <int RPW>
__device__ __forceinline__ void consume_item(const uint8_t* st, const Act& a, float2* cb, int nb, int c, int lane,
                                             float& sum) {
    const int b = c * 32 + lane;
    if (b < nb) {
        const int4 alo = a.lo[b], ahi = a.hi[b];
        const float2 dc = a.dc[b];
        const uint4* pay = reinterpret_cast<const uint4*>(st);
        const unsigned short* dw = reinterpret_cast<const unsigned short*>(st + Ring<RPW>::PAY);
#pragma unroll
        for (int j = 0; j < RPW; ++j) {
            const int isum = block_isum(pay[j * 32 + lane], alo, ahi, __float_as_int(dc.y));
            cb[j * kCbStride + lane] = make_float2(half_bits_to_float(dw[j * 32 + lane]) * dc.x, (float)isum);
        }
    }
    __syncwarp();
    if (lane < RPW) {
        const float2* row = cb + lane * kCbStride;
        const int n = min(32, nb - c * 32);
        if (n == 32) {
#pragma unroll
            for (int k = 0; k < 32; k += 2) {
                const float4 t = *reinterpret_cast<const float4*>(row + k);
                sum = fmaf(t.x, t.y, sum);
                sum = fmaf(t.z, t.w, sum);
            }
        } else {
            for (int k = 0; k < n; ++k) sum = fmaf(row[k].x, row[k].y, sum);
        }
    }
    __syncwarp();
}

// Output placement: y[idx] locally (y != nullptr), or, tensor parallel with
// y == nullptr (LL kernels only), element y_row_off + idx of the replicated
// LL buffer at byte offset `shared` of every rank's block, tagged with epoch
// ep.  AddTo reads the residual from this rank's own copy (its own rows:
// written by this rank).
template <bool LL>
struct YOut {
    float* y;
    const TpCtx& tp;
    uint64_t shared;
    int row_off;
    unsigned ep;      // epoch the outputs carry
    unsigned res_ep;  // AddTo: epoch the residual (this rank's rows) must carry
    bool replicated;
    __device__ __forceinline__ float local(int idx) const {
        if constexpr (LL) {
            if (replicated) {
                const uint2* own = reinterpret_cast<const uint2*>(tp_base(tp, tp.rank) + shared);
                return ll_load1(tp, own + row_off + idx, res_ep, 200);
            }
        }
        return y[idx];
    }
    __device__ __forceinline__ void put(int idx, float v) const {
        if constexpr (LL) {
            if (replicated) {
                ll_put_all(tp, shared, (uint64_t)(row_off + idx), v, ep);
                return;
            }
        }
        y[idx] = v;
    }
};

template <int RPW, bool LL>
__device__ __forceinline__ void epilogue(int epi, int rg, int rows, int lane, float sum, const YOut<LL>& yo) {
    if (epi == (int)Q4Epi::SiluGate) {
        // rows come in (gate_i, up_i) pairs: ff_i = g/(1+exp(-g)) * u
        const float u = __shfl_down_sync(0xffffffffu, sum, 1);
        const int r = rg * RPW + lane;
        if (lane < RPW && (lane & 1) == 0 && r + 1 < rows) yo.put(r / 2, (sum / (1.0f + expf_cr(-sum))) * u);
    } else {
        const int r = rg * RPW + lane;
        if (lane < RPW && r < rows) yo.put(r, epi == (int)Q4Epi::AddTo ? yo.local(r) + sum : sum);
    }
}

// LL: x is this rank's copy of a replicated LL buffer, read once its
// elements carry point x_point's epoch (tensor-parallel decode).  The kernel
// still waits for the previous one first (all of this rank's part of x is
// then there, only the other ranks' parts may still be in flight): polling
// from the moment the CTAs are resident measured slower, every CTA hammering
// the same few kilobytes of L2 while the producers run.
template <int RPW, bool LL, int KEEP>
__global__ void __launch_bounds__(kThreads, 3) gemv_q4_kernel(const uint4* __restrict__ qs,
                                                              const unsigned short* __restrict__ dsc, int rows,
                                                              int nb, int dstride, const void* __restrict__ x,
                                                              const float* __restrict__ norm_w, float eps, int pro,
                                                              int epi, float* __restrict__ y, const TpCtx tp,
                                                              int x_point, uint64_t y_shared, int y_row_off,
                                                              int y_point, int res_point) {
    using R = Ring<RPW>;
    const Act a = act_smem(nb);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float2* cb = a.cb + (size_t)warp * RPW * kCbStride;
    uint8_t* ring = reinterpret_cast<uint8_t*>(a.cb + (size_t)kWarps * RPW * kCbStride) + (size_t)warp * R::BYTES;
    const int row_groups = (rows + RPW - 1) / RPW;
    const int nchunk = (nb + 31) / 32;
    const int gw = blockIdx.x * kWarps + warp, GW = gridDim.x * kWarps;

    // Work items (row group, chunk), row-group-major; weights are immutable, so
    // the first S-1 items are requested before waiting on the previous kernel.
    pdl_trigger();
    int irg = gw, ic = 0;  // next item to issue
    auto step = [&](int& g, int& c) {
        if (++c == nchunk) {
            c = 0;
            g += GW;
        }
    };
#pragma unroll
    for (int k = 0; k < R::S - 1; ++k) {
        if (irg < row_groups) issue_item<RPW>(ring + k * R::STAGE, qs, dsc, rows, nb, dstride, irg, ic, lane);
        cp_async_commit();
        step(irg, ic);
    }
    const bool rms = pro == (int)Q4Pro::RmsNorm;
    NormPre np;
    norm_preload(np, norm_w, rms, nb);  // weights: before the dependency wait
    pdl_wait();
    if constexpr (LL) prologue<KEEP>(XLL{tp, static_cast<const uint2*>(x), tp_uepoch(tp, x_point), 100 + x_point},
                                     np, norm_w, eps, rms, nb, a);
    else prologue<KEEP>(XFloat{static_cast<const float4*>(x)}, np, norm_w, eps, rms, nb, a);
    const bool rep = tp.world > 1 && y == nullptr;
    const YOut<LL> yo{y, tp, y_shared, y_row_off, rep ? tp_uepoch(tp, y_point) : 0u, rep ? tp_uepoch(tp, res_point) : 0u,
                  rep};

    float sum = 0.0f;
    int rg = gw, c = 0, slot = 0, islot = R::S - 1;
    while (rg < row_groups) {
        cp_async_wait<R::S - 2>();  // this item's copies have landed (per thread)
        __syncwarp();               // ... and every lane's (the scales come from lanes 0..3)
        consume_item<RPW>(ring + slot * R::STAGE, a, cb, nb, c, lane, sum);
        if (irg < row_groups) issue_item<RPW>(ring + islot * R::STAGE, qs, dsc, rows, nb, dstride, irg, ic, lane);
        cp_async_commit();
        step(irg, ic);
        if (++islot == R::S) islot = 0;
        if (c == nchunk - 1) {
            epilogue<RPW, LL>(epi, rg, rows, lane, sum, yo);
            sum = 0.0f;
        }
        step(rg, c);
        if (++slot == R::S) slot = 0;
    }
    cp_async_wait<0>();
}

// ------------------------------------------------- cluster-shared prologue
// The activation is the same for every CTA of a GEMV, and with three CTAs on
// every SM its quantisation (and RMSNorm) is a real share of the kernel's
// critical path.  A pair of CTAs (a cluster of kCl = 2) splits it: CTA r
// loads, normalises and quantises blocks [r*nbr, (r+1)*nbr) only, keeps them
// and sends them to the other CTA's shared memory with st.async, which
// completes bytes on the receiver's mbarrier -- no fence, no cluster barrier
// on the data path (a release barrier here would also wait for this
// thread's weight prefetch).  The RMSNorm sum of squares is the fixed-order
// sum of the two partial sums, exchanged the same way.
constexpr int kCl = 2;

__device__ int g_gemv_status = 0;  // site of a GEMV wait that ran out (0: none)

struct PairX {
    uint64_t bar[2];  // [0]: the partner's partial sum (8 B), [1]: its quantised blocks
    double part[kCl];
    int abort;
};

__device__ __forceinline__ uint32_t mapa_peer(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_async_b64(uint32_t raddr, uint64_t v, uint32_t rbar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b64 [%0], %1, [%2];" ::"r"(raddr), "l"(v),
                 "r"(rbar)
                 : "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Bytes one CTA sends the other: 40 per block (lo 16, hi 16, d/sum 8).
__device__ __forceinline__ uint32_t pair_bytes(int nb, int rank) {
    const int nbr = (nb + kCl - 1) / kCl;
    const int b0 = min(nb, rank * nbr), b1 = min(nb, (rank + 1) * nbr);
    return (uint32_t)(b1 - b0) * 40u;
}

// Thread 0, first thing in the kernel: the two receive barriers, armed for
// what the partner will send; then every CTA of the cluster has started and
// sees them initialised (relaxed arrive: nothing else is published yet).
__device__ __forceinline__ void pair_setup(PairX& px, int nb, bool rms, bool exchange = true) {
    if (threadIdx.x == 0) {
        const uint32_t b = tc::smem_u32(px.bar);
        px.abort = 0;
        tc::mbar_init(b, 1);
        tc::mbar_init(b + 8, 1);
        tc::mbar_fence_init();
        if (rms) tc::mbar_expect_tx(b, 8);
        if (exchange) tc::mbar_expect_tx(b + 8, pair_bytes(nb, (int)cluster_rank() ^ 1));
    }
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}

struct PairSink {
    const Act& a;
    uint32_t peer, rbar;
    __device__ __forceinline__ void put(int b, int sub, uint2 pk, bool first, float2 dc) const {
        uint2* lp = reinterpret_cast<uint2*>(sub < 2 ? &a.lo[b] : &a.hi[b]) + (sub & 1);
        *lp = pk;
        st_async_b64(mapa_peer(tc::smem_u32(lp), peer), (uint64_t)pk.x | ((uint64_t)pk.y << 32), rbar);
        if (first) {
            a.dc[b] = dc;
            st_async_b64(mapa_peer(tc::smem_u32(&a.dc[b]), peer),
                         (uint64_t)__float_as_uint(dc.x) | ((uint64_t)__float_as_uint(dc.y) << 32), rbar);
        }
    }
};

// This CTA's slice of x in groups [g0, g1) (cluster rank r of kCl).
__device__ __forceinline__ void cluster_slice(int nb, int& g0, int& g1) {
    const int rank = (int)cg::this_cluster().block_rank(), nbr = (nb + kCl - 1) / kCl;
    g0 = min(nb, rank * nbr) * 4;
    g1 = min(nb, (rank + 1) * nbr) * 4;
}

// RMSNorm weights of this thread's first two groups of the slice (immutable:
// fetched before the dependency wait).
__device__ __forceinline__ void norm_preload_slice(NormPre& np, const float* __restrict__ norm_w, bool rms, int nb) {
    int g0, g1;
    cluster_slice(nb, g0, g1);
    const int tid = (int)threadIdx.x, bd = (int)blockDim.x;
#pragma unroll
    for (int it = 0; it < kNormKeep; ++it) {
        const int g = g0 + tid + it * bd;
        np.w[it][0] = np.w[it][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (rms && g < g1) {
            np.w[it][0] = reinterpret_cast<const float4*>(norm_w)[2 * g];
            np.w[it][1] = reinterpret_cast<const float4*>(norm_w)[2 * g + 1];
        }
    }
}

template <class Ld>
__device__ __forceinline__ void prologue_cluster(const Ld& ld, const NormPre& np, const float* __restrict__ norm_w,
                                                 float eps, bool rms, int nb, const Act& a, PairX& px) {
    static_assert(kNormKeep == 2, "two groups per thread are kept");
    static_assert(kCl == 2, "pairs of CTAs");
    const uint32_t rank = cluster_rank(), peer = rank ^ 1u;
    const uint32_t bar0 = tc::smem_u32(px.bar), bar1 = bar0 + 8;
    int g0, g1;
    cluster_slice(nb, g0, g1);
    const int bd = (int)blockDim.x, tid = (int)threadIdx.x;
    const int iters = (((nb + kCl - 1) / kCl) * 4 + bd - 1) / bd;  // the same in both CTAs
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    const int ga = g0 + tid, gb = g0 + tid + bd;
    float4 a0 = z, a1 = z, b0 = z, b1 = z;
    if (ga < g1) ld(ga, a0, a1);
    if (gb < g1) ld(gb, b0, b1);
    float inv = 1.0f;
    if (rms) {
        double ss = 0.0;
        auto acc = [&](float4 u, float4 v) {
            ss += (double)u.x * u.x + (double)u.y * u.y + (double)u.z * u.z + (double)u.w * u.w;
            ss += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
        };
        acc(a0, a1);
        acc(b0, b1);
        for (int g = g0 + tid + 2 * bd; g < g1; g += bd) {
            float4 u, v;
            ld(g, u, v);
            acc(u, v);
        }
        const double mine = block_sum_d(ss);  // ends with __syncthreads
        if (tid == 0)
            st_async_b64(mapa_peer(tc::smem_u32(&px.part[rank]), peer), (uint64_t)__double_as_longlong(mine),
                         mapa_peer(bar0, peer));
        tc::mbar_wait(bar0, 0, &px.abort, &g_gemv_status, 3);
        // rank 0's partial first in both CTAs: the same sum, the same inv
        const double tot = rank == 0 ? mine + px.part[1] : px.part[0] + mine;
        inv = 1.0f / sqrtf((float)(tot / (double)(nb * 32)) + eps);
    }
    const PairSink sink{a, peer, mapa_peer(bar1, peer)};
    if (iters > 0) quant_group(ga, ga < g1, a0, a1, np.w[0][0], np.w[0][1], rms, inv, sink);
    if (iters > 1) quant_group(gb, gb < g1, b0, b1, np.w[1][0], np.w[1][1], rms, inv, sink);
    for (int it = 2; it < iters; ++it) {
        const int g = g0 + tid + it * bd;
        const bool active = g < g1;  // uniform over the 4 lanes of a block
        float4 u = z, w = z, n0 = z, n1 = z;
        if (active) {
            ld(g, u, w);
            if (rms) {
                n0 = reinterpret_cast<const float4*>(norm_w)[2 * g];
                n1 = reinterpret_cast<const float4*>(norm_w)[2 * g + 1];
            }
        }
        quant_group(g, active, u, w, n0, n1, rms, inv, sink);
    }
    tc::mbar_wait(bar1, 0, &px.abort, &g_gemv_status, 4);  // the partner's half has landed
    __syncthreads();                                        // ... and this CTA's own half
}

// ------------------------------------------------------- row-tile kernel
// The same exact computation organised so that every lane does useful work.
// A CTA owns tiles of kTR = 16 rows (grid-stride over tiles) and walks K in
// chunks of 32 blocks through a kTS-stage cp.async ring shared by the CTA.
// Eight compute warps turn a staged chunk into per-block terms (d_w*d_a,
// float(isum)) for all 16 x 32 (row, block) pairs -- lane = row, so the
// activation block is a shared-memory broadcast -- into one of two term
// buffers; a ninth warp runs each row's FMA chain over the terms in block
// order (lane = row) while the compute warps fill the other buffer, and
// writes the outputs.  Instruction count per (row, block) is a quarter of
// the warp-per-row-group kernel above, whose chain ran on RPW lanes.
constexpr int kTR = 16;                    // rows per tile
constexpr int kTC = 32;                    // blocks per chunk
constexpr int kTS = 6;                     // ring stages (5 chunks in flight per CTA)
constexpr int kTW = kTC * 16 + 16;         // staged payload bytes per row (padded: conflict-free lane = row)
constexpr int kTSc = kTC * 2 + 16;         // staged scale bytes per row (padded)
constexpr int kTStage = kTR * (kTW + kTSc);
constexpr int kTT = kTC + 2;               // float2 per term row (padded)
constexpr int kTComp = 8;                  // compute warps
constexpr int kTThreads = (kTComp + 1) * 32;

struct TileSmem {
    int4* lo;
    int4* hi;
    float2* dc;
    float2* terms;  // [2][kTR][kTT]
    uint8_t* ring;  // [kTS][kTStage]
};

__device__ __forceinline__ TileSmem tile_smem(int nb) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    TileSmem t;
    t.lo = reinterpret_cast<int4*>(smem_raw);
    t.hi = t.lo + nb;
    t.dc = reinterpret_cast<float2*>(t.hi + nb);
    t.terms = t.dc + ((nb + 1) & ~1);
    t.ring = reinterpret_cast<uint8_t*>(t.terms + 2 * kTR * kTT);
    return t;
}

size_t tile_smem_bytes(uint64_t nb) {
    return nb * 32 + ((nb + 1) & ~1ull) * 8 + (size_t)2 * kTR * kTT * 8 + (size_t)kTS * kTStage;
}

__device__ __forceinline__ void bar_named(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Staging of chunk c of tile t: 16 rows x 32 blocks of nibbles (two 16-byte
// copies per compute thread: rows tid/32 and tid/32 + 8, block tid % 32) and
// the chunk's 32 scales of every row (threads 0..63: row tid/4, 8 scales).
struct TileIssuer {
    const uint4* qs;
    const unsigned short* dsc;
    int rows, nb, dstride, tid;
    __device__ __forceinline__ void operator()(uint8_t* st, int t, int c) const {
        const int r0 = t * kTR, blk = tid & 31, b = c * kTC + blk;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int row = (tid >> 5) + 8 * k;
            if (r0 + row < rows && b < nb)
                cp_async16(st + row * kTW + blk * 16, qs + (size_t)(r0 + row) * nb + b);
        }
        if (tid < kTR * 4) {
            const int row = tid >> 2, q = tid & 3, bs = c * kTC + q * 8;
            if (r0 + row < rows && bs < nb)
                cp_async16(st + kTR * kTW + row * kTSc + q * 16, dsc + (size_t)(r0 + row) * dstride + bs);
        }
    }
};

// (tile, chunk) of this CTA's items in order, advanced one item at a time.
// A CTA takes groups of `sup` consecutive tiles (g = blockIdx.x, then
// + gridDim.x): sup = 4 puts the 64 rows of one 32-output SiLU block in one
// CTA, in order.
struct TileCursor {
    int t, c, sub, g, sup;
    __device__ __forceinline__ TileCursor(int sup_) : t((int)blockIdx.x * sup_), c(0), sub(0), g((int)blockIdx.x),
                                                      sup(sup_) {}
    __device__ __forceinline__ void next(int nchunk) {
        if (++c == nchunk) {
            c = 0;
            if (++sub == sup) {
                sub = 0;
                g += gridDim.x;
            }
            t = g * sup + sub;
        }
    }
};

// Launched in clusters of kCl CTAs: the activation prologue is split across
// the cluster (prologue_cluster).
template <bool LL>
__global__ void __launch_bounds__(kTThreads, 3) gemv_q4_tile_kernel(const uint4* __restrict__ qs,
                                                                    const unsigned short* __restrict__ dsc, int rows,
                                                                    int nb, int dstride, const void* __restrict__ x,
                                                                    const float* __restrict__ norm_w, float eps,
                                                                    int pro, int epi, float* __restrict__ y,
                                                                    const TpCtx tp, int x_point, uint64_t y_shared,
                                                                    int y_row_off, int y_point, int res_point,
                                                                    void* __restrict__ yq) {
    __shared__ PairX px;
    __shared__ float qbuf[32];  // yq: the SiLU outputs of one Q8 block
    const bool rms = pro == (int)Q4Pro::RmsNorm, pre = pro == (int)Q4Pro::PreQuant;
    pair_setup(px, nb, rms, !pre);
    const TileSmem sm = tile_smem(nb);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int tiles = (rows + kTR - 1) / kTR, nchunk = (nb + kTC - 1) / kTC;
    // yq: groups of 4 tiles (the host checks tiles % 4 == 0)
    const int sup = yq ? 4 : 1, groups = tiles / sup;
    const int my_tiles = blockIdx.x < groups ? ((groups - 1 - blockIdx.x) / gridDim.x + 1) * sup : 0;
    const int items = my_tiles * nchunk;
    const TileIssuer issue{qs, dsc, rows, nb, dstride, tid};
    TileCursor nx(sup);  // next item to stage
    // weights are immutable: the first kTS-1 chunks are requested before
    // waiting on the previous kernel
    pdl_trigger();
    if (warp < kTComp) {
#pragma unroll
        for (int k = 0; k < kTS - 1; ++k) {
            if (k < items) {
                issue(sm.ring + k * kTStage, nx.t, nx.c);
                nx.next(nchunk);
            }
            cp_async_commit();
        }
    }
    NormPre np;
    norm_preload_slice(np, norm_w, rms, nb);
    pdl_wait();
    const Act a{sm.lo, sm.hi, sm.dc, nullptr};
    if (pre) {
        // the previous kernel quantised x already: copy its blocks as they are
        const int4* src = static_cast<const int4*>(x);
        int4* dst = sm.lo;
        const int n16 = (int)(q8_act_bytes((uint64_t)nb * 32) / 16);
        for (int i = tid; i < n16; i += (int)blockDim.x) dst[i] = src[i];
        __syncthreads();
    } else if constexpr (LL) {
        prologue_cluster(XLL{tp, static_cast<const uint2*>(x), tp_uepoch(tp, x_point), 100 + x_point}, np, norm_w,
                         eps, rms, nb, a, px);
    } else {
        prologue_cluster(XFloat{static_cast<const float4*>(x)}, np, norm_w, eps, rms, nb, a, px);
    }

    if (warp < kTComp) {
        // compute warps: lane & 15 = row, warp and lane >> 4 pick 2 blocks
        const int row = lane & 15, bq = warp * 4 + (lane >> 4) * 2;
        int c = 0, slot = 0, nslot = kTS - 1;
        for (int it = 0; it < items; ++it) {
            cp_async_wait<kTS - 2>();
            bar_named(1, kTComp * 32);  // chunk `it` landed for every thread; chunk it-1 fully read
            if (it + kTS - 1 < items) {
                issue(sm.ring + nslot * kTStage, nx.t, nx.c);
                nx.next(nchunk);
            }
            cp_async_commit();
            if (++nslot == kTS) nslot = 0;
            const uint8_t* st = sm.ring + slot * kTStage;
            if (++slot == kTS) slot = 0;
            const uint32_t sc2 = *reinterpret_cast<const uint32_t*>(st + kTR * kTW + row * kTSc + bq * 2);
            float4 out = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int b = c * kTC + bq + j;
                if (b < nb) {
                    const int4 alo = sm.lo[b], ahi = sm.hi[b];
                    const float2 dc = sm.dc[b];
                    const uint4 w = *reinterpret_cast<const uint4*>(st + row * kTW + (bq + j) * 16);
                    const int isum = block_isum(w, alo, ahi, __float_as_int(dc.y));
                    const float tw = half_bits_to_float((unsigned short)(sc2 >> (16 * j))) * dc.x;
                    if (j == 0) out.x = tw, out.y = (float)isum;
                    else out.z = tw, out.w = (float)isum;
                }
            }
            *reinterpret_cast<float4*>(sm.terms + ((it & 1) * kTR + row) * kTT + bq) = out;
            bar_named(2, kTThreads);  // terms of `it` complete; the chain of it-1 is done
            if (++c == nchunk) c = 0;
        }
        cp_async_wait<0>();
    } else {
        // chain warp: lane = row of the tile
        const bool rep = LL && tp.world > 1 && y == nullptr;
        const YOut<LL> yo{y, tp, y_shared, y_row_off, rep ? tp_uepoch(tp, y_point) : 0u,
                          rep ? tp_uepoch(tp, res_point) : 0u, rep};
        float sum = 0.0f;
        TileCursor cur(sup);
        for (int it = 0; it < items; ++it) {
            bar_named(2, kTThreads);
            const int t = cur.t, c = cur.c;
            cur.next(nchunk);
            if (lane < kTR) {
                const float2* tr = sm.terms + ((it & 1) * kTR + lane) * kTT;
                const int n = min(kTC, nb - c * kTC);
                if (n == kTC) {
#pragma unroll
                    for (int k = 0; k < kTC; k += 2) {
                        const float4 v = *reinterpret_cast<const float4*>(tr + k);
                        sum = fmaf(v.x, v.y, sum);
                        sum = fmaf(v.z, v.w, sum);
                    }
                } else {
                    for (int k = 0; k < n; ++k) sum = fmaf(tr[k].x, tr[k].y, sum);
                }
            }
            if (c == nchunk - 1) {
                const int r = t * kTR + lane;
                if (epi == (int)Q4Epi::SiluGate) {
                    const float u = __shfl_down_sync(0xffffffffu, sum, 1);
                    const float g = (sum / (1.0f + expf_cr(-sum))) * u;
                    if (lane < kTR && (lane & 1) == 0 && r + 1 < rows) yo.put(r / 2, g);
                    if (yq) {
                        // 8 outputs per tile; after the 4th tile of the group the
                        // warp quantises their 32-element block as quant_group does
                        if (lane < kTR && (lane & 1) == 0) qbuf[(t & 3) * 8 + lane / 2] = g;
                        if ((t & 3) == 3) {
                            __syncwarp();
                            const float v = qbuf[lane];
                            const float m = warp_max(fabsf(v));
                            const float d = m > 0.0f ? m / 127.0f : 1.0f;
                            const float id = 1.0f / d;
                            const int q = (int)fminf(fmaxf(roundf(v * id), -127.0f), 127.0f);
                            const int qsum = warp_sum_i(q);
                            uint32_t word = (uint32_t)(q & 0xff);
#pragma unroll
                            for (int k = 1; k < 4; ++k)
                                word |= (uint32_t)(__shfl_down_sync(0xffffffffu, q, k) & 0xff) << (8 * k);
                            const int b = t >> 2, nbo = rows / 64;
                            uint8_t* base = static_cast<uint8_t*>(yq);
                            if ((lane & 3) == 0)
                                *reinterpret_cast<uint32_t*>(base + (size_t)(lane < 16 ? b : nbo + b) * 16 +
                                                             (lane & 15)) = word;
                            if (lane == 0)
                                reinterpret_cast<float2*>(base + (size_t)nbo * 32)[b] =
                                    make_float2(d, __int_as_float(8 * qsum));
                            __syncwarp();
                        }
                    }
                } else if (lane < kTR && r < rows) {
                    yo.put(r, epi == (int)Q4Epi::AddTo ? yo.local(r) + sum : sum);
                }
                sum = 0.0f;
            }
        }
    }
}

// Diagnostic twin: the per-block int32 dots of the same device code.
__global__ void __launch_bounds__(kThreads) q4_block_dots_kernel(const uint4* __restrict__ qs, int rows, int nb,
                                                                 const float* __restrict__ x,
                                                                 int32_t* __restrict__ isum) {
    const Act a = act_smem(nb);
    NormPre np;
    norm_preload(np, nullptr, false, nb);
    prologue<2>(XFloat{reinterpret_cast<const float4*>(x)}, np, nullptr, 0.0f, false, nb, a);
    const uint64_t total = (uint64_t)rows * nb;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const int b = (int)(i % nb);
        isum[i] = block_isum(ld_stream_u4(qs + i), a.lo[b], a.hi[b], __float_as_int(a.dc[b].y));
    }
}

template <int RPW, bool LL, int KEEP>
cudaError_t launch(const GemvQ4Args& g, cudaStream_t s) {
    const mv_weight_s& w = *g.w;
    const size_t smem = act_smem_bytes(w.nb, RPW) + (size_t)kWarps * Ring<RPW>::BYTES;
    if (smem > 110 * 1024) return cudaErrorInvalidValue;  // two CTAs per SM
    ensure_smem_attr(gemv_q4_kernel<RPW, LL, KEEP>, 200 * 1024);
    const uint64_t groups = (w.rows + RPW - 1) / RPW;
    const uint64_t ctas = (groups + kWarps - 1) / kWarps;
    const uint64_t cap = (uint64_t)num_sms() * 2;
    const void* x = LL ? g.x_ll : static_cast<const void*>(g.x);
    return launch_pdl(gemv_q4_kernel<RPW, LL, KEEP>, dim3((unsigned)(ctas < cap ? ctas : cap)), dim3(kThreads), smem, s,
                      reinterpret_cast<const uint4*>(w.qs), (const unsigned short*)w.d, (int)w.rows, (int)w.nb,
                      (int)w.dstride, x, g.norm_w, g.eps, (int)g.pro, (int)g.epi, g.y, g.tp ? *g.tp : TpCtx{},
                      g.x_point, g.y_shared, g.y_row_off, g.y_point, g.res_point);
}

template <bool LL>
cudaError_t launch_tile(const GemvQ4Args& g, cudaStream_t s) {
    const mv_weight_s& w = *g.w;
    const size_t smem = tile_smem_bytes(w.nb);
    if (smem > 110 * 1024) return cudaErrorInvalidValue;  // two CTAs per SM at least
    ensure_smem_attr(gemv_q4_tile_kernel<LL>, 200 * 1024);
    // as many clusters as can be resident at once (clusters are placed
    // within a GPC, so this can be below SMs x CTAs per SM / kCl)
    static std::mutex mu;
    static std::map<std::pair<size_t, int>, int> fit;
    int dev = 0;
    cudaGetDevice(&dev);
    int clusters = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = fit.find({smem, dev});
        if (it != fit.end()) {
            clusters = it->second;
        } else {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(kCl * 64);
            cfg.blockDim = dim3(kTThreads);
            cfg.dynamicSmemBytes = smem;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = kCl;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            if (cudaOccupancyMaxActiveClusters(&clusters, gemv_q4_tile_kernel<LL>, &cfg) != cudaSuccess || clusters < 1) {
                cudaGetLastError();
                clusters = num_sms() * 2 / kCl;
            }
            fit[{smem, dev}] = clusters;
        }
    }
    const uint64_t tiles = (w.rows + kTR - 1) / kTR;
    const uint64_t units = g.yq ? tiles / 4 : tiles;  // yq: CTAs take groups of 4 tiles
    uint64_t cap = (uint64_t)clusters * kCl;
    const uint64_t keep = ((uint64_t)g.reserve + kCl - 1) / kCl * kCl;
    if (keep && cap > 2 * keep) cap -= keep;
    const uint64_t grid = ((units < cap ? units : cap) + kCl - 1) / kCl * kCl;
    const void* x = LL ? g.x_ll : static_cast<const void*>(g.x);
    return launch_pdl_cluster(gemv_q4_tile_kernel<LL>, dim3((unsigned)grid), dim3(kTThreads), smem, s, kCl,
                              reinterpret_cast<const uint4*>(w.qs), (const unsigned short*)w.d, (int)w.rows,
                              (int)w.nb, (int)w.dstride, x, g.norm_w, g.eps, (int)g.pro, (int)g.epi, g.y,
                              g.tp ? *g.tp : TpCtx{}, g.x_point, g.y_shared, g.y_row_off, g.y_point, g.res_point,
                              g.yq);
}

}  // namespace

bool gemv_q4_prequant_ok(const mv_weight_s& w) {
    return w.type == 2 && w.cols % 32 == 0 && tile_smem_bytes(w.nb) <= 110 * 1024;
}

cudaError_t gemv_q4(const GemvQ4Args& a, cudaStream_t s) {
    // x and norm_w are read as float4: the width must keep 8-element groups
    if (a.w->cols % 32) return cudaErrorInvalidValue;
    const bool tp = a.tp && a.tp->world > 1;
    if ((!a.y && !a.x_ll) || (a.x_ll && !tp) || (!a.x_ll && !a.x)) return cudaErrorInvalidValue;
    // quantised input / output: one GPU, the row-tile kernel, whole SiLU blocks
    if (a.pro == Q4Pro::PreQuant || a.yq) {
        if (tp || !gemv_q4_prequant_ok(*a.w)) return cudaErrorInvalidValue;
        if (a.yq && (a.epi != Q4Epi::SiluGate || a.w->rows % 64)) return cudaErrorInvalidValue;
        return launch_tile<false>(a, s);
    }
    if (tile_smem_bytes(a.w->nb) <= 110 * 1024) return a.x_ll ? launch_tile<true>(a, s) : launch_tile<false>(a, s);
    // Four rows per warp where the matrix has rows to spare (the chain cost
    // is shared by more rows), two otherwise so every SM has warps in flight.
    const bool r4 = a.w->rows >= 8192;
    if (a.x_ll) return r4 ? launch<4, true, 2>(a, s) : launch<2, true, 2>(a, s);
    return r4 ? launch<4, false, 2>(a, s) : launch<2, false, 2>(a, s);
}

// Adds the GEMV's status (a pair exchange whose bounded wait ran out) to
// *status (first site wins) and clears it.
cudaError_t gemv_status_take(int* status) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_gemv_status, sizeof(int));
    if (e == cudaSuccess && v) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_gemv_status, &zero, sizeof(int));
        if (!*status) *status = v;
    }
    return e;
}

cudaError_t q4_block_dots(const mv_weight_s& w, const float* x, int32_t* isum, cudaStream_t s) {
    ensure_smem_attr(q4_block_dots_kernel, 200 * 1024);
    const uint64_t total = w.rows * w.nb;
    const uint64_t ctas = (total + kThreads - 1) / kThreads, cap = (uint64_t)num_sms() * 4;
    q4_block_dots_kernel<<<(unsigned)(ctas < cap ? ctas : cap), kThreads, act_smem_bytes(w.nb, 1), s>>>(
        reinterpret_cast<const uint4*>(w.qs), (int)w.rows, (int)w.nb, x, isum);
    return cudaGetLastError();
}

}  // namespace mvb
