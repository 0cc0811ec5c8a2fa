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
// Bandwidth.  HBM-bound: each weight byte is read once with 128-bit loads
// (one 16-byte nibble payload per lane per block, plus its fp16 scale).  A
// warp owns RPW rows; its loads are double-buffered in registers in batches
// of 4 payloads per lane, and the first batch is issued before the activation
// prologue so the prologue's latency hides under the weight fetch.
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
#include "common.cuh"
#include "kernels.cuh"

namespace mvb {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kLoads = 4;        // payloads per lane per batch
constexpr int kCbStride = 34;    // float2 per chain-buffer row (16-byte aligned, conflict-free)
constexpr uint32_t kLoNib = 0x0F0F0F0Fu;

__device__ __forceinline__ int block_isum(const uint4 w, const int4 alo, const int4 ahi, int c8) {
    int s = dp4a((int)(w.x & kLoNib), alo.x, 0);
    s = dp4a((int)(w.y & kLoNib), alo.y, s);
    s = dp4a((int)(w.z & kLoNib), alo.z, s);
    s = dp4a((int)(w.w & kLoNib), alo.w, s);
    s = dp4a((int)((w.x >> 4) & kLoNib), ahi.x, s);
    s = dp4a((int)((w.y >> 4) & kLoNib), ahi.y, s);
    s = dp4a((int)((w.z >> 4) & kLoNib), ahi.z, s);
    s = dp4a((int)((w.w >> 4) & kLoNib), ahi.w, s);
    return s - c8;
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

// Quantised activations of (optionally RMS-normalised) x into shared memory.
__device__ __forceinline__ void prologue(const float* __restrict__ x, const float* __restrict__ norm_w, float eps,
                                         bool rms, int nb, const Act& a) {
    const int G = nb * 4;  // groups of 8 elements
    const int iters = (G + (int)blockDim.x - 1) / (int)blockDim.x;
    // the first kKeep groups of each thread stay in registers between the
    // RMS pass and the quantisation pass
    constexpr int kKeep = 2;
    float4 keep[kKeep][2];
    float inv = 1.0f;
    if (rms) {
        double ss = 0.0;
        int it = 0;
        for (int g = threadIdx.x; g < G; g += blockDim.x, ++it) {
            const float4 u = reinterpret_cast<const float4*>(x)[2 * g];
            const float4 v = reinterpret_cast<const float4*>(x)[2 * g + 1];
            if (it < kKeep) {
                keep[it][0] = u;
                keep[it][1] = v;
            }
            ss += (double)u.x * u.x + (double)u.y * u.y + (double)u.z * u.z + (double)u.w * u.w;
            ss += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
        }
        const double tot = block_sum_d(ss);
        inv = 1.0f / sqrtf((float)(tot / (double)(nb * 32)) + eps);
    }
    for (int it = 0; it < iters; ++it) {
        const int g = threadIdx.x + it * (int)blockDim.x;
        const bool active = g < G;  // uniform over the 4 lanes of a block
        float v[8];
        if (active) {
            float4 u, w;
            if (rms && it < kKeep) {
                u = keep[it][0];
                w = keep[it][1];
            } else {
                u = reinterpret_cast<const float4*>(x)[2 * g];
                w = reinterpret_cast<const float4*>(x)[2 * g + 1];
            }
            v[0] = u.x; v[1] = u.y; v[2] = u.z; v[3] = u.w; v[4] = w.x; v[5] = w.y; v[6] = w.z; v[7] = w.w;
            if (rms) {
                const float4 n0 = reinterpret_cast<const float4*>(norm_w)[2 * g];
                const float4 n1 = reinterpret_cast<const float4*>(norm_w)[2 * g + 1];
                const float nw[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = v[i] * inv * nw[i];  // (x*inv)*w as the reference
            }
        } else {
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
        if (active) {
            const int b = g >> 2, sub = g & 3;
            uint2* dst = reinterpret_cast<uint2*>(sub < 2 ? &a.lo[b] : &a.hi[b]) + (sub & 1);
            *dst = make_uint2(pk[0], pk[1]);
            if (sub == 0) a.dc[b] = make_float2(d, __int_as_float(8 * sum));
        }
    }
    __syncthreads();
}

// Correctly rounded expf through double precision, the closest portable
// match to the host libm's expf the reference calls.
__device__ __forceinline__ float expf_cr(float x) { return (float)exp((double)x); }

template <int RPW>
struct Batch {
    uint4 w[RPW][kLoads / RPW];
    unsigned short d[RPW][kLoads / RPW];
};

template <int RPW>
__device__ __forceinline__ void load_batch(Batch<RPW>& B, const uint4* __restrict__ qs,
                                           const unsigned short* __restrict__ dsc, int rows, int nb, int rg, int batch,
                                           int lane) {
    constexpr int PF = kLoads / RPW;  // chunks of 32 blocks per batch
#pragma unroll
    for (int p = 0; p < PF; ++p) {
        const int b = (batch * PF + p) * 32 + lane;
#pragma unroll
        for (int j = 0; j < RPW; ++j) {
            const int r = rg * RPW + j;
            if (b < nb && r < rows) {
                const size_t bi = (size_t)r * nb + b;
                B.w[j][p] = ld_stream_u4(qs + bi);
                B.d[j][p] = ld_stream_u16(dsc + bi);
            }
        }
    }
}

// Per-block terms of one batch, then each row's FMA chain over them in
// block order.  `sum` is live in lanes 0..RPW-1 (lane j = row j).
template <int RPW>
__device__ __forceinline__ void consume_batch(const Batch<RPW>& B, const Act& a, float2* cb, int nb, int batch,
                                              int lane, float& sum) {
    constexpr int PF = kLoads / RPW;
#pragma unroll
    for (int p = 0; p < PF; ++p) {
        const int c = batch * PF + p;
        const int b = c * 32 + lane;
        if (c * 32 >= nb) break;  // uniform: past the last chunk
        if (b < nb) {
            const int4 alo = a.lo[b], ahi = a.hi[b];
            const float2 dc = a.dc[b];
#pragma unroll
            for (int j = 0; j < RPW; ++j) {
                const int isum = block_isum(B.w[j][p], alo, ahi, __float_as_int(dc.y));
                cb[j * kCbStride + lane] = make_float2(half_bits_to_float(B.d[j][p]) * dc.x, (float)isum);
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
}

template <int RPW>
__device__ __forceinline__ void epilogue(int epi, int rg, int rows, int lane, float sum, float* __restrict__ y) {
    if (epi == (int)Q4Epi::SiluGate) {
        // rows come in (gate_i, up_i) pairs: ff_i = g/(1+exp(-g)) * u
        const float u = __shfl_down_sync(0xffffffffu, sum, 1);
        const int r = rg * RPW + lane;
        if (lane < RPW && (lane & 1) == 0 && r + 1 < rows) y[r / 2] = (sum / (1.0f + expf_cr(-sum))) * u;
    } else {
        const int r = rg * RPW + lane;
        if (lane < RPW && r < rows) {
            if (epi == (int)Q4Epi::AddTo) y[r] += sum;
            else y[r] = sum;
        }
    }
}

template <int RPW>
__global__ void __launch_bounds__(kThreads, 2) gemv_q4_kernel(const uint4* __restrict__ qs,
                                                              const unsigned short* __restrict__ dsc, int rows,
                                                              int nb, const float* __restrict__ x,
                                                              const float* __restrict__ norm_w, float eps, int pro,
                                                              int epi, float* __restrict__ y) {
    constexpr int PF = kLoads / RPW;
    const Act a = act_smem(nb);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float2* cb = a.cb + (size_t)warp * RPW * kCbStride;
    const int row_groups = (rows + RPW - 1) / RPW;
    const int nbatch = (nb + 32 * PF - 1) / (32 * PF);
    const int gw = blockIdx.x * kWarps + warp, GW = gridDim.x * kWarps;

    // Work items are (row group, batch) in row-group-major order.  The first
    // two items' weights are requested before waiting on the previous kernel
    // (weights are immutable), so their fetch overlaps its tail and the
    // activation prologue.
    auto advance = [&](int& g, int& b) {
        if (++b == nbatch) {
            b = 0;
            g += GW;
        }
    };
    pdl_trigger();
    int rg = gw, bt = 0;
    int rg1 = rg, bt1 = bt;
    advance(rg1, bt1);
    Batch<RPW> A, Bb;
    if (rg < row_groups) load_batch<RPW>(A, qs, dsc, rows, nb, rg, bt, lane);
    if (rg1 < row_groups) load_batch<RPW>(Bb, qs, dsc, rows, nb, rg1, bt1, lane);
    pdl_wait();
    prologue(x, norm_w, eps, pro == (int)Q4Pro::RmsNorm, nb, a);

    float sum = 0.0f;
    while (rg < row_groups) {
        // A holds item (rg, bt), Bb holds item (rg1, bt1)
        consume_batch<RPW>(A, a, cb, nb, bt, lane, sum);
        if (bt == nbatch - 1) {
            epilogue<RPW>(epi, rg, rows, lane, sum, y);
            sum = 0.0f;
        }
        int rg2 = rg1, bt2 = bt1;
        advance(rg2, bt2);
        if (rg2 < row_groups) load_batch<RPW>(A, qs, dsc, rows, nb, rg2, bt2, lane);
        if (rg1 >= row_groups) break;
        consume_batch<RPW>(Bb, a, cb, nb, bt1, lane, sum);
        if (bt1 == nbatch - 1) {
            epilogue<RPW>(epi, rg1, rows, lane, sum, y);
            sum = 0.0f;
        }
        int rg3 = rg2, bt3 = bt2;
        advance(rg3, bt3);
        if (rg3 < row_groups) load_batch<RPW>(Bb, qs, dsc, rows, nb, rg3, bt3, lane);
        rg = rg2;
        bt = bt2;
        rg1 = rg3;
        bt1 = bt3;
    }
}

// Diagnostic twin: the per-block int32 dots of the same device code.
__global__ void __launch_bounds__(kThreads) q4_block_dots_kernel(const uint4* __restrict__ qs, int rows, int nb,
                                                                 const float* __restrict__ x,
                                                                 int32_t* __restrict__ isum) {
    const Act a = act_smem(nb);
    prologue(x, nullptr, 0.0f, false, nb, a);
    const uint64_t total = (uint64_t)rows * nb;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const int b = (int)(i % nb);
        isum[i] = block_isum(ld_stream_u4(qs + i), a.lo[b], a.hi[b], __float_as_int(a.dc[b].y));
    }
}

template <int RPW>
cudaError_t launch(const GemvQ4Args& g, cudaStream_t s) {
    const mv_weight_s& w = *g.w;
    const size_t smem = act_smem_bytes(w.nb, RPW);
    ensure_smem_attr(gemv_q4_kernel<RPW>, 200 * 1024);
    const uint64_t groups = (w.rows + RPW - 1) / RPW;
    const uint64_t ctas = (groups + kWarps - 1) / kWarps;
    const uint64_t cap = (uint64_t)num_sms() * 2;
    return launch_pdl(gemv_q4_kernel<RPW>, dim3((unsigned)(ctas < cap ? ctas : cap)), dim3(kThreads), smem, s,
                      reinterpret_cast<const uint4*>(w.qs), (const unsigned short*)w.d, (int)w.rows, (int)w.nb,
                      g.x, g.norm_w, g.eps, (int)g.pro, (int)g.epi, g.y);
}

}  // namespace

cudaError_t gemv_q4(const GemvQ4Args& a, cudaStream_t s) {
    // x and norm_w are read as float4: the width must keep 8-element groups
    if (a.w->cols % 32) return cudaErrorInvalidValue;
    // Four rows per warp where the matrix has rows to spare (the chain cost
    // is shared by more rows), two otherwise so every SM has warps in flight.
    if (a.w->rows >= 8192) return launch<4>(a, s);
    return launch<2>(a, s);
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
