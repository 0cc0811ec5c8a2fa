// gemv.cu -- decode GEMV kernels.
//
// gemv_q4_kernel: y = W x for a Q4_0 weight with Q8 activations, the
// reference's decode path (tensor_matvec Q4_0 branch,
// src/gguf_kernels.cpp:246 -> quantize_q8 :161-172 -> dot_q4_q8 :189 ->
// dot_q4_q8_block :180-188).  HBM-bound: every weight byte is read once with
// 128-bit streaming loads (one 16-byte nibble payload per lane per block plus
// its fp16 scale), activations live in shared memory.
//
// Prologue (each CTA, redundantly): optional RMSNorm of x (double sum of
// squares, src/llama_model.cpp:237) and the per-32 Q8 quantisation, stored
// split into low/high 16-byte halves so a lane's two 128-bit shared loads
// are conflict-free, plus the block scale and 8*sum(q).
//
// Block dot: GGUF element i<16 is the low nibble of byte i, element 16+i the
// high nibble.  With w the 16 payload bytes as four words,
//   sum_i (nib_i - 8) * a_i = sum dp4a(w & 0x0F0F0F0F, a_lo)
//                            + sum dp4a((w>>4) & 0x0F0F0F0F, a_hi) - 8*sum(a)
// which is the reference's int32 block dot exactly (nibbles are 0..15, so
// the signed dp4a sees them as non-negative bytes).
// Row sum: acc += (d_w * d_a) * float(isum) with one FMA, as the reference's
// GCC build evaluates it; the order over blocks is a lane-strided tree
// instead of sequential, so rows agree to rounding (~1e-6 relative).
#include "common.cuh"
#include "kernels.cuh"

namespace mvb {

constexpr int kQ4Warps = 16;
constexpr int kQ4Threads = kQ4Warps * 32;
constexpr int kQ4Unroll = 4;
constexpr uint32_t kLoNib = 0x0F0F0F0Fu;

__device__ __forceinline__ int q4_block_isum(const uint4 w, const int4 alo, const int4 ahi, int c8) {
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

struct Q4Smem {
    int4* lo;
    int4* hi;
    float* d;
    int* c8;
};

__device__ __forceinline__ Q4Smem q4_smem(int nb) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Q4Smem s;
    s.lo = reinterpret_cast<int4*>(smem_raw);
    s.hi = s.lo + nb;
    s.d = reinterpret_cast<float*>(s.hi + nb);
    s.c8 = reinterpret_cast<int*>(s.d + nb);
    return s;
}

static size_t q4_smem_bytes(uint64_t nb) { return nb * (16 + 16 + 4 + 4); }

// Fills shared memory with the Q8-quantised activations (optionally after
// RMSNorm).  All threads of the CTA take part; ends with __syncthreads().
__device__ __forceinline__ void q4_prologue(const float* __restrict__ x, const float* __restrict__ norm_w, float eps,
                                            bool rms, int nb, const Q4Smem& s) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int K = nb * 32;
    float inv = 1.0f;
    if (rms) {
        __shared__ double red[32];
        double ss = 0.0;
        for (int i = threadIdx.x; i < K; i += blockDim.x) {
            const double v = (double)x[i];
            ss += v * v;
        }
        ss = warp_sum_d(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (warp == 0) {
            double t = lane < nwarps ? red[lane] : 0.0;
            t = warp_sum_d(t);
            if (lane == 0) red[0] = t;
        }
        __syncthreads();
        inv = 1.0f / sqrtf((float)(red[0] / (double)K) + eps);
    }
    for (int b = warp; b < nb; b += nwarps) {
        float v = x[b * 32 + lane];
        if (rms) v = v * inv * norm_w[b * 32 + lane];
        float dd;
        const int q = quant_q8_lane(v, dd);
        int8_t* dst = reinterpret_cast<int8_t*>(lane < 16 ? &s.lo[b] : &s.hi[b]);
        dst[lane & 15] = (int8_t)q;
        const int sum = warp_sum_i(q);
        if (lane == 0) {
            s.d[b] = dd;
            s.c8[b] = 8 * sum;
        }
    }
    __syncthreads();
}

template <int RPW>
__global__ void __launch_bounds__(kQ4Threads, 2) gemv_q4_kernel(const uint4* __restrict__ qs,
                                                             const unsigned short* __restrict__ dsc, int rows, int nb,
                                                             const float* __restrict__ x,
                                                             const float* __restrict__ norm_w, float eps, int pro,
                                                             int epi, float* __restrict__ y) {
    const Q4Smem s = q4_smem(nb);
    q4_prologue(x, norm_w, eps, pro == (int)Q4Pro::RmsNorm, nb, s);

    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * kQ4Warps + (threadIdx.x >> 5);
    const int GW = gridDim.x * kQ4Warps;
    constexpr int U = kQ4Unroll / RPW;  // 4 block payloads in flight per lane
    for (int r0 = gw * RPW; r0 < rows; r0 += GW * RPW) {
        float acc[RPW];
#pragma unroll
        for (int j = 0; j < RPW; ++j) acc[j] = 0.0f;
        for (int b0 = lane; b0 < nb; b0 += 32 * U) {
            uint4 w[RPW][U];
            unsigned short dh[RPW][U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int b = b0 + 32 * u;
#pragma unroll
                for (int j = 0; j < RPW; ++j) {
                    const int r = r0 + j;
                    if (b < nb && r < rows) {
                        const size_t bi = (size_t)r * nb + b;
                        w[j][u] = ld_stream_u4(qs + bi);
                        dh[j][u] = ld_stream_u16(dsc + bi);
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int b = b0 + 32 * u;
                if (b < nb) {
                    const int4 alo = s.lo[b], ahi = s.hi[b];
                    const float ad = s.d[b];
                    const int c8 = s.c8[b];
#pragma unroll
                    for (int j = 0; j < RPW; ++j) {
                        if (r0 + j < rows) {
                            const int isum = q4_block_isum(w[j][u], alo, ahi, c8);
                            acc[j] = fmaf(half_bits_to_float(dh[j][u]) * ad, (float)isum, acc[j]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int j = 0; j < RPW; ++j) acc[j] = warp_sum(acc[j]);
        if (lane == 0) {
            if (epi == (int)Q4Epi::SiluGate) {
                // rows (r0, r0+1) = (gate_i, up_i): ff_i = g/(1+exp(-g)) * u
                const float g = acc[0], u = RPW > 1 ? acc[RPW - 1] : 0.0f;
                y[r0 / 2] = (g / (1.0f + expf(-g))) * u;
            } else {
#pragma unroll
                for (int j = 0; j < RPW; ++j) {
                    if (r0 + j < rows) {
                        if (epi == (int)Q4Epi::AddTo) y[r0 + j] += acc[j];
                        else y[r0 + j] = acc[j];
                    }
                }
            }
        }
    }
}

// Diagnostic twin: the per-block int32 dots of the same device code.
__global__ void __launch_bounds__(kQ4Threads) q4_block_dots_kernel(const uint4* __restrict__ qs, int rows, int nb,
                                                                   const float* __restrict__ x,
                                                                   int32_t* __restrict__ isum) {
    const Q4Smem s = q4_smem(nb);
    q4_prologue(x, nullptr, 0.0f, false, nb, s);
    const uint64_t total = (uint64_t)rows * nb;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const int b = (int)(i % nb);
        isum[i] = q4_block_isum(ld_stream_u4(qs + i), s.lo[b], s.hi[b], s.c8[b]);
    }
}

static int q4_grid(uint64_t items) {
    const uint64_t ctas = (items + kQ4Warps - 1) / kQ4Warps;
    const uint64_t cap = (uint64_t)num_sms() * 4;
    return (int)(ctas < cap ? (ctas ? ctas : 1) : cap);
}

cudaError_t gemv_q4(const GemvQ4Args& a, cudaStream_t s) {
    const mv_weight_s& w = *a.w;
    const size_t smem = q4_smem_bytes(w.nb);
    const bool pairs = a.epi == Q4Epi::SiluGate;
    if (pairs) {
        ensure_smem_attr(gemv_q4_kernel<2>, 200 * 1024);
        gemv_q4_kernel<2><<<q4_grid(w.rows / 2), kQ4Threads, smem, s>>>(
            reinterpret_cast<const uint4*>(w.qs), w.d, (int)w.rows, (int)w.nb, a.x, a.norm_w, a.eps, (int)a.pro,
            (int)a.epi, a.y);
    } else {
        ensure_smem_attr(gemv_q4_kernel<1>, 200 * 1024);
        gemv_q4_kernel<1><<<q4_grid(w.rows), kQ4Threads, smem, s>>>(
            reinterpret_cast<const uint4*>(w.qs), w.d, (int)w.rows, (int)w.nb, a.x, a.norm_w, a.eps, (int)a.pro,
            (int)a.epi, a.y);
    }
    return cudaGetLastError();
}

cudaError_t q4_block_dots(const mv_weight_s& w, const float* x, int32_t* isum, cudaStream_t s) {
    ensure_smem_attr(q4_block_dots_kernel, 200 * 1024);
    q4_block_dots_kernel<<<q4_grid(w.rows), kQ4Threads, q4_smem_bytes(w.nb), s>>>(
        reinterpret_cast<const uint4*>(w.qs), (int)w.rows, (int)w.nb, x, isum);
    return cudaGetLastError();
}

// =====================================================================
// fp32-activation matmul for every weight type.
//
// The reference's fp32-activation dots: tensor_matvec for Q8_0 / Q6_K / F16 /
// F32 (src/gguf_kernels.cpp:247-250), tensor_matmul_batch (:255-259) and the
// default prefill of tensor_matmul_batch_v06 (:268).  Each weight element is
// dequantised to fp32 exactly as the reference does it (Q4_0 float(q-8)*d,
// Q8_0 float(q)*d, Q6_K d*scale*q6, F16 exact) and FMA'd against fp32
// activations; Q6_K/F16 accumulate in fp32 instead of the reference's double
// (the 5e-3 / 1e-3 tolerances hold with margin).
//
// Mapping: one warp per row, lane l owns elements [128*s + 4l, +4) of every
// 128-wide step s, so a lane reads one 32-bit payload word (4 elements) and
// one float4 of each token's activations; the token tile (T tokens x K
// floats) sits in shared memory and every float4 read is bank-conflict-free.
// =====================================================================

constexpr int kFWarps = 8;

template <int TYPE>
__device__ __forceinline__ void deq4(const mv_weight_s& w, uint64_t r, uint64_t e0, float out[4]) {
    if constexpr (TYPE == 2) {  // Q4_0: element e<16 low nibble of byte e, else high nibble of byte e-16
        const uint64_t b = r * w.nb + e0 / 32;
        const int e = (int)(e0 % 32);
        const uint32_t word = ld_stream_u32(w.qs + b * 16 + (e & 15));
        const uint32_t nib = e < 16 ? (word & kLoNib) : ((word >> 4) & kLoNib);
        const float d = half_bits_to_float(ld_stream_u16(w.d + b));
#pragma unroll
        for (int i = 0; i < 4; ++i) out[i] = u8_to_f32_minus(nib, i, 8388616.0f) * d;
    } else if constexpr (TYPE == 8) {  // Q8_0
        const uint64_t b = r * w.nb + e0 / 32;
        const uint32_t word = ld_stream_u32(w.qs + b * 32 + e0 % 32);
        const float d = half_bits_to_float(ld_stream_u16(w.d + b));
#pragma unroll
        for (int i = 0; i < 4; ++i) out[i] = s8_to_f32(word, i) * d;
    } else if constexpr (TYPE == 14) {  // Q6_K, src/gguf_kernels.cpp:122-136
        const uint64_t b = r * w.nb + e0 / 256;
        const int i0 = (int)(e0 % 256), r32 = i0 / 32, j = i0 % 32, g = r32 / 4, slot = r32 % 4;
        const uint32_t ql = ld_stream_u32(w.qs + b * 128 + g * 64 + (slot & 1) * 32 + j);
        const uint32_t qh = ld_stream_u32(w.qh + b * 64 + g * 32 + j);
        const uint32_t lo = (slot < 2 ? ql : (ql >> 4)) & kLoNib;
        const uint32_t hi = ((qh >> (2 * slot)) & 0x03030303u) << 4;
        const uint32_t q6 = lo | hi;
        const float dsc = half_bits_to_float(ld_stream_u16(w.d + b)) * (float)w.sc[b * 16 + i0 / 16];
#pragma unroll
        for (int i = 0; i < 4; ++i) out[i] = dsc * u8_to_f32_minus(q6, i, 8388640.0f);
    } else if constexpr (TYPE == 1) {  // F16
        const uint2 h = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(w.qs) + r * w.cols + e0);
        out[0] = half_bits_to_float(h.x & 0xffff);
        out[1] = half_bits_to_float(h.x >> 16);
        out[2] = half_bits_to_float(h.y & 0xffff);
        out[3] = half_bits_to_float(h.y >> 16);
    } else {  // F32
        const float4 v = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(w.qs) + r * w.cols + e0);
        out[0] = v.x;
        out[1] = v.y;
        out[2] = v.z;
        out[3] = v.w;
    }
}

template <int TYPE, int T>
__global__ void __launch_bounds__(kFWarps * 32) matmul_f32act_kernel(mv_weight_s w, const float* __restrict__ x,
                                                                     int batch, float* __restrict__ y) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float* xs = reinterpret_cast<float*>(smem_raw);
    const int K = (int)w.cols;
    const int t0 = blockIdx.y * T;
    const int nt = min(T, batch - t0);
    for (int i = threadIdx.x; i < T * K; i += blockDim.x) {
        const int t = i / K;
        xs[i] = t < nt ? x[(size_t)(t0 + t) * K + (i % K)] : 0.0f;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * kFWarps + (threadIdx.x >> 5), GW = gridDim.x * kFWarps;
    for (int r = gw; r < (int)w.rows; r += GW) {
        float acc[T];
#pragma unroll
        for (int t = 0; t < T; ++t) acc[t] = 0.0f;
        // K % 4 == 0, so a group that starts inside the row ends inside it.
        for (int e0 = lane * 4; e0 < K; e0 += 128) {
            float wv[4];
            deq4<TYPE>(w, (uint64_t)r, (uint64_t)e0, wv);
#pragma unroll
            for (int t = 0; t < T; ++t) {
                const float4 xv = *reinterpret_cast<const float4*>(xs + t * K + e0);
                acc[t] = fmaf(wv[0], xv.x, acc[t]);
                acc[t] = fmaf(wv[1], xv.y, acc[t]);
                acc[t] = fmaf(wv[2], xv.z, acc[t]);
                acc[t] = fmaf(wv[3], xv.w, acc[t]);
            }
        }
#pragma unroll
        for (int t = 0; t < T; ++t) {
            const float v = warp_sum(acc[t]);
            if (lane == 0 && t < nt) y[(size_t)(t0 + t) * w.rows + r] = v;
        }
    }
}

template <int TYPE, int T>
static cudaError_t launch_f32act(const mv_weight_s& w, const float* x, uint64_t batch, float* y, cudaStream_t s) {
    const size_t smem = (size_t)T * w.cols * sizeof(float);
    ensure_smem_attr(matmul_f32act_kernel<TYPE, T>, 220 * 1024);
    const uint64_t ctas = (w.rows + kFWarps - 1) / kFWarps;
    const uint64_t cap = (uint64_t)num_sms() * 2;
    dim3 grid((unsigned)(ctas < cap ? ctas : cap), (unsigned)((batch + T - 1) / T));
    matmul_f32act_kernel<TYPE, T><<<grid, kFWarps * 32, smem, s>>>(w, x, (int)batch, y);
    return cudaGetLastError();
}

template <int TYPE>
static cudaError_t dispatch_t(const mv_weight_s& w, const float* x, uint64_t batch, float* y, cudaStream_t s) {
    const uint64_t budget = 200 * 1024 / 4;  // floats of activation tile that fit in shared memory
    if (batch == 1) return launch_f32act<TYPE, 1>(w, x, batch, y, s);
    if (batch == 2 || 4 * w.cols > budget) {
        if (2 * w.cols > budget) return launch_f32act<TYPE, 1>(w, x, batch, y, s);
        return launch_f32act<TYPE, 2>(w, x, batch, y, s);
    }
    if (batch <= 4 || 8 * w.cols > budget) return launch_f32act<TYPE, 4>(w, x, batch, y, s);
    return launch_f32act<TYPE, 8>(w, x, batch, y, s);
}

cudaError_t matmul_f32act(const mv_weight_s& w, const float* x, uint64_t batch, float* y, cudaStream_t s) {
    if (!batch) return cudaSuccess;
    if (w.cols % 4) return cudaErrorInvalidValue;  // lanes own whole 4-element groups
    switch (w.type) {
        case 2: return dispatch_t<2>(w, x, batch, y, s);
        case 8: return dispatch_t<8>(w, x, batch, y, s);
        case 14: return dispatch_t<14>(w, x, batch, y, s);
        case 1: return dispatch_t<1>(w, x, batch, y, s);
        case 0: return dispatch_t<0>(w, x, batch, y, s);
    }
    return cudaErrorInvalidValue;
}

}  // namespace mvb
