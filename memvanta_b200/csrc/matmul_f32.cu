// matmul_f32.cu -- fp32-activation matmul for every weight type.
#include "common.cuh"
#include "kernels.cuh"

namespace mvb {

constexpr uint32_t kLoNib = 0x0F0F0F0Fu;

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
// Mapping (1 to 7 tokens): one warp per row, lane l owns elements
// [128*s + 4l, +4) of every 128-wide step s, so a lane reads one 32-bit
// payload word (4 elements) and one float4 of each token's activations; the
// token tile (T tokens x K floats) sits in shared memory and every float4
// read is bank-conflict-free.
// =====================================================================

constexpr int kFWarps = 8;

template <int TYPE>
__device__ __forceinline__ void deq4(const mv_weight_s& w, uint64_t r, uint64_t e0, float out[4]) {
    if constexpr (TYPE == 2) {  // Q4_0: element e<16 low nibble of byte e, else high nibble of byte e-16
        const uint64_t b = r * w.nb + e0 / 32;
        const int e = (int)(e0 % 32);
        const uint32_t word = ld_stream_u32(w.qs + b * 16 + (e & 15));
        const uint32_t nib = e < 16 ? (word & kLoNib) : ((word >> 4) & kLoNib);
        const float d = half_bits_to_float(ld_stream_u16(w.d + r * w.dstride + e0 / 32));
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

// ---------------------------------------------------------------------
// Batches of 8 tokens and more: a register-tiled kernel.  A CTA owns ROWS
// (64, 32 or 16) rows x 32 tokens and runs KS groups of 128 threads; group g
// takes the K chunks g, g + KS, ... (64 elements each), dequantised (deq4,
// the same per-element values) into the group's row-major shared tile next
// to the chunk's activations, so each weight element is loaded and
// dequantised once per 32 tokens instead of once per token.  A thread owns
// rows lt%16 + 16i (i < ROWS/16) and tokens 4*(lt/16) + j (j < 4) and reads
// float4 runs of 4 k from both tiles (the 16 rows a warp reads are
// consecutive: no bank conflicts); the group's next chunk is loaded into
// registers while the current one is multiplied.  The kernel is
// latency-bound on those loads, so the K groups are there for resident
// warps.  Each output is one fp32 FMA chain per group over its chunks in
// order, the groups' partial sums then added in group order.
constexpr int kTTok = 32, kTK = 64, kTThreads = 128;
constexpr int kTPad = kTK + 4;  // floats per tile row (16-byte aligned, rows 4 banks apart)

__host__ __device__ constexpr size_t tiled_smem(int rows, int ks) {
    return (size_t)ks * (rows + kTTok) * kTPad * sizeof(float);
}

template <int TYPE, int ROWS, int KS>
__global__ void __launch_bounds__(kTThreads * KS) matmul_f32act_tiled_kernel(mv_weight_s w,
                                                                             const float* __restrict__ x, int batch,
                                                                             float* __restrict__ y) {
    constexpr int RT = ROWS / 16;                       // rows per thread
    constexpr int WG = ROWS * kTK / 4 / kTThreads;      // weight groups of 4 a thread stages
    constexpr int XG = kTTok * kTK / 4 / kTThreads;     // activation float4 a thread stages
    extern __shared__ __align__(16) float tsm[];
    const int K = (int)w.cols, rows = (int)w.rows;
    const int grp = (int)threadIdx.x / kTThreads, lt = (int)threadIdx.x % kTThreads;
    float(*ws)[kTPad] = reinterpret_cast<float(*)[kTPad]>(tsm + (size_t)grp * (ROWS + kTTok) * kTPad);
    float(*xs)[kTPad] = ws + ROWS;
    const int r0 = blockIdx.x * ROWS, t0 = blockIdx.y * kTTok;
    const int tr = lt & 15, tt = (lt >> 4) * 4;
    float wv[WG][4], xv[XG][4];
    auto load = [&](int k0) {
#pragma unroll
        for (int i = 0; i < WG; ++i) {
            const int g = lt + i * kTThreads, row = g / (kTK / 4), kk = (g % (kTK / 4)) * 4;
            const int r = r0 + row, e0 = k0 + kk;
            if (r < rows && e0 < K) deq4<TYPE>(w, (uint64_t)r, (uint64_t)e0, wv[i]);
            else wv[i][0] = wv[i][1] = wv[i][2] = wv[i][3] = 0.0f;
        }
#pragma unroll
        for (int i = 0; i < XG; ++i) {
            const int g = lt + i * kTThreads, tok = g / (kTK / 4), kk = (g % (kTK / 4)) * 4;
            const int t = t0 + tok, e0 = k0 + kk;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t < batch && e0 < K) v = *reinterpret_cast<const float4*>(x + (size_t)t * K + e0);
            xv[i][0] = v.x, xv[i][1] = v.y, xv[i][2] = v.z, xv[i][3] = v.w;
        }
    };
    auto store = [&]() {
#pragma unroll
        for (int i = 0; i < WG; ++i) {
            const int g = lt + i * kTThreads, row = g / (kTK / 4), kk = (g % (kTK / 4)) * 4;
            *reinterpret_cast<float4*>(&ws[row][kk]) = make_float4(wv[i][0], wv[i][1], wv[i][2], wv[i][3]);
        }
#pragma unroll
        for (int i = 0; i < XG; ++i) {
            const int g = lt + i * kTThreads, tok = g / (kTK / 4), kk = (g % (kTK / 4)) * 4;
            *reinterpret_cast<float4*>(&xs[tok][kk]) = make_float4(xv[i][0], xv[i][1], xv[i][2], xv[i][3]);
        }
    };
    float acc[RT][4];
#pragma unroll
    for (int i = 0; i < RT; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    // every group runs the same number of rounds (a chunk past K loads zeros)
    const int rounds = ((K + kTK - 1) / kTK + KS - 1) / KS;
    load(grp * kTK);
    for (int rd = 0; rd < rounds; ++rd) {
        __syncthreads();  // the previous chunk's tiles are no longer read
        store();
        __syncthreads();
        if (rd + 1 < rounds) load((grp + (rd + 1) * KS) * kTK);  // in flight during this chunk's FMAs
#pragma unroll 4
        for (int k = 0; k < kTK; k += 4) {
            float4 a[RT], b[4];
#pragma unroll
            for (int i = 0; i < RT; ++i) a[i] = *reinterpret_cast<const float4*>(&ws[tr + 16 * i][k]);
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = *reinterpret_cast<const float4*>(&xs[tt + j][k]);
#pragma unroll
            for (int i = 0; i < RT; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    acc[i][j] = fmaf(a[i].x, b[j].x, acc[i][j]);
                    acc[i][j] = fmaf(a[i].y, b[j].y, acc[i][j]);
                    acc[i][j] = fmaf(a[i].z, b[j].z, acc[i][j]);
                    acc[i][j] = fmaf(a[i].w, b[j].w, acc[i][j]);
                }
        }
    }
    if constexpr (KS > 1) {
        // groups 1.. hand their partial sums to group 0 (the tiles are free now)
        __syncthreads();
        float* part = tsm + (size_t)lt * (KS - 1) * RT * 4;
        if (grp > 0)
#pragma unroll
            for (int i = 0; i < RT; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) part[((grp - 1) * RT + i) * 4 + j] = acc[i][j];
        __syncthreads();
        if (grp > 0) return;
#pragma unroll
        for (int g = 0; g < KS - 1; ++g)
#pragma unroll
            for (int i = 0; i < RT; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] += part[(g * RT + i) * 4 + j];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int t = t0 + tt + j;
        if (t >= batch) continue;
#pragma unroll
        for (int i = 0; i < RT; ++i) {
            const int r = r0 + tr + 16 * i;
            if (r < rows) y[(size_t)t * rows + r] = acc[i][j];
        }
    }
}

template <int TYPE, int ROWS, int KS>
static cudaError_t launch_tiled(const mv_weight_s& w, const float* x, uint64_t batch, float* y, cudaStream_t s,
                                uint64_t ttiles) {
    const size_t smem = tiled_smem(ROWS, KS);
    ensure_smem_attr(matmul_f32act_tiled_kernel<TYPE, ROWS, KS>, (int)smem);
    const dim3 grid((unsigned)((w.rows + ROWS - 1) / ROWS), (unsigned)ttiles);
    matmul_f32act_tiled_kernel<TYPE, ROWS, KS><<<grid, kTThreads * KS, smem, s>>>(w, x, (int)batch, y);
    return cudaGetLastError();
}

template <int TYPE>
static cudaError_t launch_f32act_tiled(const mv_weight_s& w, const float* x, uint64_t batch, float* y,
                                       cudaStream_t s) {
    // narrower row tiles, and more K groups, where wider ones would leave SMs
    // without two CTAs (resident warps hide the chunk loads)
    const uint64_t ttiles = (batch + kTTok - 1) / kTTok, want = 2 * (uint64_t)num_sms();
    if ((w.rows + 63) / 64 * ttiles >= want) return launch_tiled<TYPE, 64, 2>(w, x, batch, y, s, ttiles);
    if ((w.rows + 31) / 32 * ttiles >= want) return launch_tiled<TYPE, 32, 2>(w, x, batch, y, s, ttiles);
    return launch_tiled<TYPE, 16, 4>(w, x, batch, y, s, ttiles);
}

template <int TYPE>
static cudaError_t dispatch_t(const mv_weight_s& w, const float* x, uint64_t batch, float* y, cudaStream_t s) {
    const uint64_t budget = 200 * 1024 / 4;  // floats of activation tile that fit in shared memory
    if (batch >= 8) return launch_f32act_tiled<TYPE>(w, x, batch, y, s);
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
