// gemm.cu -- batched Q4_0 x Q8-activation matmul (prefill), CUDA-core path.
//
// The reference's MEMVANTA_FORCE_Q8_ACT=1 prefill
// (tensor_matmul_batch_v06, src/gguf_kernels.cpp:265-266): every activation
// row is quantised per 32-block (quantize_activations_q8, :174-178) and every
// (token, row) pair is the decode row dot dot_q4_q8 (:189).  Here a warp owns
// a weight row, loads each 16-byte block payload once and reuses it for a
// tile of T tokens whose quantised activations sit in shared memory (split
// into conflict-free low/high 16-byte halves, as in the decode GEMV).
#include "common.cuh"
#include "kernels.cuh"

namespace mvb {

constexpr int kGWarps = 8;
constexpr int kGTok = 8;
constexpr uint32_t kNib = 0x0F0F0F0Fu;

__global__ void __launch_bounds__(kGWarps * 32) gemm_q4_q8_kernel(const uint4* __restrict__ qs,
                                                                  const unsigned short* __restrict__ dsc, int rows,
                                                                  int nb, const int8_t* __restrict__ q,
                                                                  const float* __restrict__ d, int batch,
                                                                  float* __restrict__ y, int accumulate) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    int4* lo = reinterpret_cast<int4*>(smem_raw);           // [T][nb]
    int4* hi = lo + kGTok * nb;                              // [T][nb]
    float* ad = reinterpret_cast<float*>(hi + kGTok * nb);   // [T][nb]
    int* c8 = reinterpret_cast<int*>(ad + kGTok * nb);       // [T][nb]
    const int t0 = blockIdx.y * kGTok;
    const int nt = min(kGTok, batch - t0);
    const int K = nb * 32;
    // stage the token tile: 16-byte halves, scale, 8*sum(q)
    for (int i = threadIdx.x; i < kGTok * nb; i += blockDim.x) {
        const int t = i / nb, b = i % nb;
        if (t < nt) {
            const int8_t* src = q + (size_t)(t0 + t) * K + b * 32;
            const int4 l = *reinterpret_cast<const int4*>(src);
            const int4 h = *reinterpret_cast<const int4*>(src + 16);
            lo[i] = l;
            hi[i] = h;
            ad[i] = d[(size_t)(t0 + t) * nb + b];
            int s = 0;
            const int words[8] = {l.x, l.y, l.z, l.w, h.x, h.y, h.z, h.w};
#pragma unroll
            for (int k = 0; k < 8; ++k) s = dp4a(words[k], 0x01010101, s);
            c8[i] = 8 * s;
        } else {
            lo[i] = hi[i] = make_int4(0, 0, 0, 0);
            ad[i] = 0.0f;
            c8[i] = 0;
        }
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * kGWarps + (threadIdx.x >> 5), GW = gridDim.x * kGWarps;
    for (int r = gw; r < rows; r += GW) {
        float acc[kGTok];
#pragma unroll
        for (int t = 0; t < kGTok; ++t) acc[t] = 0.0f;
        for (int b = lane; b < nb; b += 32) {
            const size_t bi = (size_t)r * nb + b;
            const uint4 w = __ldg(qs + bi);
            const float dw = half_bits_to_float(__ldg(dsc + bi));
            const int wl[4] = {(int)(w.x & kNib), (int)(w.y & kNib), (int)(w.z & kNib), (int)(w.w & kNib)};
            const int wh[4] = {(int)((w.x >> 4) & kNib), (int)((w.y >> 4) & kNib), (int)((w.z >> 4) & kNib),
                               (int)((w.w >> 4) & kNib)};
#pragma unroll
            for (int t = 0; t < kGTok; ++t) {
                const int4 l = lo[t * nb + b], h = hi[t * nb + b];
                int s = dp4a(wl[0], l.x, 0);
                s = dp4a(wl[1], l.y, s);
                s = dp4a(wl[2], l.z, s);
                s = dp4a(wl[3], l.w, s);
                s = dp4a(wh[0], h.x, s);
                s = dp4a(wh[1], h.y, s);
                s = dp4a(wh[2], h.z, s);
                s = dp4a(wh[3], h.w, s);
                acc[t] = fmaf(dw * ad[t * nb + b], (float)(s - c8[t * nb + b]), acc[t]);
            }
        }
#pragma unroll
        for (int t = 0; t < kGTok; ++t) {
            const float v = warp_sum(acc[t]);
            if (lane == 0 && t < nt) {
                float* dst = y + (size_t)(t0 + t) * rows + r;
                *dst = accumulate ? *dst + v : v;
            }
        }
    }
}

cudaError_t gemm_q4_q8(const mv_weight_s& w, const int8_t* q, const float* d, uint64_t batch, float* y,
                       cudaStream_t s, bool accumulate) {
    if (!batch) return cudaSuccess;
    const size_t smem = (size_t)kGTok * w.nb * (16 + 16 + 4 + 4);
    ensure_smem_attr(gemm_q4_q8_kernel, 220 * 1024);
    const uint64_t ctas = (w.rows + kGWarps - 1) / kGWarps;
    const uint64_t cap = (uint64_t)num_sms() * 2;
    dim3 grid((unsigned)(ctas < cap ? ctas : cap), (unsigned)((batch + kGTok - 1) / kGTok));
    gemm_q4_q8_kernel<<<grid, kGWarps * 32, smem, s>>>(reinterpret_cast<const uint4*>(w.qs), w.d, (int)w.rows,
                                                       (int)w.nb, q, d, (int)batch, y, accumulate ? 1 : 0);
    return cudaGetLastError();
}

}  // namespace mvb
