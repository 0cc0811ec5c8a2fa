// gemm.cu -- batched Q4_0 x Q8-activation matmul (prefill), CUDA-core path.
//
// The reference's MEMVANTA_FORCE_Q8_ACT=1 prefill
// (tensor_matmul_batch_v06, src/gguf_kernels.cpp:265-266): every activation
// row is quantised per 32-block (quantize_activations_q8, :174-178) and every
// (token, row) output is the decode row dot dot_q4_q8 (:189) -- a sequential
// FMA chain over the blocks, sum = fma(d_w*d_a, float(isum), sum).
//
// A warp owns a weight row and a tile of T tokens whose quantised
// activations sit in shared memory (16-byte low/high halves per block).  Per
// chunk of 32 blocks each lane loads one 16-byte payload and forms the
// (d_w*d_a, isum) terms for all T tokens (dp4a, bit-exact); then lane t runs
// token t's chain over the chunk in block order, so every output equals the
// reference's bit for bit.
#include "common.cuh"
#include "kernels.cuh"

namespace mvb {

namespace {

constexpr int kGWarps = 8;
constexpr int kGTok = 8;
constexpr int kCb = 33;  // float2 per chain-buffer row (odd: conflict-free)
constexpr uint32_t kNib = 0x0F0F0F0Fu;

__global__ void __launch_bounds__(kGWarps * 32) gemm_q4_q8_kernel(const uint4* __restrict__ qs,
                                                                  const unsigned short* __restrict__ dsc, int rows,
                                                                  int nb, int dstride, const int8_t* __restrict__ q,
                                                                  const float* __restrict__ d, int batch,
                                                                  float* __restrict__ y, int accumulate) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    int4* lo = reinterpret_cast<int4*>(smem_raw);            // [T][nb]
    int4* hi = lo + kGTok * nb;                               // [T][nb]
    float2* dc = reinterpret_cast<float2*>(hi + kGTok * nb);  // [T][nb] (d, 8*sum(q))
    float2* cbuf = dc + kGTok * nb;                           // [warps][T][kCb]
    const int t0 = blockIdx.y * kGTok;
    const int nt = min(kGTok, batch - t0);
    const int K = nb * 32;
    for (int i = threadIdx.x; i < kGTok * nb; i += blockDim.x) {
        const int t = i / nb, b = i % nb;
        if (t < nt) {
            const int8_t* src = q + (size_t)(t0 + t) * K + b * 32;
            const int4 l = *reinterpret_cast<const int4*>(src);
            const int4 h = *reinterpret_cast<const int4*>(src + 16);
            lo[i] = l;
            hi[i] = h;
            int s = 0;
            const int words[8] = {l.x, l.y, l.z, l.w, h.x, h.y, h.z, h.w};
#pragma unroll
            for (int k = 0; k < 8; ++k) s = dp4a(words[k], 0x01010101, s);
            dc[i] = make_float2(d[(size_t)(t0 + t) * nb + b], __int_as_float(8 * s));
        } else {
            lo[i] = hi[i] = make_int4(0, 0, 0, 0);
            dc[i] = make_float2(0.0f, 0.0f);
        }
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float2* cb = cbuf + (size_t)warp * kGTok * kCb;
    const int gw = blockIdx.x * kGWarps + warp, GW = gridDim.x * kGWarps;
    for (int r = gw; r < rows; r += GW) {
        float sum = 0.0f;  // lane t < T: token t's chain
        for (int c = 0; c * 32 < nb; ++c) {
            const int b = c * 32 + lane;
            if (b < nb) {
                const size_t bi = (size_t)r * nb + b;
                const uint4 w = ld_stream_u4(qs + bi);
                const float dw = half_bits_to_float(ld_stream_u16(dsc + (size_t)r * dstride + b));
                const int wl[4] = {(int)(w.x & kNib), (int)(w.y & kNib), (int)(w.z & kNib), (int)(w.w & kNib)};
                const int wh[4] = {(int)((w.x >> 4) & kNib), (int)((w.y >> 4) & kNib), (int)((w.z >> 4) & kNib),
                                   (int)((w.w >> 4) & kNib)};
#pragma unroll
                for (int t = 0; t < kGTok; ++t) {
                    const int4 l = lo[t * nb + b], h = hi[t * nb + b];
                    const float2 e = dc[t * nb + b];
                    int s = dp4a(wl[0], l.x, 0);
                    s = dp4a(wl[1], l.y, s);
                    s = dp4a(wl[2], l.z, s);
                    s = dp4a(wl[3], l.w, s);
                    s = dp4a(wh[0], h.x, s);
                    s = dp4a(wh[1], h.y, s);
                    s = dp4a(wh[2], h.z, s);
                    s = dp4a(wh[3], h.w, s);
                    cb[t * kCb + lane] = make_float2(dw * e.x, (float)(s - __float_as_int(e.y)));
                }
            }
            __syncwarp();
            if (lane < kGTok) {
                const float2* row = cb + lane * kCb;
                const int n = min(32, nb - c * 32);
                for (int k = 0; k < n; ++k) sum = fmaf(row[k].x, row[k].y, sum);
            }
            __syncwarp();
        }
        if (lane < nt) {
            float* dst = y + (size_t)(t0 + lane) * rows + r;
            *dst = accumulate ? *dst + sum : sum;
        }
    }
}

}  // namespace

cudaError_t gemm_q4_q8(const mv_weight_s& w, const int8_t* q, const float* d, uint64_t batch, float* y,
                       cudaStream_t s, bool accumulate) {
    if (!batch) return cudaSuccess;
    const size_t smem = (size_t)kGTok * w.nb * (16 + 16 + 8) + (size_t)kGWarps * kGTok * kCb * 8;
    if (smem > 220 * 1024) return cudaErrorInvalidValue;
    ensure_smem_attr(gemm_q4_q8_kernel, 220 * 1024);
    const uint64_t ctas = (w.rows + kGWarps - 1) / kGWarps;
    const uint64_t cap = (uint64_t)num_sms() * 2;
    dim3 grid((unsigned)(ctas < cap ? ctas : cap), (unsigned)((batch + kGTok - 1) / kGTok));
    gemm_q4_q8_kernel<<<grid, kGWarps * 32, smem, s>>>(reinterpret_cast<const uint4*>(w.qs), w.d, (int)w.rows,
                                                       (int)w.nb, (int)w.dstride, q, d, (int)batch, y,
                                                       accumulate ? 1 : 0);
    return cudaGetLastError();
}

}  // namespace mvb
