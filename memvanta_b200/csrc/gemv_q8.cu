// gemv_q8.cu -- decode GEMV y = W x for a Q8_0 weight with fp32 x: the
// reference's tensor_matvec Q8_0 branch (src/gguf_kernels.cpp:247 ->
// dot_q8_0_fp32 :111-120), which keeps fp32 activations.
//
// Per 32-element block the reference forms s = sum_k float(q_k) * x_k in fp32
// and adds d * s to the row sum; the GPU forms the same block sums (a
// different fp32 summation order) and sums d * s over a row's blocks in a
// warp tree, so results agree to ~1e-6 relative (the tolerance is 1e-3).
//
// HBM-bound.  A warp owns a row at a time: lane l takes blocks l, l+32, ...
// (32 contiguous int8 per block, so one row is read by fully coalesced
// 128-bit loads), four blocks per lane per pass, and the next pass (of this
// row or the next) is requested before the current one is computed, so each
// warp keeps 8 KB in flight.  x sits in shared
// memory with the 16-byte chunks of block b rotated by b, so the 8 lanes of a
// quarter-warp (8 consecutive blocks) read 8 different bank groups.  int8 ->
// float is exact by the 2^23 trick (one byte permute per value and one packed
// subtract per pair), the FMAs are packed f32x2.
#include "common.cuh"
#include "kernels.cuh"
#include "tc.cuh"

namespace mvb {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxBlk = 4;  // blocks per lane kept in registers (K <= 4096 in one pass)

__device__ __forceinline__ uint64_t pk2(float a, float b) {
    return (uint64_t)__float_as_uint(a) | ((uint64_t)__float_as_uint(b) << 32);
}

// sum_k float(q_k) * x_k over one 32-element block (payload p, x chunks xs4
// rotated by `rot`), with packed pairs: acc2 carries two partial sums.
__device__ __forceinline__ float block_dot(const uint4 p0, const uint4 p1, const float4* xb, int rot) {
    const uint32_t w[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
    const uint64_t bias = pk2(8388736.0f, 8388736.0f);  // 2^23 + 128
    uint64_t acc = 0ull;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const uint32_t u = w[c] ^ 0x80808080u;  // signed byte b -> b + 128 as an unsigned byte
        const float4 xv = xb[(c + rot) & 7];
        // float bits 0x4B0000uu = 2^23 + u (byte permute: byte k of u, then 00 00 4B)
        const uint64_t q01 = (uint64_t)__byte_perm(u, 0x4B000000u, 0x7650u) |
                             ((uint64_t)__byte_perm(u, 0x4B000000u, 0x7651u) << 32);
        const uint64_t q23 = (uint64_t)__byte_perm(u, 0x4B000000u, 0x7652u) |
                             ((uint64_t)__byte_perm(u, 0x4B000000u, 0x7653u) << 32);
        acc = tc::f2_fma(tc::f2_sub(q01, bias), pk2(xv.x, xv.y), acc);
        acc = tc::f2_fma(tc::f2_sub(q23, bias), pk2(xv.z, xv.w), acc);
    }
    return __uint_as_float((uint32_t)acc) + __uint_as_float((uint32_t)(acc >> 32));
}

// Work items of a warp: (row, pass) with pass p covering blocks
// 128 p + lane + 32 j (j < 4) of the row; the item after the current one is
// requested before the current one is computed.
__global__ void __launch_bounds__(kThreads) gemv_q8_kernel(const uint4* __restrict__ qs,
                                                           const unsigned short* __restrict__ dsc, int rows,
                                                           int nb, const float* __restrict__ x,
                                                           float* __restrict__ y) {
    extern __shared__ __align__(16) float4 xs4[];  // [nb][8] rotated chunks
    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * kWarps + (threadIdx.x >> 5), GW = gridDim.x * kWarps;
    const int npass = (nb + 32 * kMaxBlk - 1) / (32 * kMaxBlk);
    pdl_trigger();
    uint4 cur[kMaxBlk][2], nxt[kMaxBlk][2];
    unsigned short dcur[kMaxBlk], dnxt[kMaxBlk];
    auto load = [&](int r, int pass, uint4 (&p)[kMaxBlk][2], unsigned short (&d)[kMaxBlk]) {
#pragma unroll
        for (int j = 0; j < kMaxBlk; ++j) {
            const int b = pass * 32 * kMaxBlk + lane + 32 * j;
            if (b < nb) {
                const uint4* src = qs + ((size_t)r * nb + b) * 2;
                p[j][0] = ld_stream_u4(src);
                p[j][1] = ld_stream_u4(src + 1);
                d[j] = ld_stream_u16(dsc + (size_t)r * nb + b);
            }
        }
    };
    int r = gw, pass = 0;
    // the first item: weights are immutable, requested before the wait
    if (r < rows) load(r, 0, cur, dcur);
    pdl_wait();
    for (int i = threadIdx.x; i < nb * 8; i += kThreads) {
        const int b = i >> 3, c = i & 7;
        xs4[b * 8 + ((c + b) & 7)] = reinterpret_cast<const float4*>(x)[i];
    }
    __syncthreads();
    float acc = 0.0f;
    while (r < rows) {
        int rn = r, pn = pass + 1;
        if (pn == npass) rn += GW, pn = 0;
        if (rn < rows) load(rn, pn, nxt, dnxt);
#pragma unroll
        for (int j = 0; j < kMaxBlk; ++j) {
            const int b = pass * 32 * kMaxBlk + lane + 32 * j;
            if (b < nb) acc = fmaf(half_bits_to_float(dcur[j]), block_dot(cur[j][0], cur[j][1], xs4 + b * 8, b), acc);
        }
        if (pass == npass - 1) {
            acc = warp_sum(acc);
            if (lane == 0) y[r] = acc;
            acc = 0.0f;
        }
#pragma unroll
        for (int j = 0; j < kMaxBlk; ++j) {
            cur[j][0] = nxt[j][0];
            cur[j][1] = nxt[j][1];
            dcur[j] = dnxt[j];
        }
        r = rn;
        pass = pn;
    }
}

}  // namespace

cudaError_t gemv_q8_0(const mv_weight_s& w, const float* x, float* y, cudaStream_t s) {
    if (w.type != 8 || w.cols % 32) return cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(x) % 16) return cudaErrorInvalidValue;
    const size_t smem = w.cols * sizeof(float);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    ensure_smem_attr(gemv_q8_kernel, 200 * 1024);
    const uint64_t ctas = (w.rows + kWarps - 1) / kWarps, cap = (uint64_t)num_sms() * 4;
    return launch_pdl(gemv_q8_kernel, dim3((unsigned)(ctas < cap ? ctas : cap)), dim3(kThreads), smem, s,
                      reinterpret_cast<const uint4*>(w.qs), (const unsigned short*)w.d, (int)w.rows, (int)w.nb, x,
                      y);
}

}  // namespace mvb
