// gemv_q6k.cu -- decode GEMV y = W x for a Q6_K weight with fp32 x: the
// reference's output head (tensor_matvec Q6_K branch, src/gguf_kernels.cpp:248
// -> dot_q6_k_fp32 :138-146 -> q6_k_value :122-136).
//
// A warp owns a row; lane l owns one 128-element half ("group") of a
// 256-element super-block: 64 bytes of low nibbles, 32 bytes of high bits,
// 8 sub-block scales -- four 128-bit, two 128-bit and one 64-bit load, plus
// the super-block's fp16 scale, all issued at once, and the next row's loads
// are issued before the current row is computed.  Element (slot s, j) of a
// group (s = 0..3, j = 0..31) is
//   lo = (ql[(s&1)*32 + j] >> (s<2 ? 0 : 4)) & 15,  hi = (qh[j] >> 2s) & 3,
//   q6 = (lo | hi<<4) - 32,  scale = scales[2s + j/16],
// done four bytes at a time.  Per 16 elements (one sub-block scale) the
// products q6*x are summed in fp32 and scaled by d*scale; the reference sums
// w*x in double, which this matches to ~1e-7 relative (tolerance 5e-3).
//
// x sits in shared memory rotated within each 128-float region r by 4*r
// floats, so the 32 lanes (32 different regions) reading the same offset hit
// 8 distinct 16-byte bank groups per quarter-warp.
#include "common.cuh"
#include "kernels.cuh"

namespace mvb {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr uint32_t kNib = 0x0F0F0F0Fu;

struct Group {
    uint4 ql[4];
    uint4 qh[2];
    uint2 sc;
    unsigned short d;
};

__device__ __forceinline__ void load_group(Group& g, const mv_weight_s& w, int row, int h, bool valid) {
    if (!valid) return;
    const uint64_t sb = (uint64_t)row * w.nb + (h >> 1);
    const int grp = h & 1;
    const uint4* ql = reinterpret_cast<const uint4*>(w.qs + sb * 128 + grp * 64);
    const uint4* qh = reinterpret_cast<const uint4*>(w.qh + sb * 64 + grp * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i) g.ql[i] = ld_stream_u4(ql + i);
    g.qh[0] = ld_stream_u4(qh);
    g.qh[1] = ld_stream_u4(qh + 1);
    const uint2* sc = reinterpret_cast<const uint2*>(w.sc + sb * 16 + grp * 8);
    uint2 s;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(s.x), "=r"(s.y) : "l"(sc));
    g.sc = s;
    g.d = ld_stream_u16(w.d + sb);
}

__device__ __forceinline__ uint32_t word_of(const uint4* v, int i) {
    const uint4 q = v[i >> 2];
    switch (i & 3) {
        case 0: return q.x;
        case 1: return q.y;
        case 2: return q.z;
        default: return q.w;
    }
}

// Dot of one 128-element group with x (region `reg` of the rotated copy).
__device__ __forceinline__ float group_dot(const Group& g, const float* xs, int reg) {
    const float d = half_bits_to_float(g.d);
    float acc = 0.0f;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
#pragma unroll
        for (int half16 = 0; half16 < 2; ++half16) {
            float part = 0.0f;
#pragma unroll
            for (int jc = half16 * 4; jc < half16 * 4 + 4; ++jc) {
                const uint32_t qlw = word_of(g.ql, (s & 1) * 8 + jc);
                const uint32_t qhw = word_of(g.qh, jc);
                const uint32_t q6 = ((s < 2 ? qlw : qlw >> 4) & kNib) | (((qhw >> (2 * s)) & 0x03030303u) << 4);
                const int k = s * 32 + jc * 4;  // logical offset in the region
                const float4 xv = *reinterpret_cast<const float4*>(xs + reg * 128 + ((k + 4 * reg) & 127));
                part = fmaf(u8_to_f32_minus(q6, 0, 8388640.0f), xv.x, part);
                part = fmaf(u8_to_f32_minus(q6, 1, 8388640.0f), xv.y, part);
                part = fmaf(u8_to_f32_minus(q6, 2, 8388640.0f), xv.z, part);
                part = fmaf(u8_to_f32_minus(q6, 3, 8388640.0f), xv.w, part);
            }
            const int si = s * 2 + half16;
            const int8_t scv = (int8_t)((si < 4 ? g.sc.x : g.sc.y) >> (8 * (si & 3)));
            acc = fmaf(d * (float)scv, part, acc);  // d*scale as the reference forms it
        }
    }
    return acc;
}

__global__ void __launch_bounds__(kThreads) gemv_q6k_kernel(mv_weight_s w, const float* __restrict__ x,
                                                            float* __restrict__ y) {
    extern __shared__ __align__(16) float xs[];
    const int K = (int)w.cols, regions = K / 128;
    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * kWarps + (threadIdx.x >> 5), GW = gridDim.x * kWarps;
    const int rows = (int)w.rows;
    // regions == number of 128-element groups in a row; lane l takes group l
    // (prefetched one row ahead) and, for K > 4096, groups l+32, l+64, ...
    pdl_trigger();
    Group cur, nxt;
    int r = gw;
    if (r < rows) load_group(cur, w, r, lane, lane < regions);  // weights: before the dependency wait
    pdl_wait();
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
        const int rr = i / 128, k = i % 128;
        xs[rr * 128 + ((k + 4 * rr) & 127)] = x[i];
    }
    __syncthreads();
    for (; r < rows; r += GW) {
        const int rn = r + GW;
        if (rn < rows) load_group(nxt, w, rn, lane, lane < regions);
        float acc = 0.0f;
        if (lane < regions) acc = group_dot(cur, xs, lane);
        for (int h = lane + 32; h < regions; h += 32) {
            Group g;
            load_group(g, w, r, h, true);
            acc += group_dot(g, xs, h);
        }
        acc = warp_sum(acc);
        if (lane == 0) y[r] = acc;
        cur = nxt;
    }
}

}  // namespace

cudaError_t gemv_q6k(const mv_weight_s& w, const float* x, float* y, cudaStream_t s) {
    if (w.type != 14 || w.cols % 256) return cudaErrorInvalidValue;
    const size_t smem = w.cols * sizeof(float);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    ensure_smem_attr(gemv_q6k_kernel, 200 * 1024);
    const uint64_t ctas = (w.rows + kWarps - 1) / kWarps, cap = (uint64_t)num_sms() * 4;
    return launch_pdl(gemv_q6k_kernel, dim3((unsigned)(ctas < cap ? ctas : cap)), dim3(kThreads), smem, s, w, x, y);
}

}  // namespace mvb
