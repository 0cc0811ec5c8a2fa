// ops.cu -- the element-wise / row ops around the matmuls
// (src/llama_model.cpp:237-258): RMSNorm, RoPE, SiLU gate, residual add,
// fp32 -> fp16 with the reference rounding, and the greedy argmax of
// Sampler::sample (src/llama_model.cpp:60).
#include "common.cuh"
#include "kernels.cuh"

namespace mvb {

// RMSNorm of one row per CTA: double sum of squares,
// inv = 1/sqrt(float(ss/n) + eps), out = x*inv*w (two roundings, as the
// reference evaluates `x[i]*inv*w[i]`).
__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w, int n, float eps,
                               float* __restrict__ out) {
    __shared__ double red[32];
    pdl_trigger();
    pdl_wait();
    const float* xr = x + (size_t)blockIdx.x * n;
    float* o = out + (size_t)blockIdx.x * n;
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const double v = (double)xr[i];
        ss += v * v;
    }
    ss = warp_sum_d(ss);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (warp == 0) {
        double t = lane < nw ? red[lane] : 0.0;
        t = warp_sum_d(t);
        if (lane == 0) red[0] = t;
    }
    __syncthreads();
    const float inv = 1.0f / sqrtf((float)(red[0] / (double)n) + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] = xr[i] * inv * w[i];
}

cudaError_t rmsnorm_rows(const float* x, const float* w, uint64_t rows, uint64_t n, float eps, float* out,
                         cudaStream_t s) {
    if (!rows) return cudaSuccess;
    return launch_pdl(rmsnorm_kernel, dim3((unsigned)rows), dim3(512), 0, s, x, w, (int)n, eps, out);
}

// Half-split RoPE: pairs (i, i+hd/2) of every head rotate by row pos of the
// host-built tables.  The reference's GCC build evaluates
// `x0*c - x1*s` as fma(x0, c, -(x1*s)) and `x0*s + x1*c` as fma(x0, s, x1*c);
// the explicit _rn intrinsics pin exactly those roundings.
__device__ __forceinline__ void rope_pair(float* b, int i, int half, float c, float s) {
    const float x0 = b[i], x1 = b[i + half];
    b[i] = __fmaf_rn(x0, c, -__fmul_rn(x1, s));
    b[i + half] = __fmaf_rn(x0, s, __fmul_rn(x1, c));
}

__global__ void rope_kernel(float* __restrict__ q, int n_head, float* __restrict__ k, int n_head_kv, int hd,
                            const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                            const int32_t* __restrict__ pos) {
    const int r = blockIdx.x, half = hd / 2;
    const int p = pos[r];
    const float* co = cos_t + (size_t)p * half;
    const float* si = sin_t + (size_t)p * half;
    float* qr = q + (size_t)r * n_head * hd;
    float* kr = k + (size_t)r * n_head_kv * hd;
    for (int i = threadIdx.x; i < (n_head + n_head_kv) * half; i += blockDim.x) {
        const int h = i / half, j = i % half;
        if (h < n_head) rope_pair(qr + h * hd, j, half, co[j], si[j]);
        else rope_pair(kr + (h - n_head) * hd, j, half, co[j], si[j]);
    }
}

cudaError_t rope_rows(float* q, uint64_t n_head, float* k, uint64_t n_head_kv, uint64_t hd, uint64_t rows,
                      const float* cos_t, const float* sin_t, const int32_t* pos, cudaStream_t s) {
    if (!rows) return cudaSuccess;
    rope_kernel<<<(unsigned)rows, 256, 0, s>>>(q, (int)n_head, k, (int)n_head_kv, (int)hd, cos_t, sin_t, pos);
    return cudaGetLastError();
}

__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ o,
                                uint64_t n) {
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const float x = g[i];
        o[i] = (x / (1.0f + expf(-x))) * u[i];
    }
}
__global__ void add_kernel(float* __restrict__ x, const float* __restrict__ y, uint64_t n) {
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        x[i] += y[i];
}
__global__ void f16_kernel(const float* __restrict__ x, uint16_t* __restrict__ h, uint64_t n) {
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        h[i] = f32_to_f16_ref(x[i]);
}

static unsigned ew_grid(uint64_t n) {
    const uint64_t g = (n + 255) / 256, cap = (uint64_t)num_sms() * 8;
    return (unsigned)(g < cap ? (g ? g : 1) : cap);
}

cudaError_t silu_mul(const float* g, const float* u, float* out, uint64_t n, cudaStream_t s) {
    silu_mul_kernel<<<ew_grid(n), 256, 0, s>>>(g, u, out, n);
    return cudaGetLastError();
}
cudaError_t add_inplace(float* x, const float* y, uint64_t n, cudaStream_t s) {
    add_kernel<<<ew_grid(n), 256, 0, s>>>(x, y, n);
    return cudaGetLastError();
}
cudaError_t f32_to_f16_ref(const float* x, uint16_t* h, uint64_t n, cudaStream_t s) {
    f16_kernel<<<ew_grid(n), 256, 0, s>>>(x, h, n);
    return cudaGetLastError();
}

// Greedy argmax: first index of the maximum, as std::max_element.
// Single CTA; (value, index) pairs reduce with ties going to the lower index.
__device__ __forceinline__ void am_merge(float& v, int& i, float v2, int i2) {
    if (v2 > v || (v2 == v && i2 < i)) {
        v = v2;
        i = i2;
    }
}
__global__ void argmax_kernel(const float* __restrict__ x, int n, int32_t* __restrict__ out) {
    __shared__ float sv[32];
    __shared__ int si[32];
    float v = -INFINITY;
    int idx = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) am_merge(v, idx, x[i], i);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
        am_merge(v, idx, v2, i2);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (lane == 0) {
        sv[warp] = v;
        si[warp] = idx;
    }
    __syncthreads();
    if (warp == 0) {
        v = lane < nw ? sv[lane] : -INFINITY;
        idx = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
            const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
            am_merge(v, idx, v2, i2);
        }
        if (lane == 0) *out = idx == 0x7fffffff ? 0 : idx;
    }
}

cudaError_t argmax_f32(const float* x, uint64_t n, int32_t* out_idx, cudaStream_t s) {
    argmax_kernel<<<1, 1024, 0, s>>>(x, (int)n, out_idx);
    return cudaGetLastError();
}

}  // namespace mvb
