// internal.cu -- device twins of the reference's internal-format kernels
// (include/memvanta/quant.hpp, src/quant.cpp, src/quant_kernels.cpp,
// src/matmul.cpp): the non-GGUF blocks the reference's kernel_bench and
// streaming engine use,
//   BlockQ8_0: 36 bytes {float d; int8 qs[32]}
//   BlockQ4_0: 20 bytes {float d; uint8 qs[16]}, element 2i = low nibble of
//              qs[i], element 2i+1 = high nibble (interleaved, unlike GGUF),
// read in place from device memory (no repack) with the reference's
// arithmetic order, so the outputs match it bit for bit:
//   * quantize: d = amax/127 (Q8) or amax/7 (Q4), zero block when amax == 0,
//     q = clamp(nearbyint(x * (1/d))) -- round half to even, unlike GGUF's
//     quantize_q8 (src/quant.cpp:44-85);
//   * dot_q4_q8: per block sum += (float(isum) * d_a) * d_x, uncontracted
//     (src/quant_kernels.cpp:52-66);
//   * dot_q4_0 / dot_q8_0 against fp32 x: eight FMA lanes over the block's
//     elements (lane l takes l, l+8, l+16, l+24), a left-to-right sum from
//     0, then sum = fma(s, d, sum) (src/quant.cpp:87-156);
//   * matvec_f32: a sequential uncontracted fp32 row dot (src/matmul.cpp:6-8).
// One warp per output row: lanes compute the per-block terms in parallel and
// every lane then runs the row's chain over them in block order (shuffles),
// which is the reference's sequence of roundings.
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "common.cuh"
#include "kernels.cuh"
#include "memvanta_b200.h"

namespace mvb {
namespace {

constexpr int kIntThreads = 256;

__device__ __forceinline__ uint32_t ld_u32(const uint8_t* p) {  // 4-byte aligned
    return *reinterpret_cast<const uint32_t*>(p);
}

// --------------------------------------------------------------- quantise
// One warp per 32-element block, lane = element.
__global__ void int_quantize_q8_0_kernel(const float* __restrict__ x, uint64_t nblocks, uint8_t* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x / 32);
    for (uint64_t b = blockIdx.x * (uint64_t)(blockDim.x / 32) + threadIdx.x / 32; b < nblocks; b += warps) {
        const float v = x[b * 32 + lane];
        float amax = fabsf(v);
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float d = amax == 0.0f ? 0.0f : __fdiv_rn(amax, 127.0f);
        uint8_t* blk = out + b * 36;
        if (lane == 0) *reinterpret_cast<float*>(blk) = d;
        int q = 0;
        if (d != 0.0f) {
            const float id = __fdiv_rn(1.0f, d);
            q = __float2int_rn(__fmul_rn(v, id));  // nearbyint: ties to even
            q = q < -127 ? -127 : q > 127 ? 127 : q;
        }
        blk[4 + lane] = (uint8_t)(int8_t)q;
    }
}

__global__ void int_quantize_q4_0_kernel(const float* __restrict__ x, uint64_t nblocks, uint8_t* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x / 32);
    for (uint64_t b = blockIdx.x * (uint64_t)(blockDim.x / 32) + threadIdx.x / 32; b < nblocks; b += warps) {
        const float v = x[b * 32 + lane];
        float amax = fabsf(v);
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float d = amax == 0.0f ? 0.0f : __fdiv_rn(amax, 7.0f);
        uint8_t* blk = out + b * 20;
        if (lane == 0) *reinterpret_cast<float*>(blk) = d;
        int q = 0;
        if (d != 0.0f) {
            const float id = __fdiv_rn(1.0f, d);
            q = __float2int_rn(__fmul_rn(v, id));
            q = (q < -8 ? -8 : q > 7 ? 7 : q) + 8;
        }
        const int hi = __shfl_down_sync(0xffffffffu, q, 1);
        // the reference clears the nibbles of a zero block (d == 0): q = 0 there
        if ((lane & 1) == 0) blk[4 + lane / 2] = d == 0.0f ? 0 : (uint8_t)(q | (hi << 4));
    }
}

// ------------------------------------------------------------ block terms
// dot_q4_q8 term of one block: (float(isum) * d_a) * d_x.
__device__ __forceinline__ float term_q4_q8(const uint8_t* a, const uint8_t* xq) {
    int isum = 0;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const uint32_t nib = ld_u32(a + 4 + 4 * w);
        const uint32_t x0 = ld_u32(xq + 4 + 8 * w), x1 = ld_u32(xq + 8 + 8 * w);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int byte = (nib >> (8 * i)) & 0xFF;
            const uint32_t xw = i < 2 ? x0 : x1;
            const int e0 = (int)(int8_t)(xw >> (16 * (i & 1)));
            const int e1 = (int)(int8_t)(xw >> (16 * (i & 1) + 8));
            isum += ((byte & 15) - 8) * e0 + ((byte >> 4) - 8) * e1;
        }
    }
    const float ad = __uint_as_float(ld_u32(a)), xd = __uint_as_float(ld_u32(xq));
    return __fmul_rn(__fmul_rn((float)isum, ad), xd);
}

// Eight-lane FMA dot of one block against fp32 x, then the left-to-right sum
// from 0 (hsum8).  q(k) is the block's k-th element as a float.
template <class Q>
__device__ __forceinline__ float block_hsum8(const float* __restrict__ xb, Q q) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < 32; k += 4) {
        const float4 xv = *reinterpret_cast<const float4*>(xb + k);
        acc[(k + 0) % 8] = __fmaf_rn(q(k + 0), xv.x, acc[(k + 0) % 8]);
        acc[(k + 1) % 8] = __fmaf_rn(q(k + 1), xv.y, acc[(k + 1) % 8]);
        acc[(k + 2) % 8] = __fmaf_rn(q(k + 2), xv.z, acc[(k + 2) % 8]);
        acc[(k + 3) % 8] = __fmaf_rn(q(k + 3), xv.w, acc[(k + 3) % 8]);
    }
    float s = 0.0f;
#pragma unroll
    for (int l = 0; l < 8; ++l) s = __fadd_rn(s, acc[l]);
    return s;
}

// ---------------------------------------------------------------- matvecs
// y[r] = chain over blocks b of term(r, b); FMA form: sum = fma(h, d, sum),
// add form: sum = sum + t.  One warp per (row, batch item).
template <int KIND>  // 0: q4 x q8 (add form), 1: q4 x f32, 2: q8 x f32 (FMA form)
__global__ void __launch_bounds__(kIntThreads) int_matvec_kernel(const uint8_t* __restrict__ A,
                                                                 const void* __restrict__ x, float* __restrict__ y,
                                                                 int rows, int nb, int batch) {
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (kIntThreads / 32);
    const int bstride = KIND == 2 ? 36 : 20;
    for (uint64_t wi = blockIdx.x * (uint64_t)(kIntThreads / 32) + threadIdx.x / 32; wi < (uint64_t)rows * batch;
         wi += warps) {
        const int r = (int)(wi % rows), t = (int)(wi / rows);
        const uint8_t* arow = A + (size_t)r * nb * bstride;
        float sum = 0.0f;
        for (int b0 = 0; b0 < nb; b0 += 32) {
            const int b = b0 + lane;
            float h = 0.0f, d = 0.0f;
            if (b < nb) {
                const uint8_t* a = arow + (size_t)b * bstride;
                if (KIND == 0) {
                    h = term_q4_q8(a, static_cast<const uint8_t*>(x) + (size_t)b * 36);
                } else {
                    const float* xb = static_cast<const float*>(x) + (size_t)t * nb * 32 + (size_t)b * 32;
                    d = __uint_as_float(ld_u32(a));
                    if (KIND == 1) {
                        h = block_hsum8(xb, [&](int k) {
                            const int byte = a[4 + k / 2];
                            return (float)(((k & 1) ? (byte >> 4) : (byte & 15)) - 8);
                        });
                    } else {
                        h = block_hsum8(xb, [&](int k) { return (float)(int8_t)a[4 + k]; });
                    }
                }
            }
            const int n = min(32, nb - b0);
            for (int k = 0; k < n; ++k) {  // every lane runs the chain (identical values)
                const float hk = __shfl_sync(0xffffffffu, h, k);
                if (KIND == 0) {
                    sum = __fadd_rn(sum, hk);
                } else {
                    const float dk = __shfl_sync(0xffffffffu, d, k);
                    sum = __fmaf_rn(hk, dk, sum);
                }
            }
        }
        if (lane == 0) y[(size_t)t * rows + r] = sum;
    }
}

// matvec_f32: s = s + A[r][c]*x[c] for c in order, no contraction.  The
// products come from the lanes, the sum is the row's chain.
__global__ void __launch_bounds__(kIntThreads) matvec_f32_kernel(const float* __restrict__ A,
                                                                 const float* __restrict__ x, float* __restrict__ y,
                                                                 int rows, int cols) {
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (kIntThreads / 32);
    for (uint64_t r = blockIdx.x * (uint64_t)(kIntThreads / 32) + threadIdx.x / 32; r < (uint64_t)rows; r += warps) {
        const float* ar = A + r * (uint64_t)cols;
        float s = 0.0f;
        for (int c0 = 0; c0 < cols; c0 += 32) {
            const int c = c0 + lane;
            const float p = c < cols ? __fmul_rn(ar[c], x[c]) : 0.0f;
            const int n = min(32, cols - c0);
            for (int k = 0; k < n; ++k) s = __fadd_rn(s, __shfl_sync(0xffffffffu, p, k));
        }
        if (lane == 0) y[r] = s;
    }
}

unsigned grid_warps(uint64_t warps) {
    const uint64_t ctas = (warps + kIntThreads / 32 - 1) / (kIntThreads / 32);
    const uint64_t cap = (uint64_t)num_sms() * 8;
    return (unsigned)(ctas < cap ? (ctas ? ctas : 1) : cap);
}

int fail(int code, const std::string& msg) {
    set_last_error(msg);
    return code;
}
int done(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return MV_OK;
    cudaGetLastError();
    return fail(MV_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}
bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3) == 0; }

}  // namespace
}  // namespace mvb

using namespace mvb;

extern "C" {

MV_API int mv_int_quantize_q8_0(const float* x_dev, uint64_t n, void* out36_dev, void* stream) {
    if (!x_dev || !out36_dev || n % 32 || !aligned4(out36_dev)) return fail(MV_ERR_INVALID, "quantize_q8_0: n % 32 or pointers");
    const uint64_t nb = n / 32;
    if (!nb) return MV_OK;
    int_quantize_q8_0_kernel<<<grid_warps(nb), kIntThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        x_dev, nb, static_cast<uint8_t*>(out36_dev));
    return done(cudaGetLastError(), "int_quantize_q8_0");
}

MV_API int mv_int_quantize_q4_0(const float* x_dev, uint64_t n, void* out20_dev, void* stream) {
    if (!x_dev || !out20_dev || n % 32 || !aligned4(out20_dev)) return fail(MV_ERR_INVALID, "quantize_q4_0: n % 32 or pointers");
    const uint64_t nb = n / 32;
    if (!nb) return MV_OK;
    int_quantize_q4_0_kernel<<<grid_warps(nb), kIntThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        x_dev, nb, static_cast<uint8_t*>(out20_dev));
    return done(cudaGetLastError(), "int_quantize_q4_0");
}

static int int_matvec(int kind, const void* A, const void* x, float* y, uint64_t rows, uint64_t cols, uint64_t batch,
                      void* stream) {
    if (!A || !x || !y || cols % 32 || !aligned4(A) || !aligned4(x) || (kind != 0 && (reinterpret_cast<uintptr_t>(x) & 15)))
        return fail(MV_ERR_INVALID, "internal matvec: cols % 32 or pointer alignment");
    if (rows >= (1ull << 31) || cols / 32 >= (1ull << 31) || batch >= (1ull << 31))
        return fail(MV_ERR_INVALID, "internal matvec: size");
    if (!rows || !cols || !batch) return MV_OK;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const unsigned g = grid_warps(rows * batch);
    const uint8_t* a = static_cast<const uint8_t*>(A);
    if (kind == 0) int_matvec_kernel<0><<<g, kIntThreads, 0, s>>>(a, x, y, (int)rows, (int)(cols / 32), (int)batch);
    else if (kind == 1) int_matvec_kernel<1><<<g, kIntThreads, 0, s>>>(a, x, y, (int)rows, (int)(cols / 32), (int)batch);
    else int_matvec_kernel<2><<<g, kIntThreads, 0, s>>>(a, x, y, (int)rows, (int)(cols / 32), (int)batch);
    return done(cudaGetLastError(), "internal matvec");
}

MV_API int mv_int_matvec_q4_q8(const void* A20_dev, const void* x36_dev, float* y_dev, uint64_t rows, uint64_t cols,
                               void* stream) {
    return int_matvec(0, A20_dev, x36_dev, y_dev, rows, cols, 1, stream);
}
MV_API int mv_int_matvec_q4_0(const void* A20_dev, const float* x_dev, float* y_dev, uint64_t rows, uint64_t cols,
                              void* stream) {
    return int_matvec(1, A20_dev, x_dev, y_dev, rows, cols, 1, stream);
}
MV_API int mv_int_matvec_q8_0(const void* A36_dev, const float* x_dev, float* y_dev, uint64_t rows, uint64_t cols,
                              void* stream) {
    return int_matvec(2, A36_dev, x_dev, y_dev, rows, cols, 1, stream);
}
MV_API int mv_int_matmul_q4_0_batch(const void* A20_dev, const float* x_dev, float* y_dev, uint64_t rows,
                                    uint64_t cols, uint64_t batch, void* stream) {
    return int_matvec(1, A20_dev, x_dev, y_dev, rows, cols, batch, stream);
}

MV_API int mv_matvec_f32(const float* A_dev, const float* x_dev, float* y_dev, uint64_t rows, uint64_t cols,
                         void* stream) {
    if (!A_dev || !x_dev || !y_dev) return fail(MV_ERR_INVALID, "matvec_f32: null pointer");
    if (rows >= (1ull << 31) || cols >= (1ull << 31)) return fail(MV_ERR_INVALID, "matvec_f32: size");
    if (!rows || !cols) return MV_OK;
    matvec_f32_kernel<<<grid_warps(rows), kIntThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        A_dev, x_dev, y_dev, (int)rows, (int)cols);
    return done(cudaGetLastError(), "matvec_f32");
}

}  // extern "C"
