// common.cuh -- device helpers shared by every memvanta_b200 kernel.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <mutex>
#include <set>
#include <utility>

namespace mvb {

constexpr int kWarp = 32;

// Raises a kernel's dynamic shared-memory limit once per (kernel, device).
template <class Kernel>
inline void ensure_smem_attr(Kernel* k, int bytes) {
    static std::mutex mu;
    static std::set<std::pair<const void*, int>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    const std::pair<const void*, int> key{reinterpret_cast<const void*>(k), dev};
    std::lock_guard<std::mutex> lock(mu);
    if (done.count(key)) return;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    done.insert(key);
}

// ------------------------------------------------- programmatic launches
// Programmatic dependent launch: a kernel launched with launch_pdl may start
// while the previous kernel in the stream is still running.  It must call
// pdl_wait() before reading anything the previous kernel writes (or writing
// anything it reads); work on immutable inputs (weights) can go before it.
// pdl_trigger() lets the next kernel start launching early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" :::); }

template <class... KArgs, class... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// launch_pdl when pdl is true, else a plain launch (full stream order: the
// kernel starts after everything before it in the stream, event waits
// included; its pdl_trigger / pdl_wait are then no-ops).
template <class... KArgs, class... Args>
inline cudaError_t launch_opt(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
    if (pdl) return launch_pdl(kernel, grid, block, smem, s, std::forward<Args>(args)...);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.numAttrs = 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// The same with thread-block clusters of `cluster` CTAs along x.
template <class... KArgs, class... Args>
inline cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                      unsigned cluster, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------- reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// --------------------------------------------------------------- loads
// Weight bytes are read exactly once per launch: bypass L1 allocation and
// go through the read-only path.
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint32_t ld_stream_u32(const void* p) {
    uint32_t r;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}
__device__ __forceinline__ unsigned short ld_stream_u16(const void* p) {
    unsigned short r;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}

__device__ __forceinline__ float half_bits_to_float(unsigned short h) {
    return __half2float(__ushort_as_half(h));
}

// ------------------------------------------------------ integer dot products
__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// Exact float of a signed byte held in the low 8 bits: 2^23 + (b ^ 0x80)
// as a float bit pattern, minus 2^23 + 128.
__device__ __forceinline__ float s8_to_f32(uint32_t word, int byte) {
    const uint32_t u = __byte_perm(word, 0x4B000000u, 0x7650u + byte) ^ 0x80u;
    return __uint_as_float(u) - 8388736.0f;
}
// Exact float of an unsigned byte minus `bias` (bias < 2^22).
__device__ __forceinline__ float u8_to_f32_minus(uint32_t word, int byte, float bias_plus_2p23) {
    const uint32_t u = __byte_perm(word, 0x4B000000u, 0x7650u + byte);
    return __uint_as_float(u) - bias_plus_2p23;
}

// --------------------------------------------------------- fp32 -> fp16
// The reference's own conversion (src/gguf_kernels.cpp:242): add half an
// output ulp to the magnitude and truncate (round-half-up on magnitude), carry
// into the exponent, >= 2^16 (and NaN) -> inf, below 2^-25 -> signed zero.
// Restated bit for bit so KV pages match the reference exactly; the
// hardware's round-to-nearest-even conversion would differ on ties.
__device__ __forceinline__ unsigned short f32_to_f16_ref(float f) {
    const uint32_t x = __float_as_uint(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t mant = x & 0x7fffffu;
    const int e = int((x >> 23) & 0xffu) - 112;
    if (e >= 31) return (unsigned short)(sign | 0x7c00u);
    if (e > 0) return (unsigned short)(sign | (uint32_t(e) << 10) | ((mant + 0x1000u) >> 13));
    if (e < -10) return (unsigned short)sign;
    mant = (mant | 0x800000u) >> (1 - e);
    return (unsigned short)(sign + ((mant + 0x1000u) >> 13));
}

// ------------------------------------------------------ activation quant
// One 32-element block of the reference's quantize_q8
// (src/gguf_kernels.cpp:161-172), one element per lane: mx = max|x|,
// d = mx>0 ? mx/127 : 1, q = clamp(round-half-away(x * (1/d)), -127, 127).
// IEEE division and multiplication (no fast-math) keep it bit-identical.
__device__ __forceinline__ int quant_q8_lane(float v, float& d_out) {
    const float mx = warp_max(fabsf(v));
    const float d = mx > 0.0f ? mx / 127.0f : 1.0f;
    const float inv = 1.0f / d;
    float r = roundf(v * inv);
    r = fminf(fmaxf(r, -127.0f), 127.0f);
    d_out = d;
    return int(r);
}

}  // namespace mvb
