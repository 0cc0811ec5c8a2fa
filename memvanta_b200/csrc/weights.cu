// weights.cu -- GGUF block repack / unpack, row dequantisation (embedding
// lookup) and the per-row Q8 activation quantiser.
#include "common.cuh"
#include "kernels.cuh"

namespace mvb {

int num_sms() {
    static thread_local int dev = -1, sms = 0;
    int d = 0;
    cudaGetDevice(&d);
    if (d != dev) {
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d);
        dev = d;
    }
    return sms;
}

// ------------------------------------------------------------- repack
// One thread per block.  Raw GGUF bytes are read with byte loads (18/34/210
// byte blocks are unaligned); the planes are written with wide stores.
__global__ void repack_q4_kernel(const uint8_t* __restrict__ raw, uint8_t* __restrict__ qs, uint16_t* __restrict__ d,
                                 uint64_t nblocks, uint64_t nb, uint64_t dstride) {
    for (uint64_t b = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; b < nblocks; b += (uint64_t)gridDim.x * blockDim.x) {
        const uint8_t* p = raw + b * 18;
        d[(b / nb) * dstride + b % nb] = (uint16_t)(p[0] | (p[1] << 8));
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            w[i] = p[2 + 4 * i] | (p[3 + 4 * i] << 8) | (p[4 + 4 * i] << 16) | ((uint32_t)p[5 + 4 * i] << 24);
        reinterpret_cast<uint4*>(qs)[b] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}
__global__ void unpack_q4_kernel(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ d, uint8_t* __restrict__ raw,
                                 uint64_t nblocks, uint64_t nb, uint64_t dstride) {
    for (uint64_t b = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; b < nblocks; b += (uint64_t)gridDim.x * blockDim.x) {
        uint8_t* p = raw + b * 18;
        const uint16_t dv = d[(b / nb) * dstride + b % nb];
        p[0] = dv & 0xff;
        p[1] = dv >> 8;
        for (int i = 0; i < 16; ++i) p[2 + i] = qs[b * 16 + i];
    }
}
__global__ void repack_q8_kernel(const uint8_t* __restrict__ raw, uint8_t* __restrict__ qs, uint16_t* __restrict__ d,
                                 uint64_t nblocks) {
    for (uint64_t b = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; b < nblocks; b += (uint64_t)gridDim.x * blockDim.x) {
        const uint8_t* p = raw + b * 34;
        d[b] = (uint16_t)(p[0] | (p[1] << 8));
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
            w[i] = p[2 + 4 * i] | (p[3 + 4 * i] << 8) | (p[4 + 4 * i] << 16) | ((uint32_t)p[5 + 4 * i] << 24);
        uint4* o = reinterpret_cast<uint4*>(qs + b * 32);
        o[0] = make_uint4(w[0], w[1], w[2], w[3]);
        o[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
}
__global__ void unpack_q8_kernel(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ d, uint8_t* __restrict__ raw,
                                 uint64_t nblocks) {
    for (uint64_t b = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; b < nblocks; b += (uint64_t)gridDim.x * blockDim.x) {
        uint8_t* p = raw + b * 34;
        p[0] = d[b] & 0xff;
        p[1] = d[b] >> 8;
        for (int i = 0; i < 32; ++i) p[2 + i] = qs[b * 32 + i];
    }
}
// Q6_K: 210 B {ql[128], qh[64], scales[16], d} -> four planes.
__global__ void repack_q6k_kernel(const uint8_t* __restrict__ raw, uint8_t* __restrict__ ql, uint8_t* __restrict__ qh,
                                  int8_t* __restrict__ sc, uint16_t* __restrict__ d, uint64_t nblocks) {
    for (uint64_t b = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; b < nblocks; b += (uint64_t)gridDim.x * blockDim.x) {
        const uint8_t* p = raw + b * 210;
        for (int i = 0; i < 128; ++i) ql[b * 128 + i] = p[i];
        for (int i = 0; i < 64; ++i) qh[b * 64 + i] = p[128 + i];
        for (int i = 0; i < 16; ++i) sc[b * 16 + i] = (int8_t)p[192 + i];
        d[b] = (uint16_t)(p[208] | (p[209] << 8));
    }
}
__global__ void unpack_q6k_kernel(const uint8_t* __restrict__ ql, const uint8_t* __restrict__ qh, const int8_t* __restrict__ sc,
                                  const uint16_t* __restrict__ d, uint8_t* __restrict__ raw, uint64_t nblocks) {
    for (uint64_t b = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; b < nblocks; b += (uint64_t)gridDim.x * blockDim.x) {
        uint8_t* p = raw + b * 210;
        for (int i = 0; i < 128; ++i) p[i] = ql[b * 128 + i];
        for (int i = 0; i < 64; ++i) p[128 + i] = qh[b * 64 + i];
        for (int i = 0; i < 16; ++i) p[192 + i] = (uint8_t)sc[b * 16 + i];
        p[208] = d[b] & 0xff;
        p[209] = d[b] >> 8;
    }
}

static dim3 grid_for(uint64_t n, int threads) {
    const uint64_t g = (n + threads - 1) / threads;
    const uint64_t cap = (uint64_t)num_sms() * 16;
    return dim3((unsigned)(g < cap ? (g ? g : 1) : cap));
}

cudaError_t repack_from_ggml(mv_weight_s& w, const uint8_t* raw, cudaStream_t s) {
    const uint64_t nblocks = w.rows * w.nb;
    switch (w.type) {
        case 2: repack_q4_kernel<<<grid_for(nblocks, 256), 256, 0, s>>>(raw, w.qs, w.d, nblocks, w.nb, w.dstride); break;
        case 8: repack_q8_kernel<<<grid_for(nblocks, 256), 256, 0, s>>>(raw, w.qs, w.d, nblocks); break;
        case 14: repack_q6k_kernel<<<grid_for(nblocks, 256), 256, 0, s>>>(raw, w.qs, w.qh, w.sc, w.d, nblocks); break;
        default: return cudaMemcpyAsync(w.qs, raw, w.rows * w.cols * (w.type == 0 ? 4 : 2), cudaMemcpyDeviceToDevice, s);
    }
    return cudaGetLastError();
}

cudaError_t unpack_to_ggml(const mv_weight_s& w, uint8_t* raw, cudaStream_t s) {
    const uint64_t nblocks = w.rows * w.nb;
    switch (w.type) {
        case 2: unpack_q4_kernel<<<grid_for(nblocks, 256), 256, 0, s>>>(w.qs, w.d, raw, nblocks, w.nb, w.dstride); break;
        case 8: unpack_q8_kernel<<<grid_for(nblocks, 256), 256, 0, s>>>(w.qs, w.d, raw, nblocks); break;
        case 14: unpack_q6k_kernel<<<grid_for(nblocks, 256), 256, 0, s>>>(w.qs, w.qh, w.sc, w.d, raw, nblocks); break;
        default: return cudaMemcpyAsync(raw, w.qs, w.rows * w.cols * (w.type == 0 ? 4 : 2), cudaMemcpyDeviceToDevice, s);
    }
    return cudaGetLastError();
}

// ------------------------------------------------------------ read rows
// out[i, :] = dequantised row rows[i], as tensor_read_row_f32
// (src/gguf_kernels.cpp:226): Q4_0 d*(q-8), Q8_0 d*q, Q6_K d*scale*q6
// (float products in that order), F16 exact, F32 copy.  One CTA per row.
__global__ void read_rows_kernel(mv_weight_s w, const int32_t* __restrict__ rows, float* __restrict__ out) {
    pdl_trigger();
    pdl_wait();
    const uint64_t r = (uint64_t)rows[blockIdx.x];
    float* o = out + (uint64_t)blockIdx.x * w.cols;
    if (r >= w.rows) {  // out-of-range ids give a NaN row instead of a wild read
        for (uint64_t c = threadIdx.x; c < w.cols; c += blockDim.x) o[c] = __int_as_float(0x7fc00000);
        return;
    }
    for (uint64_t c = threadIdx.x; c < w.cols; c += blockDim.x) {
        float v;
        if (w.type == 2) {
            const uint64_t b = r * w.nb + c / 32;
            const int e = c % 32;
            const uint8_t byte = w.qs[b * 16 + (e & 15)];
            const int q = (e < 16 ? (byte & 15) : (byte >> 4)) - 8;
            v = half_bits_to_float(w.d[r * w.dstride + c / 32]) * (float)q;
        } else if (w.type == 8) {
            const uint64_t b = r * w.nb + c / 32;
            v = half_bits_to_float(w.d[b]) * (float)(int8_t)w.qs[b * 32 + c % 32];
        } else if (w.type == 14) {
            const uint64_t b = r * w.nb + c / 256;
            const int i = c % 256, r32 = i / 32, j = i % 32, g = r32 / 4, slot = r32 % 4;
            const int lo = (w.qs[b * 128 + g * 64 + (slot & 1) * 32 + j] >> (slot < 2 ? 0 : 4)) & 15;
            const int hi = (w.qh[b * 64 + g * 32 + j] >> (2 * slot)) & 3;
            const int q6 = (lo | (hi << 4)) - 32;
            v = half_bits_to_float(w.d[b]) * (float)w.sc[b * 16 + i / 16] * (float)q6;
        } else if (w.type == 1) {
            v = half_bits_to_float(reinterpret_cast<const uint16_t*>(w.qs)[r * w.cols + c]);
        } else {
            v = reinterpret_cast<const float*>(w.qs)[r * w.cols + c];
        }
        o[c] = v;
    }
}

cudaError_t read_rows(const mv_weight_s& w, const int32_t* rows, uint64_t n, float* out, cudaStream_t s) {
    if (!n) return cudaSuccess;
    return launch_pdl(read_rows_kernel, dim3((unsigned)n), dim3(256), 0, s, w, rows, out);
}

// ------------------------------------------------------ activation quant
// Per row, per 32-element block: the reference's quantize_q8.  One warp per
// block, one element per lane.
__global__ void quantize_q8_kernel(const float* __restrict__ x, uint64_t nblocks, int8_t* __restrict__ q,
                                   float* __restrict__ d) {
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x / 32);
    for (uint64_t b = blockIdx.x * (uint64_t)(blockDim.x / 32) + threadIdx.x / 32; b < nblocks; b += warps) {
        float dd;
        const int v = quant_q8_lane(x[b * 32 + lane], dd);
        q[b * 32 + lane] = (int8_t)v;
        if (lane == 0) d[b] = dd;
    }
}

// The same quantisation laid out for the tensor-core GEMM: scales
// block-major, dT[b * ldb + row], and right after them (at dT + nb * ldb) the
// exact constants c[b * ldb + row] = 1.5 * 2^23 + 8 * sum(q of the block) that
// turn the GEMM's biased unsigned-nibble dot back into the reference's int32
// block dot (gemm_tc.cu).  Rows rows..ldb-1 of both are zero.
// qh set: the values go out as fp16 (exact: |q| <= 127) to qh instead of
// int8 to q, for the fp16 tensor-core GEMM (gemm_f16.cu).
// Position (row, block) of block b = row * nb + block, advanced by a fixed
// stride of blocks without a division per step.
constexpr int kUnroll = 4;  // blocks per warp and trip in the quantisers below
struct BlockPos {
    uint64_t row, blk, drow, dblk, nb;
    __device__ BlockPos(uint64_t b, uint64_t stride, uint64_t n)
        : row(b / n), blk(b % n), drow(stride / n), dblk(stride % n), nb(n) {}
    __device__ __forceinline__ void step() {
        blk += dblk;
        row += drow;
        if (blk >= nb) {
            blk -= nb;
            ++row;
        }
    }
};

__global__ void quantize_q8_t_kernel(const float* __restrict__ x, uint64_t rows, uint64_t nb, int8_t* __restrict__ q,
                                     float* __restrict__ dT, uint64_t ldb, uint16_t* __restrict__ qh) {
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x / 32);
    const uint64_t first = blockIdx.x * (uint64_t)(blockDim.x / 32) + threadIdx.x / 32;
    float* cT = dT + nb * ldb;
    pdl_trigger();
    pdl_wait();
    // kUnroll blocks per warp and trip, all loads issued before the first
    // block is quantised (bytes in flight bound this kernel)
    const uint64_t nbt = rows * nb;
    BlockPos bp(first, warps, nb);
    for (uint64_t b0 = first; b0 < nbt; b0 += kUnroll * warps) {
        float xv[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const uint64_t b = b0 + u * warps;
            xv[u] = b < nbt ? __ldcg(x + b * 32 + lane) : 0.0f;  // L2: x may come from other GPUs
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const uint64_t b = b0 + u * warps;
            if (b < nbt) {  // warp-uniform
                float dd;
                const int v = quant_q8_lane(xv[u], dd);
                if (qh) qh[b * 32 + lane] = __half_as_ushort(__int2half_rn(v));
                else q[b * 32 + lane] = (int8_t)v;
                const int sum = warp_sum_i(v);
                if (lane == 0) {
                    const uint64_t at = bp.blk * ldb + bp.row;
                    dT[at] = dd;
                    cT[at] = 12582912.0f + (float)(8 * sum);
                }
            }
            bp.step();
        }
    }
    const uint64_t padw = ldb - rows, padn = nb * padw;
    for (uint64_t i = first * 32 + lane; i < padn; i += warps * 32) {
        const uint64_t at = (i / padw) * ldb + rows + i % padw;
        dT[at] = 0.0f;
        cT[at] = 0.0f;
    }
}

// The same quantisation of ff = silu(g) * u computed on the fly from the
// gate|up GEMM output, whose rows come interleaved (g_i, u_i): the down
// projection's input without materialising ff.  ff is evaluated exactly as
// silu_pairs_kernel evaluates it, (g / (1 + expf(-g))) * u.
__global__ void silu_quantize_q8_t_kernel(const float* __restrict__ gu, uint64_t rows, uint64_t nb,
                                          int8_t* __restrict__ q, float* __restrict__ dT, uint64_t ldb,
                                          uint16_t* __restrict__ qh) {
    // 8 lanes per 32-element block, 4 consecutive elements each (two float4 of
    // (g, u) pairs): a warp takes 4 blocks per step and kUnroll steps' loads at
    // once; a block's max and sum are 3 shuffle steps within its 8 lanes
    const int lane = threadIdx.x & 31, sub = lane >> 3, l8 = lane & 7;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x / 32);
    const uint64_t first = blockIdx.x * (uint64_t)(blockDim.x / 32) + threadIdx.x / 32;
    float* cT = dT + nb * ldb;
    pdl_trigger();
    pdl_wait();
    const uint64_t nbt = rows * nb, ngroups = (nbt + 3) / 4;
    BlockPos bp(4 * first + sub, 4 * warps, nb);
    for (uint64_t g0 = first; g0 < ngroups; g0 += kUnroll * warps) {
        float4 pa[kUnroll], pb[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const uint64_t b = 4 * (g0 + u * warps) + sub;
            if (b < nbt) {
                const float4* src = reinterpret_cast<const float4*>(gu) + b * 16 + l8 * 2;
                pa[u] = src[0];
                pb[u] = src[1];
            } else {
                pa[u] = pb[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const uint64_t b = 4 * (g0 + u * warps) + sub;  // the same for the block's 8 lanes
            const float f0 = (pa[u].x / (1.0f + expf(-pa[u].x))) * pa[u].y;
            const float f1 = (pa[u].z / (1.0f + expf(-pa[u].z))) * pa[u].w;
            const float f2 = (pb[u].x / (1.0f + expf(-pb[u].x))) * pb[u].y;
            const float f3 = (pb[u].z / (1.0f + expf(-pb[u].z))) * pb[u].w;
            float mx = fmaxf(fmaxf(fabsf(f0), fabsf(f1)), fmaxf(fabsf(f2), fabsf(f3)));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            const float d = mx > 0.0f ? mx / 127.0f : 1.0f;
            const float id = 1.0f / d;
            const int q0 = (int)fminf(fmaxf(roundf(f0 * id), -127.0f), 127.0f);
            const int q1 = (int)fminf(fmaxf(roundf(f1 * id), -127.0f), 127.0f);
            const int q2 = (int)fminf(fmaxf(roundf(f2 * id), -127.0f), 127.0f);
            const int q3 = (int)fminf(fmaxf(roundf(f3 * id), -127.0f), 127.0f);
            int sum = q0 + q1 + q2 + q3;
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
            if (b < nbt) {
                if (qh) {
                    const uint32_t h01 = (uint32_t)__half_as_ushort(__int2half_rn(q0)) |
                                         ((uint32_t)__half_as_ushort(__int2half_rn(q1)) << 16);
                    const uint32_t h23 = (uint32_t)__half_as_ushort(__int2half_rn(q2)) |
                                         ((uint32_t)__half_as_ushort(__int2half_rn(q3)) << 16);
                    reinterpret_cast<uint2*>(qh)[b * 8 + l8] = make_uint2(h01, h23);
                } else {
                    reinterpret_cast<uint32_t*>(q)[b * 8 + l8] =
                        (uint32_t)(q0 & 0xFF) | ((uint32_t)(q1 & 0xFF) << 8) | ((uint32_t)(q2 & 0xFF) << 16) |
                        ((uint32_t)(q3 & 0xFF) << 24);
                }
                if (l8 == 0) {
                    const uint64_t at = bp.blk * ldb + bp.row;
                    dT[at] = d;
                    cT[at] = 12582912.0f + (float)(8 * sum);
                }
            }
            bp.step();
        }
    }
    const uint64_t padw = ldb - rows, padn = nb * padw;
    for (uint64_t i = first * 32 + lane; i < padn; i += warps * 32) {
        const uint64_t at = (i / padw) * ldb + rows + i % padw;
        dT[at] = 0.0f;
        cT[at] = 0.0f;
    }
}

// RMSNorm of every row (ops.cu rmsnorm_kernel: sum of squares in double,
// x * inv * w with two roundings) fused with the quantisation above, for the
// prefill GEMMs whose input is a normalised row (q|k|v, gate|up).  One CTA per
// row; each thread owns 4 consecutive elements per step, so a 32-element
// block is 8 consecutive lanes and its max / sum are 3 shuffle steps.
__global__ void rmsnorm_quantize_t_kernel(const float* __restrict__ x, const float* __restrict__ w, int n, float eps,
                                          uint64_t rows, int8_t* __restrict__ q, float* __restrict__ dT,
                                          uint64_t ldb, uint16_t* __restrict__ qh) {
    __shared__ double red[32];
    const uint64_t row = blockIdx.x;
    const int nc = n / 4, nb = n / 32;
    const int steps = (nc + blockDim.x - 1) / blockDim.x;
    const float4* xr = reinterpret_cast<const float4*>(x + row * n);
    pdl_trigger();
    pdl_wait();
    double ss = 0.0;
    for (int c = threadIdx.x; c < nc; c += blockDim.x) {
        const float4 v = __ldcg(xr + c);  // L2: x may come from other GPUs
        ss += (double)v.x * v.x;
        ss += (double)v.y * v.y;
        ss += (double)v.z * v.z;
        ss += (double)v.w * v.w;
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
    float* cT = dT + (uint64_t)nb * ldb;
    for (int st = 0; st < steps; ++st) {  // every lane takes part in the shuffles
        const int c = st * blockDim.x + threadIdx.x;
        const bool live = c < nc;       // whole 8-lane groups live or not (nc % 8 == 0)
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        if (live) {
            const float4 v = __ldcg(xr + c), g = reinterpret_cast<const float4*>(w)[c];
            o = make_float4(v.x * inv * g.x, v.y * inv * g.y, v.z * inv * g.z, v.w * inv * g.w);
        }
        float mx = fmaxf(fmaxf(fabsf(o.x), fabsf(o.y)), fmaxf(fabsf(o.z), fabsf(o.w)));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        const float d = mx > 0.0f ? mx / 127.0f : 1.0f;
        const float id = 1.0f / d;
        const int q0 = (int)fminf(fmaxf(roundf(o.x * id), -127.0f), 127.0f);
        const int q1 = (int)fminf(fmaxf(roundf(o.y * id), -127.0f), 127.0f);
        const int q2 = (int)fminf(fmaxf(roundf(o.z * id), -127.0f), 127.0f);
        const int q3 = (int)fminf(fmaxf(roundf(o.w * id), -127.0f), 127.0f);
        int sum = q0 + q1 + q2 + q3;
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        if (live) {
            if (qh) {
                const uint32_t h01 = (uint32_t)__half_as_ushort(__int2half_rn(q0)) |
                                     ((uint32_t)__half_as_ushort(__int2half_rn(q1)) << 16);
                const uint32_t h23 = (uint32_t)__half_as_ushort(__int2half_rn(q2)) |
                                     ((uint32_t)__half_as_ushort(__int2half_rn(q3)) << 16);
                reinterpret_cast<uint2*>(qh + row * n)[c] = make_uint2(h01, h23);
            } else {
                reinterpret_cast<uint32_t*>(q + row * n)[c] =
                    (uint32_t)(q0 & 0xFF) | ((uint32_t)(q1 & 0xFF) << 8) | ((uint32_t)(q2 & 0xFF) << 16) |
                    ((uint32_t)(q3 & 0xFF) << 24);
            }
            if ((c & 7) == 0) {
                const uint64_t at = (uint64_t)(c / 8) * ldb + row;
                dT[at] = d;
                cT[at] = 12582912.0f + (float)(8 * sum);
            }
        }
    }
    if (blockIdx.x == 0) {  // tokens rows..ldb-1 of every block: zero
        const uint64_t padw = ldb - rows, padn = (uint64_t)nb * padw;
        for (uint64_t i = threadIdx.x; i < padn; i += blockDim.x) {
            const uint64_t at = (i / padw) * ldb + rows + i % padw;
            dT[at] = 0.0f;
            cT[at] = 0.0f;
        }
    }
}

cudaError_t rmsnorm_quantize_q8_rows_t(const float* x, const float* w, uint64_t rows, uint64_t cols, float eps,
                                       int8_t* q, float* dT, uint64_t ldb, cudaStream_t s, uint16_t* qh) {
    if (!rows) return cudaSuccess;
    if (cols % 32 || ldb < rows) return cudaErrorInvalidValue;
    const uint64_t nc = cols / 4;
    const unsigned threads = (unsigned)(nc >= 1024 ? 1024 : (nc + 31) / 32 * 32);
    return launch_pdl(rmsnorm_quantize_t_kernel, dim3((unsigned)rows), dim3(threads), 0, s, x, w, (int)cols, eps, rows,
                      q, dT, ldb, qh);
}

cudaError_t quantize_q8_rows_t(const float* x, uint64_t rows, uint64_t cols, int8_t* q, float* dT, uint64_t ldb,
                               cudaStream_t s, uint16_t* qh) {
    const uint64_t nblocks = rows * (cols / 32);
    if (!nblocks || ldb < rows) return nblocks ? cudaErrorInvalidValue : cudaSuccess;
    const uint64_t ctas = (nblocks + 7) / 8;
    const uint64_t cap = (uint64_t)num_sms() * 8;
    return launch_pdl(quantize_q8_t_kernel, dim3((unsigned)(ctas < cap ? ctas : cap)), dim3(256), 0, s, x, rows,
                      cols / 32, q, dT, ldb, qh);
}

cudaError_t silu_quantize_q8_rows_t(const float* gu, uint64_t rows, uint64_t cols, int8_t* q, float* dT, uint64_t ldb,
                                    cudaStream_t s, uint16_t* qh) {
    const uint64_t nblocks = rows * (cols / 32);
    if (!nblocks || ldb < rows || cols % 32) return nblocks ? cudaErrorInvalidValue : cudaSuccess;
    const uint64_t ctas = (nblocks + 31) / 32;  // 8 warps of 4 blocks
    const uint64_t cap = (uint64_t)num_sms() * 8;
    return launch_pdl(silu_quantize_q8_t_kernel, dim3((unsigned)(ctas < cap ? ctas : cap)), dim3(256), 0, s, gu, rows,
                      cols / 32, q, dT, ldb, qh);
}

cudaError_t quantize_q8_rows(const float* x, uint64_t rows, uint64_t cols, int8_t* q, float* d, cudaStream_t s) {
    const uint64_t nblocks = rows * (cols / 32);
    if (!nblocks) return cudaSuccess;
    const uint64_t ctas = (nblocks + 7) / 8;
    const uint64_t cap = (uint64_t)num_sms() * 8;
    quantize_q8_kernel<<<(unsigned)(ctas < cap ? ctas : cap), 256, 0, s>>>(x, nblocks, q, d);
    return cudaGetLastError();
}

}  // namespace mvb
