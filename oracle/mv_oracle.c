/*
 * mv_oracle.c -- CPU restatement of MemVanta's quantized-matmul hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA path is
 * compared against; it is never linked into, loaded by, or called from the
 * product library (memvanta_b200/).  Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline leg may use it.
 *
 * Every function restates one piece of the reference's arithmetic and cites
 * the reference file:line (paths relative to the MemVanta project root) it
 * follows.  Where the reference's AVX2 build fixes an evaluation order (8
 * FMA lanes, then a left-to-right horizontal sum) the restatement follows
 * that order too, so this oracle agrees bit for bit with the reference built
 * with -mavx2 -mfma -mf16c (the pinning tests check exactly that).
 *
 * The reference's C++ is compiled by GCC with FMA available (-mfma or
 * -march=native), and GCC contracts C++ expressions even in ISO mode: in
 * the multi-threaded build of the GGUF kernels `s += a*b` becomes
 * fma(a,b,s), `s += a*b*c` becomes fma(a*b,c,s), `x0*c - x1*s` becomes
 * fma(x0,c,-(x1*s)) and `x0*s + x1*c` becomes fma(x0,s,x1*c).  Which
 * expressions GCC fuses depends on the inlining context: the single-thread
 * path of tensor_matvec (row lambda inlined) and the internal-format
 * dot_q4_q8 / matvec_f32 are left unfused.  The restatement spells out each
 * fusion the multi-threaded reference build performs with fmaf() and is
 * itself built with -ffp-contract=off so that nothing else is fused.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>

#define MVO_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------ */
/* half <-> float                                                      */
/* ------------------------------------------------------------------ */

static float bits_to_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f32_to_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* Exact IEEE half -> float, subnormals included.  src/gguf.cpp:110-119. */
MVO_API float mvo_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t e = (h >> 10) & 31u, m = h & 1023u;
    if (e == 0) {
        /* zero or subnormal: m * 2^-24 is exact in float */
        float v = (float)m * 5.9604644775390625e-08f;
        return bits_to_f32(f32_to_bits(v) | sign);
    }
    if (e == 31) return bits_to_f32(sign | 0x7f800000u | (m << 13));
    return bits_to_f32(sign | ((e + 112u) << 23) | (m << 13));
}

/* The reference's own float -> half: the mantissa is rounded by adding half
 * an output ulp (0x1000 at bit 12) and truncating, i.e. round-half-up on the
 * magnitude (not round-to-nearest-even); a carry out of the mantissa bumps
 * the exponent; inputs at or above 2^16 (and NaN) give +-inf; magnitudes
 * below 2^-25 give signed zero.  src/gguf_kernels.cpp:242. */
MVO_API uint16_t mvo_fp32_to_fp16(float f) {
    const uint32_t x = f32_to_bits(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t mant = x & 0x7fffffu;
    const int e = (int)((x >> 23) & 0xffu) - 112;   /* rebias 127 -> 15 */
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e > 0) return (uint16_t)(sign | ((uint32_t)e << 10) | ((mant + 0x1000u) >> 13));
    if (e < -10) return (uint16_t)sign;
    mant = (mant | 0x800000u) >> (1 - e);           /* denormalise */
    return (uint16_t)(sign + ((mant + 0x1000u) >> 13));
}

/* ------------------------------------------------------------------ */
/* helpers that mirror the reference's AVX2 reductions                 */
/* ------------------------------------------------------------------ */

/* _mm256 accumulator spilled to memory then summed t[0]+..+t[7] left to
 * right (src/gguf_kernels.cpp:104, :115, :230, ...). */
static float hsum8(const float t[8]) {
    float s = 0.0f;                     /* `float s=0; for(v:tmp) s+=v;` */
    for (int i = 0; i < 8; ++i) s += t[i];
    return s;
}
static float hsum8_direct(const float t[8]) {
    /* `t[0]+t[1]+...+t[7]` (no leading zero; identical unless t[0]==-0) */
    float s = t[0];
    for (int i = 1; i < 8; ++i) s += t[i];
    return s;
}

/* dot_f32_simd: 8 FMA lanes over i+8<=n, hsum, scalar tail.
 * src/gguf_kernels.cpp:228-234. */
MVO_API float mvo_dot_f32(const float* a, const float* b, size_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    size_t i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; ++l) acc[l] = fmaf(a[i + l], b[i + l], acc[l]);
    float s = hsum8_direct(acc);
    for (; i < n; ++i) s = fmaf(a[i], b[i], s);
    return s;
}

/* axpy_f32_simd: y += alpha*x with FMA.  src/gguf_kernels.cpp:235-241. */
MVO_API void mvo_axpy_f32(float alpha, const float* x, float* y, size_t n) {
    size_t i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; ++l) y[i + l] = fmaf(alpha, x[i + l], y[i + l]);
    for (; i < n; ++i) y[i] = fmaf(alpha, x[i], y[i]);
}

/* ------------------------------------------------------------------ */
/* GGUF block layouts (src/gguf_kernels.cpp:21-31)                     */
/*   Q4_0: 18 B  {u16 d; u8 qs[16]}  elem i<16 = qs[i]&15, 16+i = qs[i]>>4 */
/*   Q8_0: 34 B  {u16 d; i8 qs[32]}                                     */
/*   Q6_K: 210 B {u8 ql[128]; u8 qh[64]; i8 scales[16]; u16 d}          */
/* ------------------------------------------------------------------ */
#define Q4_BYTES 18
#define Q8_BYTES 34
#define Q6K_BYTES 210

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* a1: per-32 activation quantisation.  src/gguf_kernels.cpp:161-172.
 * mx = max|z|; d = mx>0 ? mx/127 : 1; inv = 1/d;
 * q = clamp(lround(z*inv), -127, 127) (round half away from zero). */
MVO_API void mvo_quantize_q8(const float* x, size_t cols, int8_t* q, float* d) {
    for (size_t b = 0; b < cols / 32; ++b) {
        const float* z = x + b * 32;
        float mx = 0.0f;
        for (int k = 0; k < 32; ++k) { float a = fabsf(z[k]); if (a > mx) mx = a; }
        const float dd = mx > 0 ? mx / 127.0f : 1.0f, inv = 1.0f / dd;
        d[b] = dd;
        for (int k = 0; k < 32; ++k) {
            long v = lroundf(z[k] * inv);
            if (v < -127) v = -127;
            if (v > 127) v = 127;
            q[b * 32 + k] = (int8_t)v;
        }
    }
}

/* a2: quantize_activations_q8 = a1 per row.  src/gguf_kernels.cpp:174-178. */
MVO_API void mvo_quantize_q8_rows(const float* x, size_t batch, size_t cols, int8_t* q, float* d) {
    for (size_t r = 0; r < batch; ++r) mvo_quantize_q8(x + r * cols, cols, q + r * cols, d + r * (cols / 32));
}

/* a3: integer dot of one Q4_0 block with 32 int8 activations.
 * src/gguf_kernels.cpp:148-158, :180-188. */
MVO_API int32_t mvo_dot_q4_q8_block(const uint8_t* blk, const int8_t* aq) {
    const uint8_t* qs = blk + 2;
    int32_t s = 0;
    for (int i = 0; i < 16; ++i) {
        s += ((int32_t)(qs[i] & 15) - 8) * aq[i];
        s += ((int32_t)(qs[i] >> 4) - 8) * aq[16 + i];
    }
    return s;
}

/* a4: row dot, sequential fp32 `sum += fp16(dw)*ad*float(isum)`.
 * src/gguf_kernels.cpp:189. */
static float dot_q4_q8_row(const uint8_t* row, const int8_t* aq, const float* ad, size_t nb) {
    float sum = 0.0f;
    for (size_t b = 0; b < nb; ++b) {
        const uint8_t* blk = row + b * Q4_BYTES;
        const float dw = mvo_fp16_to_fp32(rd16(blk));
        sum = fmaf(dw * ad[b], (float)mvo_dot_q4_q8_block(blk, aq + b * 32), sum);
    }
    return sum;
}

/* a8: Q4_0 x fp32 (no activation quantisation), AVX2 order: q as int8,
 * 8 FMA lanes per block (elements l, 8+l, 16+l, 24+l on lane l), hsum,
 * then sum += d*s.  src/gguf_kernels.cpp:93-109. */
static float dot_q4_0_fp32(const uint8_t* row, const float* x, size_t nb) {
    float sum = 0.0f;
    for (size_t b = 0; b < nb; ++b) {
        const uint8_t* blk = row + b * Q4_BYTES;
        const float d = mvo_fp16_to_fp32(rd16(blk));
        const uint8_t* qs = blk + 2;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int h = 0; h < 2; ++h)
            for (int k = 0; k < 16; k += 8)
                for (int l = 0; l < 8; ++l) {
                    const int e = k + l;
                    const int q = (h ? (qs[e] >> 4) : (qs[e] & 15)) - 8;
                    acc[l] = fmaf((float)q, x[b * 32 + h * 16 + e], acc[l]);
                }
        sum = fmaf(d, hsum8(acc), sum);
    }
    return sum;
}

/* a6: Q8_0 x fp32, 8 FMA lanes per block, hsum, sum += d*s.
 * src/gguf_kernels.cpp:111-120. */
static float dot_q8_0_fp32(const uint8_t* row, const float* x, size_t nb) {
    float sum = 0.0f;
    for (size_t b = 0; b < nb; ++b) {
        const uint8_t* blk = row + b * Q8_BYTES;
        const float d = mvo_fp16_to_fp32(rd16(blk));
        const int8_t* qs = (const int8_t*)(blk + 2);
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int k = 0; k < 32; k += 8)
            for (int l = 0; l < 8; ++l) acc[l] = fmaf((float)qs[k + l], x[b * 32 + k + l], acc[l]);
        sum = fmaf(d, hsum8(acc), sum);
    }
    return sum;
}

/* a7: one Q6_K weight as a signed 6-bit integer.  Element i of a 256-wide
 * super-block: r = i/32 picks (group r/4, slot r%4); the low nibble comes
 * from ql[group*64 + (slot&1)*32 + i%32] (low half for slots 0,1, high half
 * for 2,3), the top two bits from qh[group*32 + i%32] >> (2*slot).
 * src/gguf_kernels.cpp:122-136. */
MVO_API int mvo_q6_k_value(const uint8_t* blk, size_t i) {
    const uint8_t* ql = blk;
    const uint8_t* qh = blk + 128;
    const size_t r = i / 32, j = i % 32, group = r / 4, slot = r % 4;
    const int lo = (ql[group * 64 + (slot & 1) * 32 + j] >> (slot < 2 ? 0 : 4)) & 15;
    const int hi = (qh[group * 32 + j] >> (2 * slot)) & 3;
    return (lo | (hi << 4)) - 32;
}

/* a7: w = d*scale*q (float), double accumulation of double(w)*x.
 * src/gguf_kernels.cpp:138-146. */
static float dot_q6_k_fp32(const uint8_t* row, const float* x, size_t nsb) {
    double sum = 0.0;
    for (size_t b = 0; b < nsb; ++b) {
        const uint8_t* blk = row + b * Q6K_BYTES;
        const int8_t* sc = (const int8_t*)(blk + 192);
        const float d = mvo_fp16_to_fp32(rd16(blk + 208));
        for (size_t i = 0; i < 256; ++i) {
            const float w = d * (float)sc[i / 16] * (float)mvo_q6_k_value(blk, i);
            sum += (double)w * (double)x[b * 256 + i];
        }
    }
    return (float)sum;
}

/* F16 matrix row: double accumulation.  src/gguf_kernels.cpp:250. */
static float dot_f16_row(const uint16_t* row, const float* x, size_t cols) {
    double s = 0.0;
    for (size_t c = 0; c < cols; ++c) s += (double)mvo_fp16_to_fp32(row[c]) * (double)x[c];
    return (float)s;
}

enum { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8, T_Q6_K = 14 };

static size_t row_bytes(int type, size_t cols) {
    switch (type) {
        case T_F32: return cols * 4;
        case T_F16: return cols * 2;
        case T_Q4_0: return cols / 32 * Q4_BYTES;
        case T_Q8_0: return cols / 32 * Q8_BYTES;
        case T_Q6_K: return cols / 256 * Q6K_BYTES;
    }
    return 0;
}

/* a5: tensor_matvec type dispatch.  Q4_0 quantises x once (a1) and uses the
 * integer path; Q8_0, Q6_K, F16, F32 use fp32 x.  Returns 0, or -1 for an
 * unsupported type / misaligned cols (the reference throws).
 * src/gguf_kernels.cpp:244-253. */
MVO_API int mvo_matvec(int type, const void* w, size_t rows, size_t cols, const float* x, float* y) {
    const uint8_t* W = (const uint8_t*)w;
    const size_t rb = row_bytes(type, cols);
    if (type == T_Q4_0) {
        if (cols % 32) return -1;
        int8_t* q = (int8_t*)malloc(cols);
        float* d = (float*)malloc(sizeof(float) * (cols / 32));
        mvo_quantize_q8(x, cols, q, d);
        for (size_t r = 0; r < rows; ++r) y[r] = dot_q4_q8_row(W + r * rb, q, d, cols / 32);
        free(q); free(d);
        return 0;
    }
    if (type == T_Q8_0) {
        if (cols % 32) return -1;
        for (size_t r = 0; r < rows; ++r) y[r] = dot_q8_0_fp32(W + r * rb, x, cols / 32);
        return 0;
    }
    if (type == T_Q6_K) {
        if (cols % 256) return -1;
        for (size_t r = 0; r < rows; ++r) y[r] = dot_q6_k_fp32(W + r * rb, x, cols / 256);
        return 0;
    }
    if (type == T_F32) {
        for (size_t r = 0; r < rows; ++r) y[r] = mvo_dot_f32((const float*)(W + r * rb), x, cols);
        return 0;
    }
    if (type == T_F16) {
        for (size_t r = 0; r < rows; ++r) y[r] = dot_f16_row((const uint16_t*)(W + r * rb), x, cols);
        return 0;
    }
    return -1;
}

/* a11: tensor_matmul_batch -- every (token,row) pair through the fp32-x row
 * dot of its type (Q4_0 here uses a8, not the integer path).
 * src/gguf_kernels.cpp:255-259. */
MVO_API int mvo_matmul_batch(int type, const void* w, size_t rows, size_t cols, const float* x, size_t batch, float* y) {
    const uint8_t* W = (const uint8_t*)w;
    const size_t rb = row_bytes(type, cols);
    if (type != T_F32 && type != T_F16 && type != T_Q4_0 && type != T_Q8_0 && type != T_Q6_K) return -1;
    if ((type == T_Q4_0 || type == T_Q8_0) && cols % 32) return -1;
    if (type == T_Q6_K && cols % 256) return -1;
    for (size_t b = 0; b < batch; ++b)
        for (size_t r = 0; r < rows; ++r) {
            const float* xv = x + b * cols;
            const uint8_t* row = W + r * rb;
            float v = 0.0f;
            switch (type) {
                case T_Q4_0: v = dot_q4_0_fp32(row, xv, cols / 32); break;
                case T_Q8_0: v = dot_q8_0_fp32(row, xv, cols / 32); break;
                case T_Q6_K: v = dot_q6_k_fp32(row, xv, cols / 256); break;
                case T_F32: v = mvo_dot_f32((const float*)row, xv, cols); break;
                case T_F16: v = dot_f16_row((const uint16_t*)row, xv, cols); break;
            }
            y[b * rows + r] = v;
        }
    return 0;
}

/* a9: one weight row against 4 fp32 activation rows, AVX2 order: per block
 * the dequantised 8-wide vector q*d (rounded once) is FMA'd into 4
 * accumulators, lane l taking elements l, 8+l, 16+l, 24+l; the 4 lane
 * vectors are summed t[0]+..+t[7] at the end of the row.
 * src/gguf_kernels.cpp:191-209. */
static void row_batch4_fp32(int type, const uint8_t* row, const float* x, size_t stride, size_t nb, float out[4]) {
    float acc[4][8];
    memset(acc, 0, sizeof(acc));
    for (size_t b = 0; b < nb; ++b) {
        float deq[32];
        if (type == T_Q4_0) {
            const uint8_t* blk = row + b * Q4_BYTES;
            const float d = mvo_fp16_to_fp32(rd16(blk));
            for (int i = 0; i < 16; ++i) {
                deq[i] = (float)((int)(blk[2 + i] & 15) - 8) * d;
                deq[16 + i] = (float)((int)(blk[2 + i] >> 4) - 8) * d;
            }
        } else {
            const uint8_t* blk = row + b * Q8_BYTES;
            const float d = mvo_fp16_to_fp32(rd16(blk));
            for (int i = 0; i < 32; ++i) deq[i] = (float)((const int8_t*)(blk + 2))[i] * d;
        }
        for (int e0 = 0; e0 < 32; e0 += 8)
            for (int j = 0; j < 4; ++j)
                for (int l = 0; l < 8; ++l)
                    acc[j][l] = fmaf(deq[e0 + l], x[j * stride + b * 32 + e0 + l], acc[j][l]);
    }
    for (int j = 0; j < 4; ++j) out[j] = hsum8_direct(acc[j]);
}

/* a10: tensor_matmul_batch_v06.  batch<2, a type other than Q4_0/Q8_0 or
 * cols%32 -> a11.  force_q8 (MEMVANTA_FORCE_Q8_ACT=1): Q4_0 rows use a2 +
 * a4; Q8_0 rows keep fp32 x.  Otherwise a9 in blocks of 8 tokens for FFN
 * tensors (two blocks of 4) or 4 tokens otherwise, with a8/a6 for the
 * remaining tokens.  src/gguf_kernels.cpp:261-271. */
MVO_API int mvo_matmul_batch_v06(int type, const void* w, size_t rows, size_t cols, const float* x, size_t batch,
                                 float* y, int force_q8, int ffn) {
    if (batch < 2 || (type != T_Q4_0 && type != T_Q8_0) || cols % 32)
        return mvo_matmul_batch(type, w, rows, cols, x, batch, y);
    const uint8_t* W = (const uint8_t*)w;
    const size_t nb = cols / 32, rb = row_bytes(type, cols);
    if (force_q8) {
        int8_t* q = NULL;
        float* d = NULL;
        if (type == T_Q4_0) {
            q = (int8_t*)malloc(batch * cols);
            d = (float*)malloc(sizeof(float) * batch * nb);
            mvo_quantize_q8_rows(x, batch, cols, q, d);
        }
        for (size_t r = 0; r < rows; ++r)
            for (size_t b = 0; b < batch; ++b)
                y[b * rows + r] = type == T_Q4_0 ? dot_q4_q8_row(W + r * rb, q + b * cols, d + b * nb, nb)
                                                 : dot_q8_0_fp32(W + r * rb, x + b * cols, nb);
        free(q); free(d);
        return 0;
    }
    const size_t step = ffn ? 8 : 4;
    for (size_t r = 0; r < rows; ++r) {
        const uint8_t* row = W + r * rb;
        size_t b = 0;
        for (; b + step <= batch; b += step)
            for (size_t h = 0; h < step; h += 4) {
                float o[4];
                row_batch4_fp32(type, row, x + (b + h) * cols, cols, nb, o);
                for (int j = 0; j < 4; ++j) y[(b + h + j) * rows + r] = o[j];
            }
        for (; b < batch; ++b)
            y[b * rows + r] = type == T_Q4_0 ? dot_q4_0_fp32(row, x + b * cols, nb) : dot_q8_0_fp32(row, x + b * cols, nb);
    }
    return 0;
}

/* a12: dequantise one row to fp32 (embedding lookup).
 * src/gguf_kernels.cpp:226. */
MVO_API int mvo_read_row(int type, const void* w, size_t rows, size_t cols, size_t row, float* out) {
    if (row >= rows) return -1;
    const uint8_t* p = (const uint8_t*)w + row * row_bytes(type, cols);
    if (type == T_F32) { memcpy(out, p, cols * 4); return 0; }
    if (type == T_F16) { for (size_t i = 0; i < cols; ++i) out[i] = mvo_fp16_to_fp32(((const uint16_t*)p)[i]); return 0; }
    if (type == T_Q4_0) {
        for (size_t b = 0; b < cols / 32; ++b) {
            const uint8_t* blk = p + b * Q4_BYTES;
            const float d = mvo_fp16_to_fp32(rd16(blk));
            for (int i = 0; i < 16; ++i) {
                out[b * 32 + i] = d * (float)((int)(blk[2 + i] & 15) - 8);
                out[b * 32 + 16 + i] = d * (float)((int)(blk[2 + i] >> 4) - 8);
            }
        }
        return 0;
    }
    if (type == T_Q8_0) {
        for (size_t b = 0; b < cols / 32; ++b) {
            const uint8_t* blk = p + b * Q8_BYTES;
            const float d = mvo_fp16_to_fp32(rd16(blk));
            for (int i = 0; i < 32; ++i) out[b * 32 + i] = d * (float)((const int8_t*)(blk + 2))[i];
        }
        return 0;
    }
    if (type == T_Q6_K) {
        if (cols % 256) return -1;
        for (size_t b = 0; b < cols / 256; ++b) {
            const uint8_t* blk = p + b * Q6K_BYTES;
            const int8_t* sc = (const int8_t*)(blk + 192);
            const float d = mvo_fp16_to_fp32(rd16(blk + 208));
            for (size_t i = 0; i < 256; ++i) out[b * 256 + i] = d * (float)sc[i / 16] * (float)mvo_q6_k_value(blk, i);
        }
        return 0;
    }
    return -1;
}

/* ------------------------------------------------------------------ */
/* ops around the matmuls (src/llama_model.cpp)                        */
/* ------------------------------------------------------------------ */

/* a18: rmsnorm, double sum of squares; inv = 1/sqrt(float(ss/n)+eps);
 * o = x*inv*w.  src/llama_model.cpp:237, :245, :251. */
MVO_API void mvo_rmsnorm(const float* x, const float* w, size_t n, float eps, float* o) {
    double ss = 0.0;
    for (size_t i = 0; i < n; ++i) ss += (double)x[i] * (double)x[i];
    const float inv = 1.0f / sqrtf((float)(ss / (double)n) + eps);
    for (size_t i = 0; i < n; ++i) o[i] = x[i] * inv * w[i];
}

/* a19: RoPE tables, inv = theta^(-2i/hd) in float, angle = p*inv.
 * src/llama_model.cpp:233. */
MVO_API void mvo_rope_tables(size_t n_ctx, size_t hd, float theta, float* cosv, float* sinv) {
    const size_t half = hd / 2;
    for (size_t p = 0; p < n_ctx; ++p)
        for (size_t i = 0; i < half; ++i) {
            const float inv = powf(theta, -2.0f * (float)i / (float)hd);
            const float a = (float)p * inv;
            cosv[p * half + i] = cosf(a);
            sinv[p * half + i] = sinf(a);
        }
}

/* a19: half-split rotation of pairs (i, i+half) in every head.
 * src/llama_model.cpp:238. */
MVO_API void mvo_rope(float* q, size_t n_head, float* k, size_t n_head_kv, size_t hd, const float* cos_row,
                      const float* sin_row) {
    const size_t half = hd / 2;
    for (int which = 0; which < 2; ++which) {
        float* z = which ? k : q;
        const size_t heads = which ? n_head_kv : n_head;
        for (size_t h = 0; h < heads; ++h) {
            float* b = z + h * hd;
            for (size_t i = 0; i < half; ++i) {
                const float x0 = b[i], x1 = b[i + half], c = cos_row[i], s = sin_row[i];
                b[i] = fmaf(x0, c, -(x1 * s));
                b[i + half] = fmaf(x0, s, x1 * c);
            }
        }
    }
}

/* a20: SiLU gate, ff = g/(1+exp(-g))*u.  src/llama_model.cpp:249, :257. */
MVO_API void mvo_silu_mul(const float* g, const float* u, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = (g[i] / (1.0f + expf(-g[i]))) * u[i];
}

/* ------------------------------------------------------------------ */
/* KV cache (PagedKVCache, src/llama_model.cpp:18-55)                  */
/* kv types: 0 = F32, 1 = F16, 2 = Q8 (one scale per token over kv_dim) */
/* 3 = Q8_0 per 32-element block (BASELINE config-4 extension; same    */
/*     rules as a1 per block -- no reference implementation exists)    */
/* ------------------------------------------------------------------ */

/* a15: store one token's k (or v) row.  F16 uses the reference rounding;
 * Q8 stores s = max|v|/127 (1 if all zero) and clamp(lround(v/s)) -- note
 * the division, unlike a1's multiply-by-inverse.  src/llama_model.cpp:22. */
MVO_API void mvo_kv_store(int kv_type, const float* v, size_t kv_dim, void* dst, float* scale_out) {
    if (kv_type == 0) { memcpy(dst, v, kv_dim * 4); return; }
    if (kv_type == 1) {
        uint16_t* h = (uint16_t*)dst;
        for (size_t i = 0; i < kv_dim; ++i) h[i] = mvo_fp32_to_fp16(v[i]);
        return;
    }
    if (kv_type == 2) {
        float m = 0.0f;
        for (size_t i = 0; i < kv_dim; ++i) { float a = fabsf(v[i]); if (a > m) m = a; }
        const float s = m > 0 ? m / 127.0f : 1.0f;
        *scale_out = s;
        int8_t* q = (int8_t*)dst;
        for (size_t i = 0; i < kv_dim; ++i) {
            long t = lroundf(v[i] / s);
            if (t < -127) t = -127;
            if (t > 127) t = 127;
            q[i] = (int8_t)t;
        }
        return;
    }
    /* kv_type 3: per-32 blocks, scales written to scale_out[kv_dim/32] */
    mvo_quantize_q8(v, kv_dim, (int8_t*)dst, scale_out);
}

/* a16: q . k[offset:offset+n] for one cached token.
 * F32 -> dot_f32_simd; F16 -> 8 FMA lanes of q*half(k), hsum, tail;
 * Q8 -> 8 FMA lanes of q*float(k8), hsum, times the token scale.
 * Q8_0 (extension) -> per 32-block d * (sum of q*k8).
 * src/llama_model.cpp:23-39. */
static float kv_dot(int kv_type, const void* row, const float* scales, size_t offset, const float* q, size_t n) {
    if (kv_type == 0) return mvo_dot_f32(q, (const float*)row + offset, n);
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    size_t d = 0;
    if (kv_type == 1) {
        const uint16_t* h = (const uint16_t*)row + offset;
        for (; d + 8 <= n; d += 8)
            for (int l = 0; l < 8; ++l) acc[l] = fmaf(q[d + l], mvo_fp16_to_fp32(h[d + l]), acc[l]);
        float s = hsum8_direct(acc);
        for (; d < n; ++d) s = fmaf(q[d], mvo_fp16_to_fp32(h[d]), s);
        return s;
    }
    const int8_t* k8 = (const int8_t*)row + offset;
    if (kv_type == 2) {
        for (; d + 8 <= n; d += 8)
            for (int l = 0; l < 8; ++l) acc[l] = fmaf(q[d + l], (float)k8[d + l], acc[l]);
        float s = hsum8_direct(acc);
        for (; d < n; ++d) s = fmaf(q[d], (float)k8[d], s);
        return s * scales[0];
    }
    float s = 0.0f;
    for (size_t b = 0; b < n / 32; ++b) {
        float t = 0.0f;
        for (int i = 0; i < 32; ++i) t = fmaf(q[b * 32 + i], (float)k8[b * 32 + i], t);
        s += t * scales[(offset / 32) + b];
    }
    return s;
}

/* a16: out += alpha * v[offset:offset+n].  F16/F32 use FMA per element;
 * Q8 folds the token scale into alpha first.  src/llama_model.cpp:40-55. */
static void kv_axpy(int kv_type, const void* row, const float* scales, size_t offset, float alpha, float* out, size_t n) {
    if (kv_type == 0) { mvo_axpy_f32(alpha, (const float*)row + offset, out, n); return; }
    if (kv_type == 1) {
        const uint16_t* h = (const uint16_t*)row + offset;
        for (size_t d = 0; d < n; ++d) out[d] = fmaf(alpha, mvo_fp16_to_fp32(h[d]), out[d]);
        return;
    }
    const int8_t* v8 = (const int8_t*)row + offset;
    if (kv_type == 2) {
        const float sc = alpha * scales[0];
        for (size_t d = 0; d < n; ++d) out[d] = fmaf(sc, (float)v8[d], out[d]);
        return;
    }
    for (size_t d = 0; d < n; ++d) out[d] = fmaf(alpha * scales[(offset + d) / 32], (float)v8[d], out[d]);
}

/* Bytes per cached token row and scales per row for each kv type. */
MVO_API size_t mvo_kv_row_bytes(int kv_type, size_t kv_dim) {
    return kv_type == 0 ? kv_dim * 4 : kv_type == 1 ? kv_dim * 2 : kv_dim;
}
MVO_API size_t mvo_kv_row_scales(int kv_type, size_t kv_dim) {
    return kv_type == 2 ? 1 : kv_type == 3 ? kv_dim / 32 : 0;
}

/* a17: single-query attention for one sequence over n_ctx cached tokens.
 * The cache is paged: token t lives in page block_table[t/page] at slot
 * t%page; each page holds page*kv_dim elements of K (and of V) plus
 * page*scales_per_row scales.  For every head h (kv head h/group):
 *   s_t = dot(q_h, k_t)/sqrt(hd); m = max s_t; e_t = exp(s_t-m);
 *   den = sum double(e_t); inv = float(1/den); out_h += (e_t*inv) v_t
 * with out_h zeroed first.  src/llama_model.cpp:256 (decode) and :248. */
MVO_API void mvo_attn_decode(int kv_type, const float* q, size_t n_head, size_t n_head_kv, size_t hd,
                             const void* k_pages, const void* v_pages, const float* k_scales,
                             const float* v_scales, const int32_t* block_table, size_t page, size_t n_ctx,
                             float* out) {
    const size_t kv_dim = n_head_kv * hd, group = n_head / n_head_kv;
    const size_t rb = mvo_kv_row_bytes(kv_type, kv_dim), ns = mvo_kv_row_scales(kv_type, kv_dim);
    float* sc = (float*)malloc(sizeof(float) * (n_ctx ? n_ctx : 1));
    const float root = sqrtf((float)hd);
    for (size_t h = 0; h < n_head; ++h) {
        const size_t kb = (h / group) * hd, qb = h * hd;
        float m = -INFINITY;
        for (size_t t = 0; t < n_ctx; ++t) {
            const size_t slot = (size_t)block_table[t / page] * page + t % page;
            const void* kr = (const uint8_t*)k_pages + slot * rb;
            const float* ks = k_scales ? k_scales + slot * ns : NULL;
            const float s = kv_dot(kv_type, kr, ks, kb, q + qb, hd) / root;
            sc[t] = s;
            if (s > m) m = s;
        }
        double den = 0.0;
        for (size_t t = 0; t < n_ctx; ++t) { sc[t] = expf(sc[t] - m); den += (double)sc[t]; }
        const float inv = (float)(1.0 / den);
        memset(out + qb, 0, sizeof(float) * hd);
        for (size_t t = 0; t < n_ctx; ++t) {
            const size_t slot = (size_t)block_table[t / page] * page + t % page;
            const void* vr = (const uint8_t*)v_pages + slot * rb;
            const float* vs = v_scales ? v_scales + slot * ns : NULL;
            kv_axpy(kv_type, vr, vs, kb, sc[t] * inv, out + qb, hd);
        }
    }
    free(sc);
}

/* ------------------------------------------------------------------ */
/* internal (non-GGUF) formats, include/memvanta/quant.hpp:8-13:        */
/*   BlockQ8_0 36 B {f32 d; i8 qs[32]}                                  */
/*   BlockQ4_0 20 B {f32 d; u8 qs[16]}, element 2i = low nibble of qs[i],*/
/*   element 2i+1 = high nibble (interleaved, unlike GGUF)              */
/* ------------------------------------------------------------------ */

/* quantize_q8_0: d = amax/127 (0 if amax==0, block zeroed);
 * q = clamp(nearbyint(x/d... as x*(1/d)), -127, 127).  src/quant.cpp:44-62. */
MVO_API void mvo_int_quantize_q8_0(const float* x, size_t n, uint8_t* out36) {
    for (size_t b = 0; b < n / 32; ++b) {
        const float* p = x + b * 32;
        uint8_t* blk = out36 + b * 36;
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) { float a = fabsf(p[i]); if (a > amax) amax = a; }
        const float d = amax == 0.0f ? 0.0f : amax / 127.0f;
        memcpy(blk, &d, 4);
        if (d == 0.0f) { memset(blk + 4, 0, 32); continue; }
        const float id = 1.0f / d;
        for (int i = 0; i < 32; ++i) {
            int q = (int)nearbyintf(p[i] * id);
            if (q < -127) q = -127;
            if (q > 127) q = 127;
            blk[4 + i] = (uint8_t)(int8_t)q;
        }
    }
}

/* quantize_q4_0: d = amax/7, q = clamp(nearbyint(x*(1/d)), -8, 7) + 8,
 * interleaved nibbles.  src/quant.cpp:64-85. */
MVO_API void mvo_int_quantize_q4_0(const float* x, size_t n, uint8_t* out20) {
    for (size_t b = 0; b < n / 32; ++b) {
        const float* p = x + b * 32;
        uint8_t* blk = out20 + b * 20;
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) { float a = fabsf(p[i]); if (a > amax) amax = a; }
        const float d = amax == 0.0f ? 0.0f : amax / 7.0f;
        memcpy(blk, &d, 4);
        memset(blk + 4, 0, 16);
        if (d == 0.0f) continue;
        const float id = 1.0f / d;
        for (int i = 0; i < 32; ++i) {
            int q = (int)nearbyintf(p[i] * id);
            if (q < -8) q = -8;
            if (q > 7) q = 7;
            const uint8_t nib = (uint8_t)(q + 8);
            blk[4 + i / 2] |= (i & 1) ? (uint8_t)(nib << 4) : nib;
        }
    }
}

static float rdf32(const uint8_t* p) { float f; memcpy(&f, p, 4); return f; }

/* dot_q4_q8 (internal): per block sum += float(isum)*a.d*x.d.
 * src/quant_kernels.cpp:52-66. */
static float int_dot_q4_q8(const uint8_t* a20, const uint8_t* x36, size_t nb) {
    float sum = 0.0f;
    for (size_t b = 0; b < nb; ++b) {
        const uint8_t* a = a20 + b * 20;
        const uint8_t* x = x36 + b * 36;
        int isum = 0;
        for (int k = 0; k < 32; ++k) {
            const uint8_t pk = a[4 + k / 2];
            const int q4 = ((k & 1) ? (pk >> 4) : (pk & 15)) - 8;
            isum += q4 * (int)(int8_t)x[4 + k];
        }
        sum += (float)isum * rdf32(a) * rdf32(x);   /* GCC leaves this one uncontracted */
    }
    return sum;
}

/* dot_q4_0 (internal, AVX2 order): de-interleave to q0..q31, 8 FMA lanes
 * over elements (lane l: l, 8+l, 16+l, 24+l), hsum, sum += s*d.
 * src/quant.cpp:111-156. */
static float int_dot_q4_0(const uint8_t* a20, const float* x, size_t nb) {
    float sum = 0.0f;
    for (size_t b = 0; b < nb; ++b) {
        const uint8_t* a = a20 + b * 20;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int k = 0; k < 32; ++k) {
            const uint8_t pk = a[4 + k / 2];
            const int q = ((k & 1) ? (pk >> 4) : (pk & 15)) - 8;
            acc[k % 8] = fmaf((float)q, x[b * 32 + k], acc[k % 8]);
        }
        sum = fmaf(hsum8(acc), rdf32(a), sum);
    }
    return sum;
}

/* dot_q8_0 (internal, AVX2 order).  src/quant.cpp:87-109. */
static float int_dot_q8_0(const uint8_t* a36, const float* x, size_t nb) {
    float sum = 0.0f;
    for (size_t b = 0; b < nb; ++b) {
        const uint8_t* a = a36 + b * 36;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int k = 0; k < 32; ++k) acc[k % 8] = fmaf((float)(int8_t)a[4 + k], x[b * 32 + k], acc[k % 8]);
        sum = fmaf(hsum8(acc), rdf32(a), sum);
    }
    return sum;
}

/* matvec_q4_q8 / matvec_q4_0 / matvec_q8_0 / matmul_q4_0_batch.
 * src/quant_kernels.cpp:68-91, src/quant.cpp:158-174. */
MVO_API void mvo_int_matvec_q4_q8(const uint8_t* A20, const uint8_t* x36, float* y, size_t rows, size_t cols) {
    for (size_t r = 0; r < rows; ++r) y[r] = int_dot_q4_q8(A20 + r * (cols / 32) * 20, x36, cols / 32);
}
MVO_API void mvo_int_matvec_q4_0(const uint8_t* A20, const float* x, float* y, size_t rows, size_t cols) {
    for (size_t r = 0; r < rows; ++r) y[r] = int_dot_q4_0(A20 + r * (cols / 32) * 20, x, cols / 32);
}
MVO_API void mvo_int_matvec_q8_0(const uint8_t* A36, const float* x, float* y, size_t rows, size_t cols) {
    for (size_t r = 0; r < rows; ++r) y[r] = int_dot_q8_0(A36 + r * (cols / 32) * 36, x, cols / 32);
}
MVO_API void mvo_int_matmul_q4_0_batch(const uint8_t* A20, const float* x, float* y, size_t rows, size_t cols,
                                       size_t batch) {
    for (size_t r = 0; r < rows; ++r)
        for (size_t b = 0; b < batch; ++b) y[b * rows + r] = int_dot_q4_0(A20 + r * (cols / 32) * 20, x + b * cols, cols / 32);
}

/* matvec_f32: sequential fp32 row dot; GCC neither reorders nor contracts
 * this reduction in the reference build.  src/matmul.cpp:6-8. */
MVO_API void mvo_matvec_f32(const float* A, const float* x, float* y, size_t rows, size_t cols) {
    for (size_t r = 0; r < rows; ++r) {
        float s = 0.0f;
        for (size_t c = 0; c < cols; ++c) s += A[r * cols + c] * x[c];
        y[r] = s;
    }
}
