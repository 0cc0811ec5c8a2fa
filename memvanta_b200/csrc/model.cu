// model.cu -- device-resident LlamaModel backend (mv_model_*).
//
// Mirrors the reference's LlamaModel (src/llama_model.cpp:222-263,
// include/memvanta/llama_model.hpp:100-138) with the weights, KV cache and
// activations resident in HBM:
//
//  * load: the GGUF is mmapped (gguf_loader.cpp); every tensor's blocks are
//    uploaded once.  Per layer, q|k|v are concatenated into one weight (rows
//    q, then k, then v) and gate/up are interleaved row by row (gate_i, up_i),
//    so one GEMV launch serves three (two) of the reference's tensor_matvec
//    calls.  The RoPE tables are built on the host with the reference's own
//    float expressions (:233) and uploaded.
//  * decode (forward): one CUDA graph per step --
//      embed(token) ; per layer { qkv GEMV with RMSNorm+Q8 prologue ;
//      RoPE + KV append ; paged attention in the reference's order ; o GEMV (+= x) ;
//      gate/up GEMV with RMSNorm+Q8 prologue and SiLU-gate epilogue ;
//      down GEMV (+= x) } ; output RMSNorm ; head matvec ; greedy argmax.
//    The token id and position live in device memory, so the same graph
//    replays for every position and greedy decoding never leaves the GPU.
//  * prefill: per chunk of B tokens the reference's MEMVANTA_FORCE_Q8_ACT=1
//    numerics -- RMSNorm, per-row Q8 activations, Q4_0 x Q8 GEMM, RoPE + KV
//    append, causal attention (token b sees positions <= start+b), SiLU gate,
//    residuals; a 1-token chunk takes the reference's fp32-activation path
//    (tensor_matmul_batch_v06 routes batch < 2 to tensor_matmul_batch, :263).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/memvanta_b200.h"
#include "common.cuh"
#include "gguf_loader.hpp"
#include "kernels.cuh"
#include "tc.cuh"
#include "weights.cuh"

namespace mvb {

// ------------------------------------------------------------- kernels

// RoPE (half-split, the reference's GCC roundings: fma(x0,c,-(x1*s)) and
// fma(x0,s,x1*c)) on the q and k parts of each qkv row, and the k and v parts
// into the paged cache (F32 copy / F16 with the reference rounding / Q8_0 per
// 32-element block).  Grid (rows, ceil((n_head + 2*n_head_kv) / upc)): each
// CTA takes upc units -- a q head (rotate), k head (rotate + store) or v head
// (store).  ctx_out (optional) receives pos+1 for the attention that follows.
constexpr int kRopeUnits = 6;  // units a thread holds at once in the F32/F16 path
__global__ void rope_append_heads_kernel(float* __restrict__ qkv, int ld, int n_head, int n_head_kv, int hd,
                                         const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                         const int32_t* __restrict__ pos, int kv_type, const int32_t* __restrict__ table, int table_ld,
                                         int page, uint8_t* __restrict__ k_pages, uint8_t* __restrict__ v_pages,
                                         float* __restrict__ k_scales, float* __restrict__ v_scales,
                                         int32_t* __restrict__ ctx_out, int upc) {
    // upc units per CTA, taken four at a time (blockDim.x / 4 threads each): a
    // prefill batch gives each CTA many heads, so the chain position ->
    // cos/sin -> block table is waited for once per many heads
    const int nsub = 4, T = (int)blockDim.x / nsub, sub = (int)threadIdx.x / T, tt = (int)threadIdx.x % T;
    const int units = n_head + 2 * n_head_kv;
    const int r = blockIdx.x, u0 = (int)blockIdx.y * upc, uend = min(u0 + upc, units), half = hd / 2,
              KV = n_head_kv * hd;
    pdl_trigger();
    pdl_wait();
    float* row = qkv + (size_t)r * ld;
    const int p = pos[r];
    const float* co = cos_t + (size_t)p * half;
    const float* si = sin_t + (size_t)p * half;
    if (kv_type <= 1 && T == half && upc <= kRopeUnits * nsub) {
        // F32 / F16 pages: thread tt holds the pair (tt, tt + half) of each of
        // its units -- all loads first, then the rotation (q and k heads,
        // written back) and the append (k and v heads) from registers
        const int nrot = n_head + n_head_kv;
        const size_t slot = uend > n_head ? (size_t)table[(size_t)r * table_ld + p / page] * page + p % page : 0;
        const float c = co[tt], s = si[tt];
        float x0[kRopeUnits], x1[kRopeUnits];
#pragma unroll
        for (int k = 0; k < kRopeUnits; ++k) {
            const int unit = u0 + sub + k * nsub;
            if (unit < uend) {
                x0[k] = row[(size_t)unit * hd + tt];
                x1[k] = row[(size_t)unit * hd + tt + half];
            }
        }
#pragma unroll
        for (int k = 0; k < kRopeUnits; ++k) {
            const int unit = u0 + sub + k * nsub;
            if (unit >= uend) continue;
            float y0 = x0[k], y1 = x1[k];
            if (unit < nrot) {
                y0 = __fmaf_rn(x0[k], c, -__fmul_rn(x1[k], s));
                y1 = __fmaf_rn(x0[k], s, __fmul_rn(x1[k], c));
                row[(size_t)unit * hd + tt] = y0;
                row[(size_t)unit * hd + tt + half] = y1;
            }
            if (unit >= n_head) {
                const bool is_v = unit >= nrot;
                const int head = unit - n_head - (is_v ? n_head_kv : 0);
                const size_t base = slot * KV + (size_t)head * hd;
                if (kv_type == 0) {
                    float* dst = reinterpret_cast<float*>(is_v ? v_pages : k_pages) + base;
                    dst[tt] = y0;
                    dst[tt + half] = y1;
                } else {
                    uint16_t* dst = reinterpret_cast<uint16_t*>(is_v ? v_pages : k_pages) + base;
                    dst[tt] = f32_to_f16_ref(y0);
                    dst[tt + half] = f32_to_f16_ref(y1);
                }
            }
        }
        if (ctx_out && blockIdx.y == 0 && threadIdx.x == 0) ctx_out[r] = p + 1;
        return;
    }
#pragma unroll 2
    for (int unit = u0 + sub; unit < min(uend, n_head + n_head_kv); unit += nsub) {  // q heads, then k heads
        float* b = row + (size_t)unit * hd;
        for (int j = tt; j < half; j += T) {
            const float x0 = b[j], x1 = b[j + half], c = co[j], s = si[j];
            b[j] = __fmaf_rn(x0, c, -__fmul_rn(x1, s));
            b[j + half] = __fmaf_rn(x0, s, __fmul_rn(x1, c));
        }
    }
    __syncthreads();
    if (uend > n_head) {
        const size_t slot = (size_t)table[(size_t)r * table_ld + p / page] * page + p % page;
        for (int unit = max(u0, n_head) + sub; unit < uend; unit += nsub) {  // k heads, then v heads
            const float* b = row + (size_t)unit * hd;
            const bool is_v = unit >= n_head + n_head_kv;
            const int head = unit - n_head - (is_v ? n_head_kv : 0);
            uint8_t* pages = is_v ? v_pages : k_pages;
            const size_t base = slot * KV + (size_t)head * hd;
            if (kv_type == 0) {
                float* dst = reinterpret_cast<float*>(pages) + base;
                for (int i = tt; i < hd; i += T) dst[i] = b[i];
            } else if (kv_type == 1) {
                uint16_t* dst = reinterpret_cast<uint16_t*>(pages) + base;
                for (int i = tt; i < hd; i += T) dst[i] = f32_to_f16_ref(b[i]);
            } else {  // Q8_0: warp per 32-element block (T is a multiple of 32)
                float* scales = is_v ? v_scales : k_scales;
                int8_t* dst = reinterpret_cast<int8_t*>(pages) + base;
                const int lane = tt & 31;
                for (int blk = tt >> 5; blk < hd / 32; blk += T >> 5) {
                    float dd;
                    dst[blk * 32 + lane] = (int8_t)quant_q8_lane(b[blk * 32 + lane], dd);
                    if (lane == 0) scales[slot * (KV / 32) + (size_t)head * (hd / 32) + blk] = dd;
                }
            }
        }
    }
    if (ctx_out && blockIdx.y == 0 && threadIdx.x == 0) ctx_out[r] = p + 1;
}

// The MV_KV_Q8 cache keeps one scale per token over all kv_dim elements, so
// its store needs the whole row: RoPE and store in one CTA per row.
// RoPE (half-split, the reference's GCC roundings) on the q and k parts of
// one qkv row, then the k and v parts into the paged cache.  One CTA per row.
// ctx_out (optional) receives pos+1 for the attention that follows.
__global__ void rope_append_row_kernel(float* __restrict__ qkv, int ld, int n_head, int n_head_kv, int hd,
                                   const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                   const int32_t* __restrict__ pos, int kv_type, const int32_t* __restrict__ table, int table_ld,
                                   int page, uint8_t* __restrict__ k_pages, uint8_t* __restrict__ v_pages,
                                   float* __restrict__ k_scales, float* __restrict__ v_scales,
                                   int32_t* __restrict__ ctx_out) {
    const int r = blockIdx.x, half = hd / 2, D = n_head * hd, KV = n_head_kv * hd;
    pdl_trigger();
    pdl_wait();
    float* row = qkv + (size_t)r * ld;
    const int p = pos[r];
    const float* co = cos_t + (size_t)p * half;
    const float* si = sin_t + (size_t)p * half;
    for (int i = threadIdx.x; i < (n_head + n_head_kv) * half; i += blockDim.x) {
        const int h = i / half, j = i % half;
        float* b = row + h * hd;  // k heads directly follow the q heads in the row
        const float x0 = b[j], x1 = b[j + half], c = co[j], s = si[j];
        b[j] = __fmaf_rn(x0, c, -__fmul_rn(x1, s));
        b[j + half] = __fmaf_rn(x0, s, __fmul_rn(x1, c));
    }
    __syncthreads();
    const size_t slot = (size_t)table[(size_t)r * table_ld + p / page] * page + p % page;
    for (int which = 0; which < 2; ++which) {
        const float* src = row + D + which * KV;
        uint8_t* pages = which ? v_pages : k_pages;
        float* scales = which ? v_scales : k_scales;
        if (kv_type == 0) {
            float* dst = reinterpret_cast<float*>(pages) + slot * KV;
            for (int i = threadIdx.x; i < KV; i += blockDim.x) dst[i] = src[i];
        } else if (kv_type == 1) {
            uint16_t* dst = reinterpret_cast<uint16_t*>(pages) + slot * KV;
            for (int i = threadIdx.x; i < KV; i += blockDim.x) dst[i] = f32_to_f16_ref(src[i]);
        } else if (kv_type == 2) {
            __shared__ float red[32];
            float m = 0.0f;
            for (int i = threadIdx.x; i < KV; i += blockDim.x) m = fmaxf(m, fabsf(src[i]));
            m = warp_max(m);
            const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
            if (lane == 0) red[warp] = m;
            __syncthreads();
            if (warp == 0) {
                float t = lane < nw ? red[lane] : 0.0f;
                t = warp_max(t);
                if (lane == 0) red[0] = t;
            }
            __syncthreads();
            const float sc = red[0] > 0.0f ? red[0] / 127.0f : 1.0f;
            int8_t* dst = reinterpret_cast<int8_t*>(pages) + slot * KV;
            for (int i = threadIdx.x; i < KV; i += blockDim.x) {
                float q = roundf(src[i] / sc);
                dst[i] = (int8_t)(int)fminf(fmaxf(q, -127.0f), 127.0f);
            }
            if (threadIdx.x == 0) scales[slot] = sc;
            __syncthreads();  // red[] is reused by the V pass
        } else {
            int8_t* dst = reinterpret_cast<int8_t*>(pages) + slot * KV;
            const int lane = threadIdx.x & 31;
            for (int b = threadIdx.x >> 5; b < KV / 32; b += blockDim.x >> 5) {
                float dd;
                dst[b * 32 + lane] = (int8_t)quant_q8_lane(src[b * 32 + lane], dd);
                if (lane == 0) scales[slot * (KV / 32) + b] = dd;
            }
        }
    }
    if (ctx_out && threadIdx.x == 0) ctx_out[r] = p + 1;
}

// Prefill: gate/up rows come interleaved (g_i, u_i); ff = g/(1+exp(-g)) * u.
__global__ void silu_pairs_kernel(const float* __restrict__ gu, float* __restrict__ ff, uint64_t n) {
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const float g = gu[2 * i], u = gu[2 * i + 1];
        ff[i] = (g / (1.0f + expf(-g))) * u;
    }
}

// Greedy step tail: argmax (first index of the max, as std::max_element in
// Sampler::sample, src/llama_model.cpp:60) -> next token, token history at
// the current position, position + 1.
__global__ void greedy_step_kernel(const float* __restrict__ logits, int n, int32_t* __restrict__ token,
                                   int32_t* __restrict__ pos, int32_t* __restrict__ history) {
    __shared__ float sv[32];
    __shared__ int si[32];
    pdl_trigger();
    pdl_wait();
    float v = -INFINITY;
    int idx = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float x = __ldcg(logits + i);  // L2: other GPUs write their vocab slices
        if (x > v || (x == v && i < idx)) {
            v = x;
            idx = i;
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
        if (v2 > v || (v2 == v && i2 < idx)) {
            v = v2;
            idx = i2;
        }
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
        for (int o = 16; o > 0; o >>= 1) {
            const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
            const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
            if (v2 > v || (v2 == v && i2 < idx)) {
                v = v2;
                idx = i2;
            }
        }
        if (lane == 0) {
            const int t = idx == 0x7fffffff ? 0 : idx;
            const int p = *pos;
            *token = t;
            history[p] = t;
            *pos = p + 1;
        }
    }
}

// Decode without logits still advances the device position.
__global__ void advance_pos_kernel(int32_t* __restrict__ pos) {
    pdl_wait();
    *pos += 1;
}

// Token id and position of the next decode step, passed by value so no host
// staging buffer has to outlive the launch.
__global__ void set_inputs_kernel(int32_t* __restrict__ token_dev, int32_t* __restrict__ pos_dev, int32_t token,
                                  int32_t pos) {
    *token_dev = token;
    *pos_dev = pos;
}

unsigned ew_grid(uint64_t n) {
    const uint64_t g = (n + 255) / 256, cap = (uint64_t)num_sms() * 8;
    return (unsigned)(g < cap ? (g ? g : 1) : cap);
}

// --------------------------------------------------------------- model

struct DevBuf {
    void* p = nullptr;
    ~DevBuf() {
        if (p) cudaFree(p);
    }
    template <class T>
    T* as() const { return static_cast<T*>(p); }
};

struct Layer {
    mv_weight_s* qkv = nullptr;
    mv_weight_s* o = nullptr;
    mv_weight_s* gu = nullptr;
    mv_weight_s* down = nullptr;
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
    uint8_t* k_pages = nullptr;
    uint8_t* v_pages = nullptr;
    float* k_scales = nullptr;
    float* v_scales = nullptr;
};

}  // namespace mvb

struct mv_model_s {
    int device = 0;
    cudaStream_t stream = nullptr;
    // config (LlamaConfig, include/memvanta/llama_model.hpp:14-26)
    uint64_t n_ctx = 0, n_embd = 0, n_ff = 0, n_layer = 0, n_head = 0, n_head_kv = 0, vocab = 0;
    float eps = 1e-5f, theta = 10000.0f;
    uint64_t hd = 0, kv_dim = 0, page = 128, n_pages = 0;
    int kv_type = MV_KV_F16;
    uint64_t pos = 0;

    std::vector<mv_weight_s*> owned;  // every uploaded weight
    mv_weight_s* tok_embd = nullptr;
    mv_weight_s* output = nullptr;
    float* output_norm = nullptr;
    std::vector<mvb::Layer> layers;

    std::vector<void*> allocs;             // every other device allocation
    float* rope_cos = nullptr;
    float* rope_sin = nullptr;
    int32_t* table = nullptr;              // [max_q][n_pages] identity rows
    uint64_t table_rows = 0;
    // set while a prefill fills one sequence of a sequence set (mv_seqs_s):
    // the layers with that sequence's cache pages
    const std::vector<mvb::Layer>* kv_layers = nullptr;

    // decode state (device)
    float *x = nullptr, *qkv = nullptr, *att = nullptr, *ff = nullptr, *gu = nullptr, *nrm = nullptr;
    float* logits = nullptr;
    int32_t *token_dev = nullptr, *pos_dev = nullptr, *ctx_dev = nullptr, *history = nullptr;
    float* logits_host = nullptr;          // pinned
    cudaGraphExec_t graph_logits = nullptr, graph_nologits = nullptr;
    // decode attention in the reference's order (attention.cu), or split
    // over the context (attn_split.cu) with MV_ATTN_SPLIT=1: ~1e-6 from the
    // reference order per step, which later Q8 activation roundings amplify
    // past the end-to-end logits bar, so it is not the default
    bool attn_split = false;
    // F16/F32 reference-order decode attention over a cluster of CTAs per
    // head (attn_cluster.cu) where its staging fits; MV_ATTN_CLUSTER=0 keeps
    // the one-CTA-per-head kernel (attention.cu)
    bool attn_cluster = false;
    // one GPU, MV_DECODE_PREQUANT: the o and down GEMVs take their inputs
    // already quantised by the kernels before them (the cluster attention,
    // the gate|up GEMV) in these buffers (q8_act_bytes layout); else nullptr
    uint8_t* attq = nullptr;
    uint8_t* ffq = nullptr;
    // one GPU: every layer of a decode step in one persistent kernel
    // (decode_mk.cu), with MV_DECODE_PERSISTENT=1 where supported
    bool mk = false;
    int mk_stages = 0;
    mvb::MkLayer* mk_layers = nullptr;     // device [n_layer]
    CUtensorMap* mk_maps = nullptr;        // device [n_layer][4][2]
    unsigned* mk_bar = nullptr;
    int* mk_status = nullptr;              // device [2]: site, abort
    int* mk_status_host = nullptr;         // pinned copy of mk_status[0]

    // prefill buffers (grown on demand)
    uint64_t pf_cap = 0;
    float *X = nullptr, *N = nullptr, *QKV = nullptr, *ATT = nullptr, *GU = nullptr, *FF = nullptr, *PROJ = nullptr;
    int8_t* XQ = nullptr;
    float* XD = nullptr;
    // Single GPU: consecutive chunks of a prefill call alternate between two
    // buffer sets and two streams, so chunk c + 1 runs one layer behind chunk
    // c and its kernels fill the SMs chunk c's kernels leave idle.  Chunk
    // c + 1's layer-l attention reads chunk c's layer-l K/V: it waits for
    // pf_ev[c % 2][l], recorded after chunk c's layer-l KV append.
    struct PfSet {
        float *X = nullptr, *N = nullptr, *QKV = nullptr, *ATT = nullptr, *GU = nullptr, *FF = nullptr,
              *PROJ = nullptr;
        int8_t* XQ = nullptr;
        float* XD = nullptr;
        cudaStream_t stream = nullptr;
    } pf_alt;
    std::vector<cudaEvent_t> pf_ev[2];
    const std::vector<cudaEvent_t>* pf_wait = nullptr;  // the previous chunk's events (nullptr: first chunk)
    const std::vector<cudaEvent_t>* pf_rec = nullptr;   // this chunk's events
    cudaEvent_t pf_join = nullptr;                      // main stream <-> alternate stream
    // token ids / positions / context lengths of a whole prefill call
    uint64_t in_cap = 0;
    int32_t *pf_tok = nullptr, *pf_pos = nullptr, *pf_ctx = nullptr;
    int32_t* pf_host = nullptr;            // pinned staging, 3 * in_cap

    // Tensor parallelism (tp.cuh).  This rank holds q heads [rank*nh, +nh), kv
    // heads [rank*nkv, +nkv) with their KV cache, o/down rows [rank*Dl, +Dl),
    // ff rows [rank*Fl, +Fl) of gate and up, head rows [rank*Vl, +Vl); every
    // GEMV keeps its full contraction, so the outputs equal one GPU's bit for
    // bit.  One rank: the local sizes equal the global ones.
    int tp_rank = 0, tp_world = 1;
    uint64_t nh = 0, nkv = 0, kvd = 0, qkvw = 0, Dl = 0, Fl = 0, Vl = 0;
    char* tp_block = nullptr;               // this rank's shared block (IPC-exported)
    uint64_t tp_bytes = 0, tp_bmax = 0;     // size; prefill rows it holds
    uint64_t off_x = 0, off_att = 0, off_ff = 0, off_logits = 0, off_X = 0, off_ATT = 0, off_FF = 0;
    std::vector<void*> tp_opened;           // peers' blocks mapped into this process
    mvb::TpCtx tp;
    int* tp_step = nullptr;
    unsigned* tp_counters = nullptr;
    int* tp_status = nullptr;
    long long* tp_limit = nullptr;          // wait bound in ns (device)
    float* logits_l = nullptr;              // this rank's vocab slice
    float *ATT_l = nullptr, *FF_l = nullptr, *PROJ_l = nullptr;  // prefill slices
    bool tp_ready = false;                  // peers connected, graphs captured
    int* tp_status_host = nullptr;          // pinned copy of tp_status
};

namespace {

thread_local std::string g_model_err;

struct ModelError : std::runtime_error {
    int code;
    ModelError(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

void ck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        throw ModelError(e == cudaErrorMemoryAllocation ? MV_ERR_OOM : MV_ERR_CUDA,
                         std::string(what) + ": " + cudaGetErrorString(e));
    }
}

template <class T>
T* dalloc(mv_model_s* m, uint64_t count) {
    void* p = nullptr;
    ck(cudaMalloc(&p, count * sizeof(T) + 16), "cudaMalloc(model)");
    m->allocs.push_back(p);
    return static_cast<T*>(p);
}

// One contiguous run of a tensor's raw GGML bytes, in upload order.
struct Seg {
    const uint8_t* src;
    uint64_t n;
};

// GGUF -> HBM upload pipeline.  A tensor's raw blocks go from the mapped file
// through two pinned chunks -- the CPU gathers the next chunk (page-faulting
// the file in, interleaving gate/up rows, slicing a rank's share) while the
// copy engine sends the previous one -- into a device staging buffer, and
// the repack kernel turns them into the planar layout the kernels read
// (mv_weight_from_device).  The staging buffer is reused for every tensor
// and freed with the uploader.
struct Uploader {
    static constexpr uint64_t kChunk = 8ull << 20;
    cudaStream_t s;
    uint8_t* pin[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    int cur = 0;
    uint8_t* dstage = nullptr;
    uint64_t dcap = 0;

    explicit Uploader(cudaStream_t st) : s(st) {
        for (int k = 0; k < 2; ++k) {
            ck(cudaMallocHost(reinterpret_cast<void**>(&pin[k]), kChunk), "cudaMallocHost(upload)");
            ck(cudaEventCreateWithFlags(&ev[k], cudaEventDisableTiming), "cudaEventCreate(upload)");
        }
    }
    ~Uploader() {
        cudaStreamSynchronize(s);
        for (int k = 0; k < 2; ++k) {
            if (pin[k]) cudaFreeHost(pin[k]);
            if (ev[k]) cudaEventDestroy(ev[k]);
        }
        if (dstage) cudaFree(dstage);
    }

    mv_weight_s* upload(mv_model_s* m, const std::vector<Seg>& segs, int type, uint64_t rows, uint64_t cols) {
        uint64_t total = 0;
        for (const Seg& g : segs) total += g.n;
        if (total > dcap) {
            ck(cudaStreamSynchronize(s), "sync(upload)");
            if (dstage) cudaFree(dstage);
            dstage = nullptr;
            ck(cudaMalloc(reinterpret_cast<void**>(&dstage), total), "cudaMalloc(upload staging)");
            dcap = total;
        }
        size_t si = 0;
        uint64_t so = 0;
        for (uint64_t off = 0; off < total;) {
            const uint64_t c = std::min(kChunk, total - off);
            ck(cudaEventSynchronize(ev[cur]), "upload chunk free");  // its previous copy has finished
            for (uint64_t filled = 0; filled < c;) {
                const uint64_t take = std::min(c - filled, segs[si].n - so);
                std::memcpy(pin[cur] + filled, segs[si].src + so, take);
                filled += take;
                so += take;
                if (so == segs[si].n) ++si, so = 0;
            }
            ck(cudaMemcpyAsync(dstage + off, pin[cur], c, cudaMemcpyHostToDevice, s), "upload copy");
            ck(cudaEventRecord(ev[cur], s), "upload event");
            cur ^= 1;
            off += c;
        }
        mv_weight_t w = nullptr;
        if (int rc = mv_weight_from_device(dstage, total, type, rows, cols, s, &w))  // repack, then sync
            throw ModelError(rc, std::string("weight upload: ") + mv_last_error());
        m->owned.push_back(w);
        return w;
    }
};

mv_weight_s* upload_tensor(mv_model_s* m, Uploader& up, const mvb::GgufReader& f, const mvb::GgufTensorInfo& t) {
    if (t.dims.size() < 2) throw ModelError(MV_ERR_INVALID, "matrix tensor needs rank 2: " + t.name);
    return up.upload(m, {{f.data(t), t.nbytes}}, (int)t.type, t.ne(1), t.ne(0));
}

float* upload_vector(mv_model_s* m, const mvb::GgufReader& f, const mvb::GgufTensorInfo& t, uint64_t n) {
    // tensor_vector_to_f32 (src/gguf_kernels.cpp:224): F32 copied, F16 widened
    if (t.elements() != n) throw ModelError(MV_ERR_INVALID, "tensor vector size mismatch: " + t.name);
    std::vector<float> v(n);
    if (t.type == 0) {
        std::memcpy(v.data(), f.data(t), n * 4);
    } else if (t.type == 1) {
        const uint16_t* h = reinterpret_cast<const uint16_t*>(f.data(t));
        for (uint64_t i = 0; i < n; ++i) {
            const uint32_t s = (h[i] >> 15) & 1u, e = (h[i] >> 10) & 31u, mm = h[i] & 1023u;
            float val;
            if (e == 0) val = std::ldexp((float)mm, -24);
            else if (e == 31) val = mm ? NAN : INFINITY;
            else val = std::ldexp((float)(mm | 1024u), (int)e - 25);
            v[i] = s ? -val : val;
        }
    } else {
        throw ModelError(MV_ERR_UNSUPPORTED, "unsupported vector tensor type: " + t.name);
    }
    float* d = dalloc<float>(m, n);
    ck(cudaMemcpy(d, v.data(), n * 4, cudaMemcpyHostToDevice), "upload vector");
    return d;
}

// Rows [r0, r0 + n) of a matrix tensor (whole rows are contiguous bytes).
struct RowRange {
    const mvb::GgufTensorInfo* t;
    uint64_t r0, n;
};

mv_weight_s* upload_rows(mv_model_s* m, Uploader& up, const mvb::GgufReader& f, const std::vector<RowRange>& parts,
                         bool interleave) {
    const uint32_t type = parts[0].t->type;
    const uint64_t cols = parts[0].t->ne(0);
    for (auto& pr : parts)
        if (pr.t->type != type || pr.t->ne(0) != cols || pr.t->dims.size() < 2 || pr.r0 + pr.n > pr.t->ne(1))
            throw ModelError(MV_ERR_UNSUPPORTED, "row slices to fuse differ in type or width: " + pr.t->name);
    const uint64_t row_bytes = parts[0].t->nbytes / parts[0].t->ne(1);
    uint64_t rows = 0;
    for (auto& pr : parts) rows += pr.n;
    std::vector<Seg> segs;
    if (interleave) {  // gate/up: row 2i = gate_i, row 2i+1 = up_i
        if (parts.size() != 2 || parts[0].n != parts[1].n)
            throw ModelError(MV_ERR_INVALID, "gate/up shapes differ: " + parts[0].t->name);
        const uint8_t* g = f.data(*parts[0].t) + parts[0].r0 * row_bytes;
        const uint8_t* u = f.data(*parts[1].t) + parts[1].r0 * row_bytes;
        segs.reserve(2 * parts[0].n);
        for (uint64_t i = 0; i < parts[0].n; ++i) {
            segs.push_back({g + i * row_bytes, row_bytes});
            segs.push_back({u + i * row_bytes, row_bytes});
        }
    } else {
        for (auto& pr : parts) segs.push_back({f.data(*pr.t) + pr.r0 * row_bytes, pr.n * row_bytes});
    }
    return up.upload(m, segs, (int)type, rows, cols);
}

// Concatenates whole rows of same-typed, same-width tensors (raw GGML bytes).
mv_weight_s* upload_concat(mv_model_s* m, Uploader& up, const mvb::GgufReader& f,
                           const std::vector<const mvb::GgufTensorInfo*>& ts, bool interleave) {
    const uint32_t type = ts[0]->type;
    const uint64_t cols = ts[0]->ne(0);
    for (auto* t : ts)
        if (t->type != type || t->ne(0) != cols || t->dims.size() < 2)
            throw ModelError(MV_ERR_UNSUPPORTED, "layer tensors to fuse differ in type or width: " + t->name);
    const uint64_t row_bytes = ts[0]->nbytes / ts[0]->ne(1);
    uint64_t rows = 0;
    for (auto* t : ts) rows += t->ne(1);
    std::vector<Seg> segs;
    if (interleave) {  // gate/up: row 2i = gate_i, row 2i+1 = up_i
        if (ts.size() != 2 || ts[0]->ne(1) != ts[1]->ne(1))
            throw ModelError(MV_ERR_INVALID, "gate/up shapes differ: " + ts[0]->name);
        const uint8_t* g = f.data(*ts[0]);
        const uint8_t* u = f.data(*ts[1]);
        segs.reserve(2 * ts[0]->ne(1));
        for (uint64_t i = 0; i < ts[0]->ne(1); ++i) {
            segs.push_back({g + i * row_bytes, row_bytes});
            segs.push_back({u + i * row_bytes, row_bytes});
        }
    } else {
        for (auto* t : ts) segs.push_back({f.data(*t), t->nbytes});
    }
    return up.upload(m, segs, (int)type, rows, cols);
}

void ensure_prefill(mv_model_s* m, uint64_t B) {
    if (B <= m->pf_cap) return;
    const uint64_t D = m->n_embd, F = m->n_ff;
    const uint64_t K = std::max(D, F);
    const bool tp = m->tp_world > 1;
    if (tp && B > m->tp_bmax)
        throw ModelError(MV_ERR_INVALID, "prefill batch above the tensor-parallel prefill buffers (" +
                                             std::to_string(m->tp_bmax) + " tokens)");
    // replicated X / ATT / FF live in the shared block under tensor parallelism
    m->X = tp ? reinterpret_cast<float*>(m->tp_block + m->off_X) : dalloc<float>(m, B * D);
    m->N = dalloc<float>(m, B * D);
    m->QKV = dalloc<float>(m, B * m->qkvw);
    m->ATT = tp ? reinterpret_cast<float*>(m->tp_block + m->off_ATT) : dalloc<float>(m, B * D);
    m->GU = dalloc<float>(m, B * 2 * m->Fl);
    m->FF = tp ? reinterpret_cast<float*>(m->tp_block + m->off_FF) : dalloc<float>(m, B * F);
    m->PROJ = dalloc<float>(m, B * D);
    if (tp) {
        m->ATT_l = dalloc<float>(m, B * m->Dl);
        m->FF_l = dalloc<float>(m, B * m->Fl);
        m->PROJ_l = dalloc<float>(m, B * m->Dl);
    }
    m->XQ = dalloc<int8_t>(m, B * K * 2);  // int8, or fp16 for the fp16 tensor-core GEMM
    m->XD = dalloc<float>(m, 2 * mvb::gemm_tc_ldb(B) * K / 32);  // block-major scales + constants
    if (!tp) {
        auto& a = m->pf_alt;
        a.X = dalloc<float>(m, B * D);
        a.N = dalloc<float>(m, B * D);
        a.QKV = dalloc<float>(m, B * m->qkvw);
        a.ATT = dalloc<float>(m, B * D);
        a.GU = dalloc<float>(m, B * 2 * m->Fl);
        a.FF = dalloc<float>(m, B * F);
        a.PROJ = dalloc<float>(m, B * D);
        a.XQ = dalloc<int8_t>(m, B * K * 2);
        a.XD = dalloc<float>(m, 2 * mvb::gemm_tc_ldb(B) * K / 32);
        if (!a.stream) ck(cudaStreamCreateWithFlags(&a.stream, cudaStreamNonBlocking), "cudaStreamCreate(prefill)");
        if (!m->pf_join) ck(cudaEventCreateWithFlags(&m->pf_join, cudaEventDisableTiming), "cudaEventCreate(prefill)");
        for (auto& v : m->pf_ev)
            while (v.size() < m->n_layer) {
                cudaEvent_t e;
                ck(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate(prefill)");
                v.push_back(e);
            }
    }
    if (B > m->table_rows) {
        std::vector<int32_t> t(B * m->n_pages);
        for (uint64_t r = 0; r < B; ++r)
            for (uint64_t p = 0; p < m->n_pages; ++p) t[r * m->n_pages + p] = (int32_t)p;
        m->table = dalloc<int32_t>(m, t.size());
        ck(cudaMemcpy(m->table, t.data(), t.size() * 4, cudaMemcpyHostToDevice), "table upload");
        m->table_rows = B;
    }
    m->pf_cap = B;
}

// x_out = W x_in for one weight of any type, with the decode path's fused
// prologue/epilogue where the weight is Q4_0.
// xq: the input already quantised (Q4_0 weights only); yq: SiluGate also
// writes its outputs quantised.
void project_decode(mv_model_s* m, mv_weight_s* w, const float* x, const float* norm_w, float* y, mvb::Q4Epi epi,
                    int reserve = 0, void* yq = nullptr, const void* xq = nullptr) {
    cudaStream_t s = m->stream;
    if (w->type == 2) {
        mvb::GemvQ4Args a{w, x, norm_w, m->eps, y, norm_w ? mvb::Q4Pro::RmsNorm : mvb::Q4Pro::Plain, epi};
        if (xq) {
            a.x = static_cast<const float*>(xq);
            a.pro = mvb::Q4Pro::PreQuant;
        }
        a.reserve = reserve;
        a.yq = yq;
        ck(mvb::gemv_q4(a, s), "gemv_q4");
        return;
    }
    const float* in = x;
    if (norm_w) {
        ck(mvb::rmsnorm_rows(x, norm_w, 1, w->cols, m->eps, m->nrm, s), "rmsnorm");
        in = m->nrm;
    }
    if (epi == mvb::Q4Epi::Store) {
        if (w->type == 14 && w->cols * 4 <= 200 * 1024) ck(mvb::gemv_q6k(*w, in, y, s), "gemv_q6k");
        else if (w->type == 8 && w->cols * 4 <= 200 * 1024) ck(mvb::gemv_q8_0(*w, in, y, s), "gemv_q8_0");
        else ck(mvb::matmul_f32act(*w, in, 1, y, s), "matmul");
    } else if (epi == mvb::Q4Epi::AddTo) {
        ck(mvb::matmul_f32act(*w, in, 1, m->logits, s), "matmul");  // logits buffer as scratch
        ck(mvb::add_inplace(y, m->logits, w->rows, s), "add");
    } else {
        ck(mvb::matmul_f32act(*w, in, 1, m->gu, s), "matmul");
        mvb::silu_pairs_kernel<<<mvb::ew_grid(w->rows / 2), 256, 0, s>>>(m->gu, y, w->rows / 2);
        ck(cudaGetLastError(), "silu_pairs");
    }
}

// plain = true: a full-order launch, for a launch right after an event wait
// (the attention after it, a PDL launch, relies on this kernel's completion
// implying the event's).
// table: block-table rows of `table_ld` pages, row r for qkv row r (table_ld 0:
// every row is a token of the one sequence whose pages row 0 lists).
void rope_append(mv_model_s* m, const mvb::Layer& L, float* qkv, uint64_t rows, const int32_t* pos, int32_t* ctx_out,
                 bool plain = false, const int32_t* table = nullptr, int table_ld = 0) {
    if (!table) table = m->table;
    const uint64_t QKVW = m->qkvw;  // this rank's heads
    cudaError_t e;
    if (m->kv_type == MV_KV_Q8) {
        e = mvb::launch_opt(!plain, mvb::rope_append_row_kernel, dim3((unsigned)rows), dim3(256), 0, m->stream, qkv,
                            (int)QKVW, (int)m->nh, (int)m->nkv, (int)m->hd, (const float*)m->rope_cos,
                            (const float*)m->rope_sin, pos, m->kv_type, table, table_ld, (int)m->page,
                            L.k_pages, L.v_pages, L.k_scales, L.v_scales, ctx_out);
    } else {
        // four heads at a time per CTA; a prefill batch (rows x (heads + 2 kv
        // heads) units) gives each CTA 24 of them in turn, a decode step 4
        const int T = m->kv_type == MV_KV_Q8_0 ? (int)std::max<uint64_t>(64, m->hd) : (int)(m->hd / 2);
        const int upc = rows >= 64 ? 24 : 4, units = (int)(m->nh + 2 * m->nkv);
        e = mvb::launch_opt(!plain, mvb::rope_append_heads_kernel,
                            dim3((unsigned)rows, (unsigned)((units + upc - 1) / upc)), dim3(T * 4), 0,
                            m->stream, qkv, (int)QKVW, (int)m->nh, (int)m->nkv, (int)m->hd,
                            (const float*)m->rope_cos, (const float*)m->rope_sin, pos, m->kv_type,
                            table, table_ld, (int)m->page, L.k_pages, L.v_pages, L.k_scales, L.v_scales,
                            ctx_out, upc);
    }
    ck(e, "rope_append");
}

mvb::AttnArgs attn_args(mv_model_s* m, const mvb::Layer& L, const float* q, uint64_t q_stride, uint64_t n_q,
                        const int32_t* ctx, uint64_t max_ctx, float* out) {
    return mvb::AttnArgs{m->kv_type, q, q_stride, n_q, m->nh, m->nkv, m->hd, L.k_pages, L.v_pages,
                         L.k_scales, L.v_scales, m->table, m->n_pages, m->page, ctx, max_ctx, out};
}

// Sync points of one step under tensor parallelism (tp.cuh): per layer the
// attention heads, the o rows, the ff rows and the down rows, then the
// logits and (decode) the embedding.
int pt_att(uint64_t l) { return (int)(4 * l); }
int pt_o(uint64_t l) { return (int)(4 * l + 1); }
int pt_gu(uint64_t l) { return (int)(4 * l + 2); }
int pt_down(uint64_t l) { return (int)(4 * l + 3); }
int pt_head(const mv_model_s* m) { return (int)(4 * m->n_layer); }
int pt_embed(const mv_model_s* m) { return (int)(4 * m->n_layer + 1); }
int points_per_step(const mv_model_s* m) { return (int)(4 * m->n_layer + 2); }

// One Q4_0 GEMV of a tensor-parallel decode step: reads this rank's copy of
// the replicated LL input `x_off` once it carries point x_point; y == nullptr
// stores this rank's rows at `row_off` of every rank's LL output `y_off`
// (point y_point), otherwise y is a local float output.
void gemv_tp(mv_model_s* m, mv_weight_s* w, uint64_t x_off, int x_point, const float* norm_w, mvb::Q4Epi epi,
             float* y, uint64_t y_off, uint64_t row_off, int y_point, int res_point = 0, int reserve = 0) {
    mvb::GemvQ4Args a{w, nullptr, norm_w, m->eps, y, norm_w ? mvb::Q4Pro::RmsNorm : mvb::Q4Pro::Plain, epi};
    a.tp = &m->tp;
    a.x_ll = m->tp_block + x_off;
    a.x_point = x_point;
    a.y_shared = y_off;
    a.y_row_off = (int)row_off;
    a.y_point = y_point;
    a.res_point = res_point;
    a.reserve = reserve;
    ck(mvb::gemv_q4(a, m->stream), "gemv_q4 (tensor parallel)");
}

// Every kernel of one decode step, in order, on m->stream.
void launch_decode(mv_model_s* m, bool with_logits) {
    cudaStream_t s = m->stream;
    const bool tp = m->tp_world > 1;
    const uint64_t r = m->tp_rank;
    ck(mvb::read_rows(*m->tok_embd, m->token_dev, 1, m->x, s), "embed");
    if (tp) ck(mvb::tp_pack(m->tp, m->x, m->n_embd, m->off_x, pt_embed(m), s), "pack");
    // F16/F32 KV: RoPE, the KV append and the attention are one kernel
    const bool fused = m->kv_type == MV_KV_F32 || m->kv_type == MV_KV_F16;
    if (m->mk) {
        mvb::MkArgs a{};
        a.layers = m->mk_layers;
        a.maps = m->mk_maps;
        a.n_layer = (int)m->n_layer;
        a.n_head = (int)m->n_head;
        a.n_head_kv = (int)m->n_head_kv;
        a.hd = (int)m->hd;
        a.kv_type = m->kv_type;
        a.page = (int)m->page;
        a.max_ctx = (int)m->n_ctx;
        a.max_pages = (int)m->n_pages;
        a.eps = m->eps;
        a.x = m->x;
        a.qkv = m->qkv;
        a.att = m->att;
        a.ff = m->ff;
        a.cos_t = m->rope_cos;
        a.sin_t = m->rope_sin;
        a.pos = m->pos_dev;
        a.block_table = m->table;
        a.ctx_out = m->ctx_dev;
        a.bar = m->mk_bar;
        a.status = m->mk_status;
        a.stages = m->mk_stages;
        ck(mvb::decode_mk(a, s), "decode layers (persistent kernel)");
    }
    for (uint64_t l = 0; !m->mk && l < m->n_layer; ++l) {
        auto& L = m->layers[l];
        // the q|k|v GEMV leaves two CTA slots per attention CTA free (fused path)
        // (measured on the 7B step: 0, 32, 64, 96, 128 slots -> 681, 681, 683, 670, 651 tok/s)
        const int reserve = fused ? (int)(2 * m->nh) : 0;
        if (tp) gemv_tp(m, L.qkv, m->off_x, l ? pt_down(l - 1) : pt_embed(m), L.attn_norm, mvb::Q4Epi::Store, m->qkv,
                        0, 0, 0, 0, reserve);
        else project_decode(m, L.qkv, m->x, L.attn_norm, m->qkv, mvb::Q4Epi::Store, reserve);
        if (fused) {
            mvb::AttnFusedArgs fa{m->kv_type, m->qkv, m->nh, m->nkv, m->hd,
                                  (const float*)m->rope_cos, (const float*)m->rope_sin, m->pos_dev,
                                  (const int32_t*)m->table, m->n_pages, m->page, m->n_ctx,
                                  L.k_pages, L.v_pages, m->ctx_dev, m->att};
            if (tp) {
                fa.tp = m->tp;
                fa.out_shared = m->off_att;
                fa.head_off = (int)(r * m->nh);
                fa.out_point = pt_att(l);
            }
            fa.xq = m->attq;  // set only with the cluster kernel on one GPU
            ck(m->attn_split     ? mvb::attn_decode_fused_split(fa, s)
               : m->attn_cluster ? mvb::attn_decode_cluster(fa, s)
                                 : mvb::attn_decode_fused(fa, s),
               "attention (fused)");
        } else {
            rope_append(m, L, m->qkv, 1, m->pos_dev, m->ctx_dev);
            float* out = tp ? m->ATT_l : m->att;
            const mvb::AttnArgs aa = attn_args(m, L, m->qkv, m->qkvw, 1, m->ctx_dev, m->n_ctx, out);
            ck(m->attn_split ? mvb::paged_attn_decode_split(aa, s) : mvb::paged_attn_decode(aa, s), "attention");
            if (tp) ck(mvb::tp_scatter_ll(m->tp, out, m->Dl, m->off_att, r * m->Dl, pt_att(l), s), "scatter");
        }
        if (tp) {
            gemv_tp(m, L.o, m->off_att, pt_att(l), nullptr, mvb::Q4Epi::AddTo, nullptr, m->off_x, r * m->Dl, pt_o(l),
                    l ? pt_down(l - 1) : pt_embed(m));
            gemv_tp(m, L.gu, m->off_x, pt_o(l), L.ffn_norm, mvb::Q4Epi::SiluGate, nullptr, m->off_ff, r * m->Fl,
                    pt_gu(l));
            gemv_tp(m, L.down, m->off_ff, pt_gu(l), nullptr, mvb::Q4Epi::AddTo, nullptr, m->off_x, r * m->Dl,
                    pt_down(l), pt_o(l));
        } else {
            project_decode(m, L.o, m->att, nullptr, m->x, mvb::Q4Epi::AddTo, 0, nullptr, m->attq);
            project_decode(m, L.gu, m->x, L.ffn_norm, m->ff, mvb::Q4Epi::SiluGate, 0, m->ffq);
            project_decode(m, L.down, m->ff, nullptr, m->x, mvb::Q4Epi::AddTo, 0, nullptr, m->ffq);
        }
    }
    // every rank's down rows, as floats, before the head (and before the next
    // step's embedding reuses the buffer)
    if (tp) ck(mvb::tp_unpack(m->tp, m->off_x, m->n_embd, m->x, pt_down(m->n_layer - 1), s), "unpack");
    if (with_logits) {
        if (tp) {
            project_decode(m, m->output, m->x, m->output_norm, m->logits_l, mvb::Q4Epi::Store);
            ck(mvb::tp_scatter_ll(m->tp, m->logits_l, m->Vl, m->off_logits, r * m->Vl, pt_head(m), s), "scatter");
            ck(mvb::tp_unpack(m->tp, m->off_logits, m->vocab, m->logits, pt_head(m), s), "unpack");
        } else {
            project_decode(m, m->output, m->x, m->output_norm, m->logits, mvb::Q4Epi::Store);
        }
        ck(mvb::launch_pdl(mvb::greedy_step_kernel, dim3(1), dim3(1024), 0, s, (const float*)m->logits,
                           (int)m->vocab, m->token_dev, m->pos_dev, m->history),
           "greedy_step");
    } else {
        mvb::advance_pos_kernel<<<1, 1, 0, s>>>(m->pos_dev);
        ck(cudaGetLastError(), "advance_pos");
    }
    if (tp) ck(mvb::tp_step(m->tp_step, s), "tp step");
}

cudaGraphExec_t capture_decode(mv_model_s* m, bool with_logits) {
    cudaGraph_t g = nullptr;
    ck(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
    try {
        launch_decode(m, with_logits);
    } catch (...) {
        cudaStreamEndCapture(m->stream, &g);
        if (g) cudaGraphDestroy(g);
        throw;
    }
    ck(cudaStreamEndCapture(m->stream, &g), "end capture");
    cudaGraphExec_t exec = nullptr;
    cudaError_t e = cudaGraphInstantiate(&exec, g, 0);
    cudaGraphDestroy(g);
    ck(e, "graph instantiate");
    return exec;
}

void set_decode_inputs(mv_model_s* m, int32_t token) {
    mvb::set_inputs_kernel<<<1, 1, 0, m->stream>>>(m->token_dev, m->pos_dev, token, (int32_t)m->pos);
    ck(cudaGetLastError(), "set_inputs");
}

// Stages the token ids, positions and context lengths of a whole prefill
// call with one copy each.  The caller has synchronised the stream, so the
// pinned staging buffer is free to overwrite.
void stage_prefill_inputs(mv_model_s* m, const int32_t* tokens, uint64_t n, const uint64_t* row_pos = nullptr) {
    if (n > m->in_cap) {
        m->pf_tok = dalloc<int32_t>(m, n);
        m->pf_pos = dalloc<int32_t>(m, n);
        m->pf_ctx = dalloc<int32_t>(m, n);
        if (m->pf_host) cudaFreeHost(m->pf_host);
        m->pf_host = nullptr;
        ck(cudaMallocHost(reinterpret_cast<void**>(&m->pf_host), 3 * n * sizeof(int32_t)), "cudaMallocHost");
        m->in_cap = n;
    }
    for (uint64_t i = 0; i < n; ++i) {
        const uint64_t p = row_pos ? row_pos[i] : m->pos + i;  // row_pos: one decode row per sequence
        m->pf_host[i] = tokens[i];
        m->pf_host[n + i] = (int32_t)p;
        m->pf_host[2 * n + i] = (int32_t)(p + 1);
    }
    ck(cudaMemcpyAsync(m->pf_tok, m->pf_host, n * 4, cudaMemcpyHostToDevice, m->stream), "tokens H2D");
    ck(cudaMemcpyAsync(m->pf_pos, m->pf_host + n, n * 4, cudaMemcpyHostToDevice, m->stream), "pos H2D");
    ck(cudaMemcpyAsync(m->pf_ctx, m->pf_host + 2 * n, n * 4, cudaMemcpyHostToDevice, m->stream), "ctx H2D");
}

// One eager step (pos 0, token 0) makes every kernel's attributes and the
// library's lazy state ready before the decode graphs are captured; the KV
// row it writes at position 0 is overwritten by the first real token.  With
// tensor parallelism every rank runs it together (it synchronises).
void ready_decode(mv_model_s* m) {
    m->pos = 0;
    set_decode_inputs(m, 0);
    launch_decode(m, true);
    ck(cudaStreamSynchronize(m->stream), "warm-up step");
    m->graph_logits = capture_decode(m, true);
    m->graph_nologits = capture_decode(m, false);
    m->pos = 0;
    m->tp_ready = true;
}

// One GPU, Q4_0 layer weights, F16/F32 KV: the decode layers run as one
// persistent kernel (decode_mk.cu) when MV_DECODE_PERSISTENT=1.  Its
// outputs are bit-identical to the per-kernel path (reference-order
// attention).
void setup_persistent_decode(mv_model_s* m) {
    // opt-in while its step is slower than the per-kernel path's;
    // MV_DECODE_PERSISTENT=1 demands it: a model it cannot serve fails to open
    const char* env = std::getenv("MV_DECODE_PERSISTENT");
    if (!env || std::string(env) != "1") return;
    const bool forced = true;
    auto skip = [&](const std::string& why) {
        if (forced) throw ModelError(MV_ERR_UNSUPPORTED, "persistent decode kernel: " + why);
    };
    if (m->tp_world != 1) return skip("tensor parallel");
    if (m->kv_type != MV_KV_F32 && m->kv_type != MV_KV_F16) return skip("KV cache type is not F32/F16");
    if (m->n_head > (uint64_t)mvb::num_sms()) return skip("more heads than SMs");
    if (m->n_embd % 32 || m->n_ff % 32) return skip("n_embd / n_ff not multiples of 32");
    std::vector<mvb::MkLayer> hl(m->n_layer);
    uint64_t max_nb = 0;
    for (uint64_t l = 0; l < m->n_layer; ++l) {
        const auto& L = m->layers[l];
        const mv_weight_s* ws[4] = {L.qkv, L.o, L.gu, L.down};
        for (int i = 0; i < 4; ++i) {
            if (ws[i]->type != 2) return skip("layer weights are not Q4_0");
            max_nb = std::max(max_nb, ws[i]->nb);
            hl[l].w[i] = mvb::MkGemv{ws[i]->qs, ws[i]->d, (int)ws[i]->rows, (int)ws[i]->nb, (int)ws[i]->dstride};
        }
        hl[l].attn_norm = L.attn_norm;
        hl[l].ffn_norm = L.ffn_norm;
        hl[l].k_pages = L.k_pages;
        hl[l].v_pages = L.v_pages;
    }
    // the TMA maps of every layer weight's nibble and scale planes
    const mvb::tc::EncodeFn enc = mvb::tc::encode_fn();
    if (!enc) return skip("cuTensorMapEncodeTiled is unavailable");
    std::vector<CUtensorMap> maps(m->n_layer * 8);
    for (uint64_t l = 0; l < m->n_layer; ++l) {
        const auto& L = m->layers[l];
        const mv_weight_s* ws[4] = {L.qkv, L.o, L.gu, L.down};
        for (int i = 0; i < 4; ++i) {
            const mv_weight_s& w = *ws[i];
            const cuuint64_t qd[2] = {w.nb * 4, w.rows}, qst[1] = {w.nb * 16};
            const cuuint32_t qb[2] = {128, 16};
            const cuuint64_t dd[2] = {w.dstride, w.rows}, dst[1] = {w.dstride * 2};
            const cuuint32_t db[2] = {32, 16};
            if (!mvb::tc::encode(enc, &maps[(l * 4 + i) * 2], CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, w.qs, qd, qst, qb,
                                 CU_TENSOR_MAP_SWIZZLE_NONE) ||
                !mvb::tc::encode(enc, &maps[(l * 4 + i) * 2 + 1], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, w.d, dd, dst, db,
                                 CU_TENSOR_MAP_SWIZZLE_NONE))
                return skip("a weight's tensor map was rejected");
        }
    }
    int stages = 0;
    std::string why;
    if (!mvb::decode_mk_supported((int)m->hd, m->kv_type, (int)m->n_ctx, (int)m->n_pages, max_nb, m->n_embd, &stages,
                                  &why))
        return skip(why);
    m->mk_layers = dalloc<mvb::MkLayer>(m, m->n_layer);
    ck(cudaMemcpy(m->mk_layers, hl.data(), hl.size() * sizeof(mvb::MkLayer), cudaMemcpyHostToDevice), "layer table");
    m->mk_maps = dalloc<CUtensorMap>(m, maps.size());  // 256-byte aligned allocation (maps need 64)
    ck(cudaMemcpy(m->mk_maps, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice), "tensor maps");
    m->mk_bar = dalloc<unsigned>(m, 1);
    m->mk_status = dalloc<int>(m, 2);
    ck(cudaMemset(m->mk_status, 0, 8), "clear status");
    ck(cudaMallocHost(reinterpret_cast<void**>(&m->mk_status_host), sizeof(int)), "cudaMallocHost");
    *m->mk_status_host = 0;
    m->mk_stages = stages;
    m->mk = true;
}

void load_model(mv_model_s* m, const char* path, uint64_t ctx, uint64_t page, int kv_type, int rank = 0,
                int world = 1, uint64_t tp_bmax = 0) {
    mvb::GgufReader f(path);
    std::string arch;
    f.get_string("general.architecture", arch);
    if (arch != "llama")
        throw ModelError(MV_ERR_UNSUPPORTED, "MemVanta real-model path currently supports GGUF architecture=llama, got: " + arch);
    auto req = [&](const char* k) {
        uint64_t v;
        if (!f.get_u64(k, v)) throw ModelError(MV_ERR_IO, std::string("missing GGUF metadata: ") + k);
        return v;
    };
    m->n_ctx = req("llama.context_length");
    m->n_embd = req("llama.embedding_length");
    m->n_ff = req("llama.feed_forward_length");
    m->n_layer = req("llama.block_count");
    m->n_head = req("llama.attention.head_count");
    uint64_t kvh;
    m->n_head_kv = f.get_u64("llama.attention.head_count_kv", kvh) ? kvh : m->n_head;
    double dv;
    m->eps = f.get_f64("llama.attention.layer_norm_rms_epsilon", dv) ? (float)dv : 1e-5f;
    m->theta = f.get_f64("llama.rope.freq_base", dv) ? (float)dv : 10000.0f;
    const auto& te = f.tensor("token_embd.weight");
    m->vocab = te.ne(1);
    if (te.ne(0) != m->n_embd) throw ModelError(MV_ERR_INVALID, "token embedding shape mismatch");
    if (ctx) m->n_ctx = std::min(m->n_ctx, ctx);
    if (m->n_embd % m->n_head || !m->n_head_kv || m->n_head % m->n_head_kv)
        throw ModelError(MV_ERR_INVALID, "invalid Llama head configuration");
    m->hd = m->n_embd / m->n_head;
    m->kv_dim = m->n_head_kv * m->hd;
    if (m->hd != 64 && m->hd != 128 && m->hd != 256)
        throw ModelError(MV_ERR_UNSUPPORTED, "device attention supports head_dim 64, 128, 256");
    if (m->n_head / m->n_head_kv > 8) throw ModelError(MV_ERR_UNSUPPORTED, "GQA group above 8");
    if (kv_type < 0 || kv_type > 3) throw ModelError(MV_ERR_UNSUPPORTED, "unknown KV cache type");
    if (kv_type == MV_KV_Q8_0 && m->kv_dim % 32) throw ModelError(MV_ERR_INVALID, "Q8_0 KV needs kv_dim % 32 == 0");
    if (world > 1 && kv_type == MV_KV_Q8)
        throw ModelError(MV_ERR_UNSUPPORTED, "tensor parallelism splits the kv heads; the Q8 cache's per-token scale "
                                             "spans all of them (use F16, F32 or Q8_0)");
    m->kv_type = kv_type;
    m->page = page ? page : 128;
    m->n_pages = (m->n_ctx + m->page - 1) / m->page;
    // this rank's share (tensor parallel); the whole model on one rank
    if (world < 1 || world > mvb::kTpMaxWorld || rank < 0 || rank >= world)
        throw ModelError(MV_ERR_INVALID, "tensor-parallel rank/world out of range");
    if (m->n_head % world || m->n_head_kv % world || m->n_embd % world || m->n_ff % world || m->vocab % world)
        throw ModelError(MV_ERR_UNSUPPORTED, "tensor parallelism needs heads, kv heads, n_embd, n_ff and the vocab "
                                             "divisible by the number of GPUs");
    m->tp_rank = rank;
    m->tp_world = world;
    m->nh = m->n_head / world;
    m->nkv = m->n_head_kv / world;
    m->kvd = m->nkv * m->hd;
    m->qkvw = m->nh * m->hd + 2 * m->kvd;
    m->Dl = m->n_embd / world;
    m->Fl = m->n_ff / world;
    m->Vl = m->vocab / world;
    f.advise_sequential();
    Uploader up(m->stream);

    m->tok_embd = upload_tensor(m, up, f, te);
    const auto& on = f.tensor("output_norm.weight");
    m->output_norm = upload_vector(m, f, on, m->n_embd);
    const mvb::GgufTensorInfo* out = f.find("output.weight");
    if (world == 1) m->output = out ? upload_tensor(m, up, f, *out) : m->tok_embd;  // tied output (:226)
    else m->output = upload_rows(m, up, f, {{out ? out : &te, rank * m->Vl, m->Vl}}, false);

    const uint64_t rows = m->n_pages * m->page;
    const uint64_t rb = mvb::kv_row_bytes(kv_type, m->kvd), ns = mvb::kv_row_scales(kv_type, m->kvd);
    m->layers.resize(m->n_layer);
    for (uint64_t i = 0; i < m->n_layer; ++i) {
        auto name = [&](const char* s) { return "blk." + std::to_string(i) + s; };
        auto& L = m->layers[i];
        L.attn_norm = upload_vector(m, f, f.tensor(name(".attn_norm.weight")), m->n_embd);
        L.ffn_norm = upload_vector(m, f, f.tensor(name(".ffn_norm.weight")), m->n_embd);
        const auto &tq = f.tensor(name(".attn_q.weight")), &tk = f.tensor(name(".attn_k.weight")),
                   &tv = f.tensor(name(".attn_v.weight"));
        const auto &to = f.tensor(name(".attn_output.weight")), &tg = f.tensor(name(".ffn_gate.weight")),
                   &tu = f.tensor(name(".ffn_up.weight")), &td = f.tensor(name(".ffn_down.weight"));
        if (world == 1) {
            L.qkv = upload_concat(m, up, f, {&tq, &tk, &tv}, false);
            L.o = upload_tensor(m, up, f, to);
            L.gu = upload_concat(m, up, f, {&tg, &tu}, true);
            L.down = upload_tensor(m, up, f, td);
        } else {
            const uint64_t q0 = rank * m->nh * m->hd, k0 = rank * m->kvd;
            L.qkv = upload_rows(m, up, f, {{&tq, q0, m->nh * m->hd}, {&tk, k0, m->kvd}, {&tv, k0, m->kvd}}, false);
            L.o = upload_rows(m, up, f, {{&to, rank * m->Dl, m->Dl}}, false);
            L.gu = upload_rows(m, up, f, {{&tg, rank * m->Fl, m->Fl}, {&tu, rank * m->Fl, m->Fl}}, true);
            L.down = upload_rows(m, up, f, {{&td, rank * m->Dl, m->Dl}}, false);
            if (L.qkv->type != 2 || L.o->type != 2 || L.gu->type != 2 || L.down->type != 2)
                throw ModelError(MV_ERR_UNSUPPORTED, "tensor parallelism needs Q4_0 layer weights");
        }
        if (L.qkv->rows != m->qkvw) throw ModelError(MV_ERR_INVALID, "q/k/v shape mismatch");
        L.k_pages = dalloc<uint8_t>(m, rows * rb);
        L.v_pages = dalloc<uint8_t>(m, rows * rb);
        L.k_scales = ns ? dalloc<float>(m, rows * ns) : nullptr;
        L.v_scales = ns ? dalloc<float>(m, rows * ns) : nullptr;
    }
    // RoPE tables exactly as the reference builds them (src/llama_model.cpp:233)
    const uint64_t half = m->hd / 2;
    std::vector<float> co(m->n_ctx * half), si(m->n_ctx * half);
    for (uint64_t p = 0; p < m->n_ctx; ++p)
        for (uint64_t i = 0; i < half; ++i) {
            const float inv = std::pow(m->theta, -2.0f * float(i) / float(m->hd));
            const float a = float(p) * inv;
            co[p * half + i] = std::cos(a);
            si[p * half + i] = std::sin(a);
        }
    m->rope_cos = dalloc<float>(m, co.size());
    m->rope_sin = dalloc<float>(m, si.size());
    ck(cudaMemcpy(m->rope_cos, co.data(), co.size() * 4, cudaMemcpyHostToDevice), "rope cos");
    ck(cudaMemcpy(m->rope_sin, si.data(), si.size() * 4, cudaMemcpyHostToDevice), "rope sin");

    const uint64_t D = m->n_embd, F = m->n_ff;
    if (world > 1) {
        // the shared block every rank maps: flags, then the replicated buffers
        auto up = [](uint64_t b) { return (b + 255) / 256 * 256; };
        m->tp_bmax = tp_bmax ? tp_bmax : 64;
        uint64_t off = mvb::kTpFlagsBytes;
        m->off_x = off, off += up(D * 8);  // decode: LL buffers, 8 bytes per element
        m->off_att = off, off += up(D * 8);
        m->off_ff = off, off += up(F * 8);
        m->off_logits = off, off += up(m->vocab * 8);
        m->off_X = off, off += up(m->tp_bmax * D * 4);
        m->off_ATT = off, off += up(m->tp_bmax * D * 4);
        m->off_FF = off, off += up(m->tp_bmax * F * 4);
        m->tp_bytes = off;
        ck(cudaMalloc(reinterpret_cast<void**>(&m->tp_block), m->tp_bytes), "cudaMalloc(shared block)");
        ck(cudaMemset(m->tp_block, 0, m->tp_bytes), "clear shared block");
        m->x = dalloc<float>(m, D);  // the embedding, and the final x before the head
        m->att = dalloc<float>(m, D);
        m->ff = dalloc<float>(m, F);
        m->logits = dalloc<float>(m, m->vocab);
        m->logits_l = dalloc<float>(m, std::max(m->Vl, std::max(2 * m->Fl, D)));
        m->tp_step = dalloc<int>(m, 1);
        m->tp_counters = dalloc<unsigned>(m, 8);
        m->tp_status = dalloc<int>(m, 1);
        ck(cudaMemset(m->tp_step, 0, 4), "clear step");
        ck(cudaMemset(m->tp_counters, 0, 32), "clear counters");
        ck(cudaMemset(m->tp_status, 0, 4), "clear status");
        m->tp_limit = dalloc<long long>(m, 1);
        const long long lim = mvb::kTpDefaultLimitNs;
        ck(cudaMemcpy(m->tp_limit, &lim, 8, cudaMemcpyHostToDevice), "wait limit");
    } else {
        m->x = dalloc<float>(m, D);
        m->att = dalloc<float>(m, D);
        m->ff = dalloc<float>(m, F);
        m->logits = dalloc<float>(m, std::max(m->vocab, std::max(2 * F, D)));
    }
    m->qkv = dalloc<float>(m, m->qkvw);
    m->gu = dalloc<float>(m, 2 * m->Fl);
    m->nrm = dalloc<float>(m, D);
    m->token_dev = dalloc<int32_t>(m, 1);
    m->pos_dev = dalloc<int32_t>(m, 1);
    m->ctx_dev = dalloc<int32_t>(m, 1);
    m->history = dalloc<int32_t>(m, m->n_ctx + 1);
    ck(cudaMallocHost(reinterpret_cast<void**>(&m->logits_host), m->vocab * sizeof(float)), "cudaMallocHost");
    ensure_prefill(m, 1);  // identity block table
    {
        const char* env = std::getenv("MV_ATTN_SPLIT");
        m->attn_split = env && std::string(env) == "1";
        const bool fused = m->kv_type == MV_KV_F32 || m->kv_type == MV_KV_F16;
        const uint64_t need = fused ? mvb::attn_fused_split_smem_bytes(m->hd, m->n_pages, m->kv_type) : 0;
        if (fused && (need == 0 || need > 200 * 1024)) m->attn_split = false;
        const char* cenv = std::getenv("MV_ATTN_CLUSTER");
        const uint64_t cneed = fused ? mvb::attn_cluster_smem_bytes(m->hd, m->n_ctx, m->n_pages, m->kv_type) : 0;
        m->attn_cluster = cneed && cneed <= 110 * 1024 && !(cenv && std::string(cenv) == "0");
        // quantised hand-offs, opt-in: MV_DECODE_PREQUANT=1 (both), o, ff.  Measured
        // slower on the 7B step (683 tok/s without, 679 o only, 671 ff only, 661
        // both): the cluster barrier the attention adds and the 4-tile groups the
        // gate|up GEMV needs cost more than the copied prologue saves
        const char* qenv = std::getenv("MV_DECODE_PREQUANT");
        const std::string qv = qenv ? qenv : "0";
        const bool pq = world == 1 && qv != "0";
        bool o_ok = pq && qv != "ff" && fused && m->attn_cluster && !m->attn_split, f_ok = pq && qv != "o";
        for (const auto& L : m->layers) {
            o_ok = o_ok && mvb::gemv_q4_prequant_ok(*L.o);
            f_ok = f_ok && mvb::gemv_q4_prequant_ok(*L.gu) && mvb::gemv_q4_prequant_ok(*L.down) && L.gu->rows % 64 == 0;
        }
        if (o_ok) m->attq = dalloc<uint8_t>(m, mvb::q8_act_bytes(m->n_embd));
        if (f_ok) m->ffq = dalloc<uint8_t>(m, mvb::q8_act_bytes(m->n_ff));
    }
    if (world == 1) setup_persistent_decode(m);
    if (world == 1) ready_decode(m);  // tensor parallel: once the peers are connected
}

void free_model(mv_model_s* m) {
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->graph_logits) cudaGraphExecDestroy(m->graph_logits);
    if (m->graph_nologits) cudaGraphExecDestroy(m->graph_nologits);
    for (void* p : m->tp_opened) cudaIpcCloseMemHandle(p);
    if (m->tp_block) cudaFree(m->tp_block);
    if (m->tp_status_host) cudaFreeHost(m->tp_status_host);
    if (m->mk_status_host) cudaFreeHost(m->mk_status_host);
    for (auto* w : m->owned) mv_weight_free(w);
    for (void* p : m->allocs) cudaFree(p);
    if (m->logits_host) cudaFreeHost(m->logits_host);
    if (m->pf_host) cudaFreeHost(m->pf_host);
    if (m->pf_alt.stream) {
        cudaStreamSynchronize(m->pf_alt.stream);
        cudaStreamDestroy(m->pf_alt.stream);
    }
    for (auto& v : m->pf_ev)
        for (cudaEvent_t e : v) cudaEventDestroy(e);
    if (m->pf_join) cudaEventDestroy(m->pf_join);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

template <class Fn>
int guarded(Fn&& fn) {
    try {
        fn();
        return MV_OK;
    } catch (const ModelError& e) {
        g_model_err = e.what();
        return e.code;
    } catch (const std::exception& e) {
        g_model_err = e.what();
        return MV_ERR_IO;
    }
}

int model_fail(int rc) {
    mvb::set_last_error(g_model_err);  // surfaces through mv_last_error()
    return rc;
}

// Tensor parallel: calls need every rank connected; the status word a bounded
// wait sets is copied back with the call's results and checked after its sync.
void require_ready(const mv_model_s* m) {
    if (m->tp_world > 1 && !m->tp_ready)
        throw ModelError(MV_ERR_INVALID, "tensor-parallel model used before mv_model_tp_connect");
}
void enqueue_tp_status(mv_model_s* m) {
    if (m->tp_world > 1)
        ck(cudaMemcpyAsync(m->tp_status_host, m->tp_status, 4, cudaMemcpyDeviceToHost, m->stream), "status D2H");
    if (m->mk)
        ck(cudaMemcpyAsync(m->mk_status_host, m->mk_status, 4, cudaMemcpyDeviceToHost, m->stream), "status D2H");
}
void check_tp_status(const mv_model_s* m) {
    if (m->tp_world > 1 && *m->tp_status_host)
        throw ModelError(MV_ERR_TIMEOUT, "tensor-parallel wait for the other ranks gave up (site " +
                                             std::to_string(*m->tp_status_host) + ")");
    if (m->mk && *m->mk_status_host) {
        const int site = *m->mk_status_host;
        *m->mk_status_host = 0;
        cudaMemset(m->mk_status, 0, 8);  // the next step starts clean
        throw ModelError(MV_ERR_TIMEOUT, "persistent decode kernel gave up a bounded wait (site " +
                                             std::to_string(site) + ")");
    }
}

// Swaps the model's prefill buffers and stream with the alternate set (and
// back, on leaving the scope), so prefill_chunk runs a chunk on the other set.
struct AltSet {
    mv_model_s* m;
    bool on;
    AltSet(mv_model_s* m_, bool on_) : m(m_), on(on_) { flip(); }
    ~AltSet() { flip(); }
    void flip() {
        if (!on) return;
        auto& a = m->pf_alt;
        std::swap(m->X, a.X);
        std::swap(m->N, a.N);
        std::swap(m->QKV, a.QKV);
        std::swap(m->ATT, a.ATT);
        std::swap(m->GU, a.GU);
        std::swap(m->FF, a.FF);
        std::swap(m->PROJ, a.PROJ);
        std::swap(m->XQ, a.XQ);
        std::swap(m->XD, a.XD);
        std::swap(m->stream, a.stream);
    }
};

// Tokens one merged prefill batch holds at most.
constexpr uint64_t kMergedPrefill = 512;

// One decode step of every sequence of a set (mv_seqs_s): row i of the batch
// is sequence i's token at its own position, reading its own cache pages
// through row i of the set's block table.
struct SeqStep {
    const std::vector<mvb::Layer>* layers;  // the set's caches (weights shared)
    const int32_t* table;                   // device [n_seq][pages]
    uint64_t pages, max_ctx;
    float* logits;                          // device [n_seq][vocab]
};

// One chunk of B tokens; `off` indexes the call's staged inputs.  With `st`,
// the B rows are one decode token of each of B sequences instead (the
// reference's LlamaModel::forward per sequence): Q8 activations for every
// Q4_0 projection as tensor_matvec uses them, the decode attention over each
// row's own pages, and logits for every row.
void prefill_chunk(mv_model_s* m, uint64_t off, uint64_t B, bool logits_last, const SeqStep* st = nullptr) {
    cudaStream_t s = m->stream;
    const uint64_t D = m->n_embd, F = m->n_ff;
    const bool tp = m->tp_world > 1;
    const uint64_t start = m->pos;
    const int32_t* tok = m->pf_tok + off;
    const int32_t* pos = m->pf_pos + off;
    const int32_t* ctx = m->pf_ctx + off;
    // Q8 (tensor-core) projections: a chunk of 2+ tokens, or decode rows
    const bool q8 = B >= 2 || st;
    ck(mvb::read_rows(*m->tok_embd, tok, B, m->X, s), "embed");
    // Q8 activations when B >= 2 and the weight is Q4_0 (FORCE_Q8 path);
    // fp32 activations otherwise, as tensor_matmul_batch_v06 dispatches.
    // 64 tokens and more: fp16 activations and the fp16 tensor-core GEMM
    uint16_t* XH = mvb::gemm_f16_preferred(B) ? reinterpret_cast<uint16_t*>(m->XQ) : nullptr;
    auto gemm = [&](mv_weight_s* w, uint64_t ldb, float* out, bool accumulate) {
        if (XH) ck(mvb::gemm_q4_q8_f16(*w, XH, m->XD, ldb, B, out, s, accumulate), "gemm (fp16)");
        else ck(mvb::gemm_q4_q8_tc(*w, m->XQ, m->XD, ldb, B, out, s, accumulate), "gemm");
    };
    auto project = [&](mv_weight_s* w, const float* in, uint64_t K, float* out, bool accumulate) {
        if (q8 && w->type == 2) {
            const uint64_t ldb = mvb::gemm_tc_ldb(B);
            ck(mvb::quantize_q8_rows_t(in, B, K, m->XQ, m->XD, ldb, s, XH), "quantize");
            gemm(w, ldb, out, accumulate);
        } else if (accumulate) {
            ck(mvb::matmul_f32act(*w, in, B, m->PROJ, s), "matmul");
            ck(mvb::add_inplace(out, m->PROJ, B * w->rows, s), "add");
        } else {
            ck(mvb::matmul_f32act(*w, in, B, out, s), "matmul");
        }
    };
    // rmsnorm(X) as the input of a projection: fused into the quantisation on
    // the tensor-core path, materialised otherwise
    auto project_normed = [&](mv_weight_s* w, const float* norm_w, float* out) {
        if (q8 && w->type == 2) {
            const uint64_t ldb = mvb::gemm_tc_ldb(B);
            ck(mvb::rmsnorm_quantize_q8_rows_t(m->X, norm_w, B, D, m->eps, m->XQ, m->XD, ldb, s, XH),
               "rmsnorm+quantize");
            gemm(w, ldb, out, false);
        } else {
            ck(mvb::rmsnorm_rows(m->X, norm_w, B, D, m->eps, m->N, s), "rmsnorm");
            project(w, m->N, D, out, false);
        }
    };
    // tensor parallel: this rank's columns [col, col + w) of every row into
    // every rank's replicated buffer, then wait for the other ranks' columns
    auto exchange = [&](const float* src, uint64_t w, uint64_t dst_off, uint64_t dst_ld, uint64_t col, bool add,
                        int point) {
        ck(mvb::tp_scatter(m->tp, src, B, w, w, dst_off, dst_ld, col, add, point, point & 3, s), "scatter");
        ck(mvb::tp_wait(m->tp, point, s), "tp wait");
    };
    const std::vector<mvb::Layer>& layers = st ? *st->layers : m->kv_layers ? *m->kv_layers : m->layers;
    for (uint64_t l = 0; l < m->n_layer; ++l) {
        const auto& L = layers[l];
        project_normed(L.qkv, L.attn_norm, m->QKV);
        if (m->pf_wait) ck(cudaStreamWaitEvent(s, (*m->pf_wait)[l], 0), "wait (previous chunk's KV)");
        rope_append(m, L, m->QKV, B, pos, nullptr, m->pf_wait != nullptr, st ? st->table : nullptr,
                    st ? (int)st->pages : 0);
        if (m->pf_rec) ck(cudaEventRecord((*m->pf_rec)[l], s), "record (this chunk's KV)");
        mvb::AttnArgs aa = attn_args(m, L, m->QKV, m->qkvw, B, ctx, st ? st->max_ctx : start + B,
                                     tp ? m->ATT_l : m->ATT);
        // single GPU, tensor-core o projection: the attention kernel also
        // writes the o GEMM's Q8 input (no separate quantisation launch)
        const bool fuse_o = !tp && !st && B >= 2 && L.o->type == 2;
        if (st) {
            aa.block_table = st->table;
            aa.max_pages = st->pages;
            ck(m->attn_split ? mvb::paged_attn_decode_split(aa, s) : mvb::paged_attn_decode(aa, s), "attention");
        } else {
            aa.one_seq = 1;
            if (fuse_o) {
                aa.xq = m->XQ;
                aa.xdT = m->XD;
                aa.xq_ldb = mvb::gemm_tc_ldb(B);
                aa.xq_f16 = XH != nullptr;
            }
            ck(mvb::paged_attn_prefill(aa, s), "attention");
        }
        if (tp) {
            exchange(m->ATT_l, m->Dl, m->off_ATT, D, m->tp_rank * m->Dl, false, pt_att(l));
            project(L.o, m->ATT, D, m->PROJ_l, false);
            exchange(m->PROJ_l, m->Dl, m->off_X, D, m->tp_rank * m->Dl, true, pt_o(l));
        } else if (fuse_o) {
            gemm(L.o, mvb::gemm_tc_ldb(B), m->X, true);
        } else {
            project(L.o, m->ATT, D, m->X, true);
        }
        project_normed(L.gu, L.ffn_norm, m->GU);
        if (!tp && q8 && L.down->type == 2) {
            // SiLU gate fused into the down GEMM's Q8 quantisation
            const uint64_t ldb = mvb::gemm_tc_ldb(B);
            ck(mvb::silu_quantize_q8_rows_t(m->GU, B, F, m->XQ, m->XD, ldb, s, XH), "silu+quantize");
            gemm(L.down, ldb, m->X, true);
            continue;
        }
        float* ff = tp ? m->FF_l : m->FF;
        mvb::silu_pairs_kernel<<<mvb::ew_grid(B * m->Fl), 256, 0, s>>>(m->GU, ff, B * m->Fl);
        ck(cudaGetLastError(), "silu_pairs");
        if (tp) {
            exchange(m->FF_l, m->Fl, m->off_FF, F, m->tp_rank * m->Fl, false, pt_gu(l));
            project(L.down, m->FF, F, m->PROJ_l, false);
            exchange(m->PROJ_l, m->Dl, m->off_X, D, m->tp_rank * m->Dl, true, pt_down(l));
        } else {
            project(L.down, m->FF, F, m->X, true);
        }
    }
    if (st) {  // every row's logits: rmsnorm and the output projection over the batch
        project_normed(m->output, m->output_norm, st->logits);
        return;
    }
    m->pos += B;
    if (logits_last) {
        const float* last = m->X + (B - 1) * D;
        if (tp) {
            project_decode(m, m->output, last, m->output_norm, m->logits_l, mvb::Q4Epi::Store);
            ck(mvb::tp_scatter_ll(m->tp, m->logits_l, m->Vl, m->off_logits, m->tp_rank * m->Vl, pt_head(m), s),
               "scatter logits");
            ck(mvb::tp_unpack(m->tp, m->off_logits, m->vocab, m->logits, pt_head(m), s), "unpack logits");
        } else {
            project_decode(m, m->output, last, m->output_norm, m->logits, mvb::Q4Epi::Store);
        }
    }
    if (tp) ck(mvb::tp_step(m->tp_step, s), "tp step");
}

}  // namespace

extern "C" {

MV_API int mv_model_open(const char* path, uint64_t ctx, uint64_t page_tokens, int kv_type, mv_model_t* out) {
    if (!out || !path) return MV_ERR_INVALID;
    *out = nullptr;
    auto* m = new mv_model_s();
    int rc = guarded([&] {
        ck(cudaGetDevice(&m->device), "cudaGetDevice");
        ck(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking), "cudaStreamCreate");
        load_model(m, path, ctx, page_tokens, kv_type);
    });
    if (rc) {
        free_model(m);
        return model_fail(rc);
    }
    *out = m;
    return MV_OK;
}

MV_API int mv_model_open_tp(const char* path, uint64_t ctx, uint64_t page_tokens, int kv_type, int rank, int world,
                            uint64_t prefill_batch, mv_model_t* out) {
    if (!out || !path) return MV_ERR_INVALID;
    *out = nullptr;
    auto* m = new mv_model_s();
    int rc = guarded([&] {
        ck(cudaGetDevice(&m->device), "cudaGetDevice");
        ck(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking), "cudaStreamCreate");
        load_model(m, path, ctx, page_tokens, kv_type, rank, world, prefill_batch);
        if (world > 1)
            ck(cudaMallocHost(reinterpret_cast<void**>(&m->tp_status_host), sizeof(int)), "cudaMallocHost");
    });
    if (rc) {
        free_model(m);
        return model_fail(rc);
    }
    *out = m;
    return MV_OK;
}

MV_API int mv_model_tp_handle(mv_model_t m, void* handle_out) {
    if (!m || !handle_out || m->tp_world < 2) return MV_ERR_INVALID;
    int rc = guarded([&] {
        cudaIpcMemHandle_t h;
        ck(cudaIpcGetMemHandle(&h, m->tp_block), "cudaIpcGetMemHandle");
        std::memcpy(handle_out, &h, sizeof(h));
    });
    return rc ? model_fail(rc) : MV_OK;
}

MV_API int mv_model_tp_connect(mv_model_t m, const void* handles) {
    if (!m || !handles || m->tp_world < 2 || m->tp_ready) return MV_ERR_INVALID;
    int rc = guarded([&] {
        static_assert(sizeof(cudaIpcMemHandle_t) == MV_TP_HANDLE_BYTES, "IPC handle size");
        mvb::TpCtx t;
        t.world = m->tp_world;
        t.rank = m->tp_rank;
        for (int d = 0; d < m->tp_world; ++d) {
            if (d == m->tp_rank) {
                t.base[d] = m->tp_block;
                continue;
            }
            cudaIpcMemHandle_t h;
            std::memcpy(&h, static_cast<const char*>(handles) + d * sizeof(h), sizeof(h));
            void* p = nullptr;
            ck(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
            m->tp_opened.push_back(p);
            t.base[d] = static_cast<char*>(p);
        }
        t.step = m->tp_step;
        t.pps = points_per_step(m);
        t.counters = m->tp_counters;
        t.status = m->tp_status;
        t.limit_ns = m->tp_limit;
        m->tp = t;
        ready_decode(m);  // every rank together: the warm-up step exchanges
        enqueue_tp_status(m);
        ck(cudaStreamSynchronize(m->stream), "sync");
        check_tp_status(m);
    });
    return rc ? model_fail(rc) : MV_OK;
}

MV_API int mv_model_tp_disconnect(mv_model_t m) {
    if (!m || m->tp_world < 2) return MV_ERR_INVALID;
    int rc = guarded([&] {
        ck(cudaStreamSynchronize(m->stream), "sync");
        for (void* p : m->tp_opened) ck(cudaIpcCloseMemHandle(p), "cudaIpcCloseMemHandle");
        m->tp_opened.clear();
        m->tp_ready = false;
    });
    return rc ? model_fail(rc) : MV_OK;
}

MV_API int mv_model_tp_set_timeout(mv_model_t m, uint64_t ms) {
    if (!m || m->tp_world < 2 || ms == 0) return MV_ERR_INVALID;
    int rc = guarded([&] {
        const long long ns = (long long)std::min<uint64_t>(ms, 3600000) * 1000000ll;
        ck(cudaMemcpyAsync(m->tp_limit, &ns, 8, cudaMemcpyHostToDevice, m->stream), "wait limit");
        ck(cudaStreamSynchronize(m->stream), "sync");
    });
    return rc ? model_fail(rc) : MV_OK;
}

MV_API int mv_model_close(mv_model_t m) {
    if (m) free_model(m);
    return MV_OK;
}

MV_API int mv_model_config(mv_model_t m, uint64_t* o) {
    if (!m || !o) return MV_ERR_INVALID;
    o[0] = m->n_ctx;
    o[1] = m->n_embd;
    o[2] = m->n_ff;
    o[3] = m->n_layer;
    o[4] = m->n_head;
    o[5] = m->n_head_kv;
    o[6] = m->vocab;
    return MV_OK;
}

MV_API int mv_model_reset(mv_model_t m) {
    if (!m) return MV_ERR_INVALID;
    m->pos = 0;
    return MV_OK;
}

MV_API uint64_t mv_model_position(mv_model_t m) { return m ? m->pos : 0; }

MV_API uint64_t mv_model_kv_bytes(mv_model_t m) {
    // pages the current position has touched, as PagedKVCache allocates them
    if (!m) return 0;
    const uint64_t pages = (m->pos + m->page - 1) / m->page;
    const uint64_t per_row = mvb::kv_row_bytes(m->kv_type, m->kvd) +  // this rank's kv heads
                             4 * mvb::kv_row_scales(m->kv_type, m->kvd);
    return 2 * m->n_layer * pages * m->page * per_row;
}

MV_API void* mv_model_stream(mv_model_t m) { return m ? m->stream : nullptr; }

MV_API int mv_model_decode_persistent(mv_model_t m) { return m && m->mk ? 1 : 0; }

MV_API int mv_model_forward(mv_model_t m, int32_t token, int compute_logits, float* logits_host) {
    if (!m) return MV_ERR_INVALID;
    int rc = guarded([&] {
        if (token < 0 || (uint64_t)token >= m->vocab) throw ModelError(MV_ERR_INVALID, "token id out of range");
        if (m->pos >= m->n_ctx) throw ModelError(MV_ERR_INVALID, "context exhausted");
        require_ready(m);
        set_decode_inputs(m, token);
        ck(cudaGraphLaunch(compute_logits ? m->graph_logits : m->graph_nologits, m->stream), "graph launch");
        m->pos += 1;
        if (compute_logits) {
            ck(cudaMemcpyAsync(m->logits_host, m->logits, m->vocab * 4, cudaMemcpyDeviceToHost, m->stream), "logits D2H");
            enqueue_tp_status(m);
            ck(cudaStreamSynchronize(m->stream), "sync");
            check_tp_status(m);
            if (logits_host) std::memcpy(logits_host, m->logits_host, m->vocab * 4);
        }
    });
    return rc ? model_fail(rc) : MV_OK;
}

}  // extern "C"

namespace {

void prefill_impl(mv_model_t m, const int32_t* tokens, uint64_t n, uint64_t batch, int compute_logits,
                  float* logits_host) {
    {
        if (!tokens) throw ModelError(MV_ERR_INVALID, "null tokens");
        if (m->pos + n > m->n_ctx) throw ModelError(MV_ERR_INVALID, "context exhausted");
        for (uint64_t i = 0; i < n; ++i)
            if (tokens[i] < 0 || (uint64_t)tokens[i] >= m->vocab) throw ModelError(MV_ERR_INVALID, "token id out of range");
        require_ready(m);
        const uint64_t B0 = std::max<uint64_t>(1, batch);
        // The reference prefills in chunks of `batch` (LlamaModel::prefill,
        // src/llama_model.cpp:260), but every token's arithmetic is the same
        // whatever chunk it is in -- per-token Q8 activations, per-(token, row)
        // GEMM chains, the chunk's K/V appended before its causal attention --
        // except that a 1-token chunk takes the fp32-activation path
        // (tensor_matmul_batch_v06 routes batch < 2 to tensor_matmul_batch).
        // So the chunks of 2 or more tokens run together as one batch of up to
        // kMergedPrefill tokens (every weight read once per layer, not once per
        // chunk; tensor parallel: up to the prefill rows the shared buffers
        // hold); a last chunk of 1 token (n % batch == 1) runs on its own.
        // Outputs are identical to chunk-by-chunk execution.
        const char* env = std::getenv("MV_PREFILL_MERGE");
        const uint64_t cap = m->tp_world > 1 ? std::min<uint64_t>(kMergedPrefill, m->tp_bmax) : kMergedPrefill;
        const bool merge = B0 >= 2 && (m->tp_world == 1 || cap > B0) && !(env && std::string(env) == "0");
        const uint64_t tail1 = (B0 >= 2 && n % B0 == 1) ? 1 : 0;
        const uint64_t B = merge ? std::min<uint64_t>(std::max(B0, cap), n - tail1 ? n - tail1 : 1) : B0;
        ck(cudaStreamSynchronize(m->stream), "sync");
        ensure_prefill(m, std::min(B, n));
        stage_prefill_inputs(m, tokens, n);
        // single GPU, several chunks: odd chunks on the alternate buffers and
        // stream, one layer behind the chunk before them
        const bool wave = m->tp_world == 1 && m->pf_alt.stream && n > B;
        if (wave) {
            ck(cudaEventRecord(m->pf_join, m->stream), "record (prefill start)");
            ck(cudaStreamWaitEvent(m->pf_alt.stream, m->pf_join, 0), "wait (prefill start)");
        }
        try {
            uint64_t nb = 0;
            for (uint64_t i = 0, c = 0; i < n; i += nb, ++c) {
                nb = std::min(B, n - i);
                if (merge) {
                    // the merged span stops before the 1-token tail, which runs alone
                    const uint64_t q8_end = n - tail1;
                    nb = i < q8_end ? std::min(B, q8_end - i) : n - i;
                }
                m->pf_wait = wave && c ? &m->pf_ev[(c - 1) & 1] : nullptr;
                m->pf_rec = wave ? &m->pf_ev[c & 1] : nullptr;
                AltSet alt(m, wave && (c & 1));
                prefill_chunk(m, i, nb, compute_logits && i + nb == n);
            }
        } catch (...) {
            // an error part-way: nothing of this call may still run on the
            // alternate stream when the caller goes on (its next call restages
            // the inputs this call's chunks read)
            m->pf_wait = m->pf_rec = nullptr;
            if (wave) cudaStreamSynchronize(m->pf_alt.stream);
            throw;
        }
        m->pf_wait = m->pf_rec = nullptr;
        if (wave) {
            ck(cudaEventRecord(m->pf_join, m->pf_alt.stream), "record (prefill end)");
            ck(cudaStreamWaitEvent(m->stream, m->pf_join, 0), "wait (prefill end)");
        }
        if (compute_logits)
            ck(cudaMemcpyAsync(m->logits_host, m->logits, m->vocab * 4, cudaMemcpyDeviceToHost, m->stream), "logits D2H");
        enqueue_tp_status(m);
        ck(cudaStreamSynchronize(m->stream), "sync");
        check_tp_status(m);
        if (compute_logits && logits_host) std::memcpy(logits_host, m->logits_host, m->vocab * 4);
        int status = 0;
        ck(mvb::tc_status(m->stream, &status), "status");
        if (status)
            throw ModelError(MV_ERR_TIMEOUT, "prefill GEMM gave up a bounded wait (site " + std::to_string(status) + ")");
    }
}

}  // namespace

extern "C" {

MV_API int mv_model_prefill(mv_model_t m, const int32_t* tokens, uint64_t n, uint64_t batch, int compute_logits,
                            float* logits_host) {
    if (!m) return MV_ERR_INVALID;
    if (n == 0) return MV_OK;
    int rc = guarded([&] { prefill_impl(m, tokens, n, batch, compute_logits, logits_host); });
    return rc ? model_fail(rc) : MV_OK;
}

MV_API int mv_model_generate_greedy(mv_model_t m, int32_t token, uint64_t n, int32_t* out_tokens) {
    if (!m) return MV_ERR_INVALID;
    if (n == 0) return MV_OK;
    int rc = guarded([&] {
        if (!out_tokens) throw ModelError(MV_ERR_INVALID, "null output");
        if (token < 0 || (uint64_t)token >= m->vocab) throw ModelError(MV_ERR_INVALID, "token id out of range");
        if (m->pos + n > m->n_ctx) throw ModelError(MV_ERR_INVALID, "context exhausted");
        require_ready(m);
        const uint64_t start = m->pos;
        set_decode_inputs(m, token);
        for (uint64_t i = 0; i < n; ++i) ck(cudaGraphLaunch(m->graph_logits, m->stream), "graph launch");
        ck(cudaMemcpyAsync(out_tokens, m->history + start, n * 4, cudaMemcpyDeviceToHost, m->stream), "tokens D2H");
        enqueue_tp_status(m);
        ck(cudaStreamSynchronize(m->stream), "sync");
        m->pos += n;
        check_tp_status(m);
    });
    return rc ? model_fail(rc) : MV_OK;
}

}  // extern "C"

// ------------------------------------------------------- sequence sets
// Several sequences decoded together against one model's weights: each has
// its own paged KV cache (a run of pages of one pool per layer, placed in
// the pool in reverse sequence order so the block table is not the
// identity), filled by its own prefill, and every mv_model_forward_batch
// call advances all of them by one token as one batch -- the weights are
// read once per step for all sequences.  Row i of the step is sequence i's
// LlamaModel::forward (src/llama_model.cpp:253-257): the same per-token
// arithmetic as a single-sequence decode (Q8 activations and the per-row FMA
// chain for Q4_0, fp32 activations otherwise), the attention over its own
// pages through the block table (config 4's layout).
struct mv_seqs_s {
    mv_model_s* m = nullptr;
    uint64_t n_seq = 0, ctx = 0, pages = 0;       // pages per sequence
    std::vector<uint64_t> slot;                   // pool run of each sequence
    std::vector<std::vector<mvb::Layer>> views;   // [seq]: layers with that sequence's pages
    std::vector<mvb::Layer> pool;                 // layers with the pool's base
    std::vector<void*> allocs;
    int32_t* table = nullptr;                     // device [n_seq][pages]
    float* logits = nullptr;                      // device [n_seq][vocab]
    float* logits_host = nullptr;                 // pinned
    std::vector<uint64_t> pos;
    ~mv_seqs_s() {
        for (void* p : allocs) cudaFree(p);  // (synchronises with the device's work)
        if (logits_host) cudaFreeHost(logits_host);
    }
    template <class T>
    T* alloc(uint64_t count) {
        void* p = nullptr;
        ck(cudaMalloc(&p, count * sizeof(T) + 16), "cudaMalloc(sequence set)");
        allocs.push_back(p);
        return static_cast<T*>(p);
    }
};

namespace {

void seqs_open(mv_model_s* m, mv_seqs_s* S, uint64_t n_seq, uint64_t ctx) {
    if (m->tp_world != 1) throw ModelError(MV_ERR_UNSUPPORTED, "sequence sets run on one GPU");
    if (n_seq == 0 || n_seq > 4096) throw ModelError(MV_ERR_INVALID, "sequence count must be 1..4096");
    if (ctx == 0 || ctx > m->n_ctx) throw ModelError(MV_ERR_INVALID, "sequence context must be 1..the model's");
    S->m = m;
    S->n_seq = n_seq;
    S->ctx = ctx;
    S->pages = (ctx + m->page - 1) / m->page;
    S->pos.assign(n_seq, 0);
    S->slot.resize(n_seq);
    for (uint64_t i = 0; i < n_seq; ++i) S->slot[i] = n_seq - 1 - i;
    const uint64_t rows = n_seq * S->pages * m->page;
    const uint64_t rb = mvb::kv_row_bytes(m->kv_type, m->kvd), ns = mvb::kv_row_scales(m->kv_type, m->kvd);
    S->pool = m->layers;
    for (auto& L : S->pool) {
        L.k_pages = S->alloc<uint8_t>(rows * rb);
        L.v_pages = S->alloc<uint8_t>(rows * rb);
        L.k_scales = ns ? S->alloc<float>(rows * ns) : nullptr;
        L.v_scales = ns ? S->alloc<float>(rows * ns) : nullptr;
    }
    S->views.assign(n_seq, S->pool);
    std::vector<int32_t> t(n_seq * S->pages);
    for (uint64_t i = 0; i < n_seq; ++i) {
        const uint64_t first = S->slot[i] * S->pages;  // first page of the sequence's run
        for (auto& L : S->views[i]) {
            L.k_pages += first * m->page * rb;
            L.v_pages += first * m->page * rb;
            if (ns) {
                L.k_scales += first * m->page * ns;
                L.v_scales += first * m->page * ns;
            }
        }
        for (uint64_t j = 0; j < S->pages; ++j) t[i * S->pages + j] = (int32_t)(first + j);
    }
    S->table = S->alloc<int32_t>(t.size());
    ck(cudaMemcpy(S->table, t.data(), t.size() * 4, cudaMemcpyHostToDevice), "block table upload");
    S->logits = S->alloc<float>(n_seq * m->vocab);
    ck(cudaMallocHost(reinterpret_cast<void**>(&S->logits_host), n_seq * m->vocab * sizeof(float)),
       "cudaMallocHost(sequence set)");
}

void seqs_forward(mv_model_s* m, mv_seqs_s* S, const int32_t* tokens, float* logits_host) {
    if (!tokens) throw ModelError(MV_ERR_INVALID, "null tokens");
    const uint64_t n = S->n_seq;
    for (uint64_t i = 0; i < n; ++i) {
        if (tokens[i] < 0 || (uint64_t)tokens[i] >= m->vocab) throw ModelError(MV_ERR_INVALID, "token id out of range");
        if (S->pos[i] >= S->ctx) throw ModelError(MV_ERR_INVALID, "context exhausted (sequence " + std::to_string(i) + ")");
    }
    ck(cudaStreamSynchronize(m->stream), "sync");
    ensure_prefill(m, n);
    stage_prefill_inputs(m, tokens, n, S->pos.data());
    const SeqStep st{&S->pool, S->table, S->pages, S->ctx, S->logits};
    prefill_chunk(m, 0, n, false, &st);
    ck(cudaMemcpyAsync(S->logits_host, S->logits, n * m->vocab * 4, cudaMemcpyDeviceToHost, m->stream),
       "logits D2H");
    ck(cudaStreamSynchronize(m->stream), "sync");
    int status = 0;
    ck(mvb::tc_status(m->stream, &status), "status");
    if (status)
        throw ModelError(MV_ERR_TIMEOUT, "batched decode GEMM gave up a bounded wait (site " + std::to_string(status) + ")");
    for (auto& p : S->pos) ++p;
    if (logits_host) std::memcpy(logits_host, S->logits_host, n * m->vocab * 4);
}

}  // namespace

extern "C" {

MV_API int mv_model_seqs_open(mv_model_t m, uint64_t n_seq, uint64_t ctx, mv_seqs_t* out) {
    if (!m || !out) return MV_ERR_INVALID;
    *out = nullptr;
    auto* S = new mv_seqs_s();
    int rc = guarded([&] { seqs_open(m, S, n_seq, ctx); });
    if (rc) {
        delete S;
        return model_fail(rc);
    }
    *out = S;
    return MV_OK;
}

MV_API int mv_model_seqs_free(mv_seqs_t s) {
    delete s;
    return MV_OK;
}

MV_API int mv_model_seqs_prefill(mv_seqs_t s, uint64_t seq, const int32_t* tokens, uint64_t n, uint64_t batch,
                                 int compute_logits, float* logits_host) {
    if (!s || seq >= s->n_seq) return MV_ERR_INVALID;
    if (n == 0) return MV_OK;
    mv_model_s* m = s->m;
    int rc = guarded([&] {
        if (s->pos[seq] + n > s->ctx) throw ModelError(MV_ERR_INVALID, "context exhausted");
        // the model's prefill, pointed at this sequence's pages and position
        const uint64_t saved = m->pos;
        m->pos = s->pos[seq];
        m->kv_layers = &s->views[seq];
        try {
            prefill_impl(m, tokens, n, batch, compute_logits, logits_host);
        } catch (...) {
            m->kv_layers = nullptr;
            m->pos = saved;
            throw;
        }
        s->pos[seq] = m->pos;
        m->kv_layers = nullptr;
        m->pos = saved;
    });
    return rc ? model_fail(rc) : MV_OK;
}

MV_API int mv_model_seqs_position(mv_seqs_t s, uint64_t seq, uint64_t* pos) {
    if (!s || !pos || seq >= s->n_seq) return MV_ERR_INVALID;
    *pos = s->pos[seq];
    return MV_OK;
}

MV_API int mv_model_seqs_reset(mv_seqs_t s, uint64_t seq) {
    if (!s || seq >= s->n_seq) return MV_ERR_INVALID;
    s->pos[seq] = 0;
    return MV_OK;
}

MV_API int mv_model_forward_batch(mv_model_t m, mv_seqs_t s, const int32_t* tokens, float* logits_host) {
    if (!m || !s || s->m != m) return MV_ERR_INVALID;
    int rc = guarded([&] { seqs_forward(m, s, tokens, logits_host); });
    return rc ? model_fail(rc) : MV_OK;
}

}  // extern "C"
