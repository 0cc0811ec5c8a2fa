// kernels.cuh -- host-side launchers of every kernel, shared by the C ABI
// (capi.cu) and the device-resident model (model.cu).  All launchers are
// asynchronous on `s` and return cudaGetLastError() of the launch.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include "tp.cuh"
#include "weights.cuh"

#include <string>

namespace mvb {

int num_sms();
void set_last_error(const std::string& msg);  // capi.cu: the message mv_last_error() returns

// ---- weights.cu
cudaError_t repack_from_ggml(mv_weight_s& w, const uint8_t* raw_dev, cudaStream_t s);
cudaError_t unpack_to_ggml(const mv_weight_s& w, uint8_t* raw_dev, cudaStream_t s);
cudaError_t read_rows(const mv_weight_s& w, const int32_t* rows, uint64_t n, float* out, cudaStream_t s);
cudaError_t quantize_q8_rows(const float* x, uint64_t rows, uint64_t cols, int8_t* q, float* d, cudaStream_t s);
// for the tensor-core GEMM: scales block-major, dT[b * ldb + row], then at
// dT + nb * ldb the GEMM's per-block constants; 2 * nb * ldb floats in all,
// rows..ldb-1 zero-filled (ldb >= rows)
// (qh set: the values as fp16 into qh[rows][cols] instead of int8 into q)
cudaError_t quantize_q8_rows_t(const float* x, uint64_t rows, uint64_t cols, int8_t* q, float* dT, uint64_t ldb,
                               cudaStream_t s, uint16_t* qh = nullptr);
// the same on rmsnorm(x) * w (the reference's rmsnorm), without materialising it
cudaError_t rmsnorm_quantize_q8_rows_t(const float* x, const float* w, uint64_t rows, uint64_t cols, float eps,
                                       int8_t* q, float* dT, uint64_t ldb, cudaStream_t s, uint16_t* qh = nullptr);
// the same on ff = silu(g) * u of a gate|up output with interleaved (g, u)
// rows: gu is [rows][2 * cols], the quantised ff [rows][cols]
cudaError_t silu_quantize_q8_rows_t(const float* gu, uint64_t rows, uint64_t cols, int8_t* q, float* dT, uint64_t ldb,
                                    cudaStream_t s, uint16_t* qh = nullptr);

// ---- gemv_q4.cu : decode GEMV over Q4_0 with Q8 activations (integer path)
enum class Q4Pro : int {
    Plain = 0,     // activations = x
    RmsNorm = 1,   // activations = rmsnorm(x) * norm_w (the reference's rmsnorm)
    PreQuant = 2,  // x points to activations already quantised (q8_act_bytes layout)
};
// Quantised activations of K elements as the decode GEMV keeps them in shared
// memory, also written by the kernel before it so that the GEMV only copies
// them: per 32-element block b, int8 q[0..15] at 16*b, q[16..31] at
// 16*(nb + b), and (d, bits of float 8*sum q) as float2 at 32*nb + 8*b.
__host__ __device__ inline uint64_t q8_act_bytes(uint64_t K) {
    const uint64_t nb = K / 32;
    return nb * 32 + (nb + 1) / 2 * 16;
}
enum class Q4Epi : int {
    Store = 0,     // y[r] = acc
    AddTo = 1,     // y[r] += acc          (residual stream)
    SiluGate = 2,  // rows come in (gate,up) pairs: y[r/2] = silu(g) * u
};
struct GemvQ4Args {
    const mv_weight_s* w;
    const float* x;
    const float* norm_w;  // RmsNorm only
    float eps;
    float* y;
    Q4Pro pro;
    Q4Epi epi;
    // Tensor-parallel decode (tp.cuh, LL buffers).  x_ll set: the input is
    // this rank's copy of a replicated LL buffer, read once its elements carry
    // point x_point's epoch (x is ignored).  y == nullptr: the output is the
    // replicated LL buffer at byte offset y_shared of every rank's block; this
    // rank's rows land at y_row_off + row (SiluGate: y_row_off + row/2),
    // tagged with point y_point's epoch; AddTo reads the residual (this
    // rank's rows of the same buffer) once it carries res_point's epoch.
    const TpCtx* tp = nullptr;
    const void* x_ll = nullptr;
    int x_point = 0;
    uint64_t y_shared = 0;
    int y_row_off = 0;
    int y_point = 0;
    int res_point = 0;
    // CTA slots the launch leaves free for the kernel after it (the decode
    // attention after the q|k|v GEMV starts on them while this one runs)
    int reserve = 0;
    // SiluGate, one GPU: also write the outputs' Q8 blocks (q8_act_bytes
    // layout) for the next GEMV's PreQuant input
    void* yq = nullptr;
};
// Whether a one-GPU GEMV of this weight takes PreQuant input / writes yq.
bool gemv_q4_prequant_ok(const mv_weight_s& w);
cudaError_t gemv_q4(const GemvQ4Args& a, cudaStream_t s);
cudaError_t q4_block_dots(const mv_weight_s& w, const float* x, int32_t* isum, cudaStream_t s);

// ---- gemv_q8.cu : decode GEMV for Q8_0 weights (fp32 x, 16-byte aligned)
cudaError_t gemv_q8_0(const mv_weight_s& w, const float* x, float* y, cudaStream_t s);

// ---- gemv_q6k.cu : decode GEMV for the Q6_K output head (fp32 x)
cudaError_t gemv_q6k(const mv_weight_s& w, const float* x, float* y, cudaStream_t s);

// ---- matmul_f32.cu : fp32-activation matmul for every type (T tokens per pass)
cudaError_t matmul_f32act(const mv_weight_s& w, const float* x, uint64_t batch, float* y, cudaStream_t s);

// ---- gemm_tc.cu : batched Q4_0 x Q8 activations (prefill) on the tensor cores
// (tcgen05 int8 MMA, TMEM, TMA); y += result instead of y = result when accumulate
// q: [batch][cols] int8, dT: the 2 * nb * ldb floats of quantize_q8_rows_t
// with ldb = gemm_tc_ldb(batch).  Exactly the reference's FORCE_Q8 chain per
// output.
uint64_t gemm_tc_ldb(uint64_t batch);
cudaError_t gemm_q4_q8_tc(const mv_weight_s& w, const int8_t* q, const float* dT, uint64_t ldb, uint64_t batch,
                          float* y, cudaStream_t s, bool accumulate = false);
// synchronise s; *status = site code of an expired bounded wait (0 = none), cleared
cudaError_t tc_status(cudaStream_t s, int* status);
// ---- gemm_f16.cu : the same matmul on fp16 tensor-core operands (kind::f16),
// for batches of 64 tokens and more: qh [batch][cols] fp16 activations
// (quantize_q8_rows_t & co. with qh), dT the block-major scales (ldb as above)
cudaError_t gemm_q4_q8_f16(const mv_weight_s& w, const uint16_t* qh, const float* dT, uint64_t ldb, uint64_t batch,
                           float* y, cudaStream_t s, bool accumulate = false);
cudaError_t f16_status_take(int* status);
// The same for the decode GEMV's pair exchange and the cluster attention's
// exchanges (bounded waits on their receive barriers).
cudaError_t gemv_status_take(int* status);
cudaError_t attn_status_take(int* status);
// whether a Q8-activation matmul of `batch` tokens takes gemm_q4_q8_f16
// (64 tokens and more; MV_GEMM_F16=0 keeps the int8 kernel everywhere)
bool gemm_f16_preferred(uint64_t batch);
// Test hook: the next fp16 GEMM launch leaves out the MMA commit of stage
// skip_commit (-1: none) and bounds its waits by wait_ns (0: the default).
void gemm_f16_test_stall(int skip_commit, uint64_t wait_ns);

// ---- ops.cu
cudaError_t rmsnorm_rows(const float* x, const float* w, uint64_t rows, uint64_t n, float eps, float* out,
                         cudaStream_t s);
cudaError_t rope_rows(float* q, uint64_t n_head, float* k, uint64_t n_head_kv, uint64_t hd, uint64_t rows,
                      const float* cos_t, const float* sin_t, const int32_t* pos, cudaStream_t s);
cudaError_t silu_mul(const float* g, const float* u, float* out, uint64_t n, cudaStream_t s);
cudaError_t add_inplace(float* x, const float* y, uint64_t n, cudaStream_t s);
cudaError_t f32_to_f16_ref(const float* x, uint16_t* h, uint64_t n, cudaStream_t s);
cudaError_t argmax_f32(const float* x, uint64_t n, int32_t* out_idx, cudaStream_t s);

// ---- attention.cu
uint64_t kv_row_bytes(int kv_type, uint64_t kv_dim);
uint64_t kv_row_scales(int kv_type, uint64_t kv_dim);
cudaError_t kv_append(int kv_type, const float* k, const float* v, uint64_t rows, uint64_t kv_dim,
                      const int32_t* seq, const int32_t* pos, const int32_t* block_table, uint64_t max_pages,
                      uint64_t page, void* k_pages, void* v_pages, float* k_scales, float* v_scales,
                      cudaStream_t s);
struct AttnArgs {
    int kv_type;
    const float* q;          // query row s at q + s * q_stride
    uint64_t q_stride;
    uint64_t n_seq, n_head, n_head_kv, hd;
    const void* k_pages;
    const void* v_pages;
    const float* k_scales;
    const float* v_scales;
    const int32_t* block_table;
    uint64_t max_pages, page;
    const int32_t* ctx_len;  // per query row
    uint64_t max_ctx;        // upper bound of ctx_len (sizes shared memory)
    float* out;              // [n_seq][n_head*hd]
    int one_seq = 0;         // 1: every query row reads block-table row 0 (rows of one sequence)
    // paged_attn_prefill only: when xq is set, the output rows are also
    // quantised for the tensor-core GEMM (quantize_q8_rows_t's layout, ldb)
    int8_t* xq = nullptr;
    float* xdT = nullptr;
    uint64_t xq_ldb = 0;
    bool xq_f16 = false;  // xq holds fp16 values of the Q8 integers (the fp16 GEMM's input)
};
uint64_t attn_smem_bytes(uint64_t hd, uint64_t max_ctx, uint64_t max_pages, int kv_type);
cudaError_t paged_attn_decode(const AttnArgs& a, cudaStream_t s);
// attn_split.cu: the same, split over the context (warps merge their softmax
// states); not bit-exact (~1e-6 of the output scale), for throughput
cudaError_t paged_attn_decode_split(const AttnArgs& a, cudaStream_t s);
// Prefill form: the query rows belong to ONE sequence (a.one_seq, or every
// row's block-table row is the same), so groups of them share each staged K/V
// tile; results identical to paged_attn_decode.
cudaError_t paged_attn_prefill(const AttnArgs& a, cudaStream_t s);

// One decode token (F32 or F16 KV): RoPE + KV append + attention in one kernel.
struct AttnFusedArgs {
    int kv_type;                     // 0 F32, 1 F16
    const float* qkv;                // this token's q heads | k heads | v heads (fp32, before RoPE)
    uint64_t n_head, n_head_kv, hd;
    const float* cos_t;              // [n_ctx][hd/2]
    const float* sin_t;
    const int32_t* pos;              // device: this token's position (tokens 0..pos-1 are cached)
    const int32_t* block_table;      // [max_pages] page of every logical page
    uint64_t max_pages, page, max_ctx;
    void* k_pages;
    void* v_pages;
    int32_t* ctx_out;                // optional: receives pos + 1
    float* out;                      // [n_head][hd]
    // tensor parallel: out is the replicated LL buffer at byte offset
    // out_shared of every rank's block; this rank's heads start at head
    // head_off; elements are tagged with point out_point's epoch
    TpCtx tp;
    uint64_t out_shared = 0;
    int head_off = 0;
    int out_point = 0;
    // one GPU: also write the output's Q8 blocks (q8_act_bytes layout) for
    // the o projection's PreQuant input (attn_decode_cluster only)
    void* xq = nullptr;
};
// ---- tp.cu (tensor parallel, protocol in tp.cuh)
cudaError_t tp_wait(const TpCtx& tp, int point, cudaStream_t s);
cudaError_t tp_scatter(const TpCtx& tp, const float* src, uint64_t rows, uint64_t w, uint64_t src_ld,
                       uint64_t dst_shared, uint64_t dst_ld, uint64_t col_off, bool add, int point, int slot,
                       cudaStream_t s);
cudaError_t tp_step(int* step, cudaStream_t s);
// LL buffers (decode): this rank's float vector into its own copy; an own
// copy into a float vector once every element carries the point's epoch;
// a float slice into every rank's copy at element col_off.
cudaError_t tp_pack(const TpCtx& tp, const float* src, uint64_t n, uint64_t dst_shared, int point, cudaStream_t s);
cudaError_t tp_unpack(const TpCtx& tp, uint64_t src_shared, uint64_t n, float* dst, int point, cudaStream_t s);
cudaError_t tp_scatter_ll(const TpCtx& tp, const float* src, uint64_t n, uint64_t dst_shared, uint64_t col_off,
                          int point, cudaStream_t s);

uint64_t attn_fused_smem_bytes(uint64_t hd, uint64_t max_ctx, uint64_t max_pages, int kv_type);
cudaError_t attn_decode_fused(const AttnFusedArgs& a, cudaStream_t s);
// The same step with the attention split over the context (attn_split.cu):
// a cluster of CTAs per head, partial softmax states merged in a fixed order
// (outputs within ~1e-6 of the exact kernel; cache rows identical).
// attn_fused_split_smem_bytes is 0 for an unsupported kv type / head size.
uint64_t attn_fused_split_smem_bytes(uint64_t hd, uint64_t max_pages, int kv_type);
// The same step in the reference's order over a cluster of CTAs per head
// (attn_cluster.cu); attn_cluster_smem_bytes is 0 when unsupported.
uint64_t attn_cluster_smem_bytes(uint64_t hd, uint64_t max_ctx, uint64_t max_pages, int kv_type);
cudaError_t attn_decode_cluster(const AttnFusedArgs& a, cudaStream_t s);
cudaError_t attn_decode_fused_split(const AttnFusedArgs& a, cudaStream_t s);

// ---- decode_mk.cu : every layer of one decode step as one persistent
// (cooperative) kernel, one CTA per SM; one GPU, Q4_0 layer weights, F32/F16 KV
struct MkGemv {                 // one Q4_0 weight in the planar layout (weights.cuh)
    const uint8_t* qs;
    const uint16_t* d;
    int rows, nb, dstride;
};
struct MkLayer {
    MkGemv w[4];                // q|k|v, o, gate|up (rows interleaved), down
    const float* attn_norm;
    const float* ffn_norm;
    uint8_t* k_pages;
    uint8_t* v_pages;
};
struct MkArgs {
    const MkLayer* layers;      // device array [n_layer]
    // device array [n_layer][4][2]: per layer weight (q|k|v, o, gate|up, down)
    // the TMA maps of its nibble plane (uint32 words, box 128 x 16 rows) and
    // its scale plane (fp16, box 32 x 16 rows)
    const CUtensorMap* maps;
    int n_layer, n_head, n_head_kv, hd, kv_type, page, max_ctx, max_pages;
    float eps;
    float* x;                   // [n_embd] residual stream: the embedding in, the last layer's out
    float* qkv;                 // [(n_head + 2 n_head_kv) hd]
    float* att;                 // [n_embd]
    float* ff;                  // [n_ff]
    const float* cos_t;         // RoPE tables [n_ctx][hd/2]
    const float* sin_t;
    const int32_t* pos;         // device: this token's position
    const int32_t* block_table; // [max_pages]
    int32_t* ctx_out;           // optional: receives pos + 1
    unsigned* bar;              // grid-barrier counter (device word, zeroed by the launcher)
    int* status;                // [0] site of an expired bounded wait (0: none), [1] abort word
    int stages;                 // weight ring stages (decode_mk_supported)
};
// Whether this shape runs on the persistent kernel; *stages = ring depth
// that fits the device's shared memory.
bool decode_mk_supported(int hd, int kv_type, int max_ctx, int max_pages, uint64_t max_nb, uint64_t norm_cols,
                         int* stages, std::string* why = nullptr);
cudaError_t decode_mk(const MkArgs& a, cudaStream_t s);

}  // namespace mvb
