/*
 * memvanta_b200.h -- C ABI of the B200 (sm_100a) implementation of
 * MemVanta's GGUF block-quantized matmul hot path.
 *
 * Conventions
 *  - Every function returns an int status: MV_OK (0) or one of the MV_ERR_*
 *    codes below; mv_last_error() then returns a thread-local message.  No
 *    C++ exception ever crosses this boundary (the reference throws
 *    std::runtime_error at the same points; a C++ caller re-throws).
 *  - Pointers named *_dev are device (HBM) pointers; *_host are host
 *    pointers.  `stream` is a cudaStream_t passed as void* (NULL = legacy
 *    default stream).  Device-pointer calls are asynchronous on `stream`.
 *  - Matrices follow GGML order: a weight has `cols` = ne0 (the contraction
 *    dimension K) and `rows` = ne1.  Batched activations are x[b*cols + c],
 *    outputs y[b*rows + r] (the reference's layout, src/gguf_kernels.cpp:257).
 *  - GGML type ids: 0 F32, 1 F16, 2 Q4_0, 8 Q8_0, 14 Q6_K.
 *
 * Reference citations are path:line inside the MemVanta project.
 */
#ifndef MEMVANTA_B200_H
#define MEMVANTA_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MV_API __attribute__((visibility("default")))
#else
#define MV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define MV_OK 0
#define MV_ERR_INVALID 1      /* bad argument / shape (reference: runtime_error) */
#define MV_ERR_UNSUPPORTED 2  /* unsupported tensor type for this operation     */
#define MV_ERR_CUDA 3         /* a CUDA runtime error                            */
#define MV_ERR_OOM 4          /* device allocation failed                        */
#define MV_ERR_IO 5           /* GGUF file could not be read / parsed            */
#define MV_ERR_TIMEOUT 6      /* a bounded device-side wait ran out              */
#define MV_ERR_NOT_BUILT 7    /* feature not available in this build             */

#define MV_TYPE_F32 0
#define MV_TYPE_F16 1
#define MV_TYPE_Q4_0 2
#define MV_TYPE_Q8_0 8
#define MV_TYPE_Q6_K 14

/* activation modes for mv_gemm (tensor_matmul_batch_v06) */
#define MV_ACT_F32 0  /* fp32 activations: the reference's default prefill (src/gguf_kernels.cpp:268)            */
#define MV_ACT_Q8 1   /* per-row Q8 activations: MEMVANTA_FORCE_Q8_ACT=1 (src/gguf_kernels.cpp:265-266)           */

/* KV cache element types (reference KVCacheType, include/memvanta/llama_model.hpp:28) */
#define MV_KV_F32 0
#define MV_KV_F16 1
#define MV_KV_Q8 2    /* one fp32 scale per token over kv_dim (src/llama_model.cpp:22)                            */
#define MV_KV_Q8_0 3  /* one fp32 scale per 32-element block (extension; no reference counterpart)               */

typedef struct mv_weight_s* mv_weight_t;
typedef struct mv_model_s* mv_model_t;
typedef struct mv_seqs_s* mv_seqs_t;

/* ------------------------------------------------------------ runtime */

/* Selects the CUDA device for this thread and checks it is an sm_100 part.
 * Replaces nothing in the reference (CPU-only); called once by the host. */
MV_API int mv_init(int device);
MV_API const char* mv_last_error(void);
MV_API int mv_version(void);
/* Architecture of the device code the library loaded on the current device,
 * as cudaFuncGetAttributes' binaryVersion (100 = sm_100).  No counterpart in
 * the reference; lets a caller or a test check the build at run time. */
MV_API int mv_binary_arch(int* out);
/* Synchronises `stream` and reports MV_ERR_TIMEOUT if a kernel with bounded
 * device-side waits (the tensor-core GEMMs of mv_gemm with MV_ACT_Q8 and of
 * the model's prefill, the decode GEMV's and the cluster attention's
 * exchanges between CTAs) gave up a wait since the last check -- its outputs
 * are then invalid.  Host-pointer calls and the model's prefill check this
 * themselves.  No counterpart in the reference. */
MV_API int mv_stream_status(void* stream);
/* Test hook for the bounded waits (no counterpart in the reference): the
 * next fp16 tensor-core GEMM launch (mv_gemm, MV_ACT_Q8, batch >= 64) leaves
 * out the MMA commit of its pipeline stage `skip_commit_stage` (-1: none) and
 * bounds each of its mbarrier waits by wait_limit_us (0: the default 2 s).
 * A wait then runs out; the kernel drains its copies and MMAs, frees its
 * tensor memory and returns, and mv_stream_status reports MV_ERR_TIMEOUT.
 * Applies to one launch; later launches are unaffected. */
MV_API int mv_test_gemm_stall(int skip_commit_stage, uint64_t wait_limit_us);

/* ------------------------------------------------------------ weights */

/* Uploads one GGUF tensor (raw GGML blocks as they sit in the mmap) to HBM
 * and repacks it into the planar device layout.  Called once per tensor at
 * load time; replaces the reference's per-call reads of block bytes through
 * GgufFile::tensor_data (src/gguf.cpp:139) in tensor_matvec & co.
 * nbytes must equal ggml_tensor_nbytes(type, rows*cols) (src/gguf.cpp:82-105). */
MV_API int mv_weight_upload(const void* host_blocks, uint64_t nbytes, int ggml_type, uint64_t rows, uint64_t cols,
                     void* stream, mv_weight_t* out);
/* Same, from raw GGML blocks already in device memory. */
MV_API int mv_weight_from_device(const void* dev_blocks, uint64_t nbytes, int ggml_type, uint64_t rows, uint64_t cols,
                          void* stream, mv_weight_t* out);
MV_API int mv_weight_free(mv_weight_t w);
MV_API int mv_weight_info(mv_weight_t w, int* ggml_type, uint64_t* rows, uint64_t* cols, uint64_t* device_bytes);
/* Writes the weight back out as raw GGML blocks (host) -- the inverse of the
 * upload repack, used to prove the repack lossless. */
MV_API int mv_weight_download(mv_weight_t w, void* host_blocks, uint64_t nbytes);

/* --------------------------------------------------- matmuls (device ptrs) */

/* y[rows] = W x.  Q4_0 quantises x to Q8 per 32-block and runs the integer
 * path; Q8_0, Q6_K, F16, F32 use fp32 x.
 * Replaces tensor_matvec (src/gguf_kernels.cpp:244-253, declared
 * include/memvanta/gguf_kernels.hpp:26). */
MV_API int mv_gemv(mv_weight_t w, const float* x_dev, float* y_dev, void* stream);

/* Y[batch,rows] = X[batch,cols] W^T.  act_mode MV_ACT_Q8 is the reference's
 * MEMVANTA_FORCE_Q8_ACT=1 path (Q4_0 rows with Q8 activations, batch >= 2, on
 * the tensor cores, bit-exact with the reference; Q8_0 keeps fp32
 * activations); MV_ACT_F32 is its default fp32-activation path.  Q6_K, F16
 * and F32 always take fp32 activations, as tensor_matmul_batch does.
 * Replaces tensor_matmul_batch_v06 (src/gguf_kernels.cpp:261-271,
 * include/memvanta/gguf_kernels.hpp:30) and tensor_matmul_batch (:255-259). */
MV_API int mv_gemm(mv_weight_t w, const float* x_dev, uint64_t batch, float* y_dev, int act_mode, void* stream);

/* mv_gemm(w, x, batch, y, MV_ACT_Q8, stream) for a Q4_0 weight, with the
 * same result, for callers that must not allocate device memory while they
 * run (a framework whose own pool owns all GPU memory, a fixed memory budget,
 * a latency-critical loop).  No counterpart in the reference.  The quantised
 * activations go to one 8 MiB array compiled into the library, held on every
 * GPU that loads it until the process exits, so round_up(batch * cols, 256)
 * bytes of int8 values plus (cols / 32) * round_up(batch, 64) * 8 bytes of
 * scales and GEMM constants must fit in 8 MiB (larger calls return
 * MV_ERR_INVALID).  The first call on a device looks the array's address up
 * (cudaGetSymbolAddress) and keeps it for the process: make that call before
 * any stream capture, and do not reset the device (cudaDeviceReset) after it.
 * Calls that overlap on the GPU share the array and race; the caller
 * serialises them.  Allocates nothing, frees nothing. */
MV_API int mv_gemm_q8_noalloc(mv_weight_t w, const float* x_dev, uint64_t batch, float* y_dev, void* stream);

/* Per-row Q8 activation quantisation: q[rows*cols] int8, d[rows*cols/32] fp32.
 * Replaces quantize_q8 / quantize_activations_q8
 * (src/gguf_kernels.cpp:161-178). */
MV_API int mv_quantize_q8(const float* x_dev, uint64_t rows, uint64_t cols, int8_t* q_dev, float* d_dev, void* stream);

/* Diagnostic: the int32 dot of every Q4_0 block of W with the Q8-quantised x,
 * isum[rows*(cols/32)], computed by the same device code as mv_gemv.
 * Counterpart of dot_q4_q8_block (src/gguf_kernels.cpp:180-188). */
MV_API int mv_q4_0_block_dots(mv_weight_t w, const float* x_dev, int32_t* isum_dev, void* stream);

/* Dequantised row (embedding lookup): out[cols] = W[row,:].
 * Replaces tensor_read_row_f32 (src/gguf_kernels.cpp:226). */
MV_API int mv_read_row(mv_weight_t w, uint64_t row, float* out_dev, void* stream);
/* Same for `n` rows given by a device array of token ids (out[n*cols]). */
MV_API int mv_read_rows(mv_weight_t w, const int32_t* rows_dev, uint64_t n, float* out_dev, void* stream);

/* --------------------------------------------------- ops (device ptrs) */

/* out = x * (1/sqrt(mean(x^2)+eps)) * w per row of n; sum of squares in
 * double.  Replaces LlamaModel::rmsnorm / rms_batch (src/llama_model.cpp:237,
 * :245). */
MV_API int mv_rmsnorm(const float* x_dev, const float* w_dev, uint64_t rows, uint64_t n, float eps, float* out_dev,
               void* stream);
/* Half-split RoPE in place for `rows` tokens: q[rows, n_head*hd],
 * k[rows, n_head_kv*hd]; token r rotates with row pos[r] of the host-built
 * cos/sin tables [n_ctx, hd/2].  Replaces LlamaModel::rope_ptr
 * (src/llama_model.cpp:238). */
MV_API int mv_rope(float* q_dev, uint64_t n_head, float* k_dev, uint64_t n_head_kv, uint64_t head_dim, uint64_t rows,
            const float* cos_dev, const float* sin_dev, const int32_t* pos_dev, void* stream);
/* out = g/(1+exp(-g)) * u.  src/llama_model.cpp:249, :257. */
MV_API int mv_silu_mul(const float* g_dev, const float* u_dev, float* out_dev, uint64_t n, void* stream);
/* x += y.  src/llama_model.cpp:249, :257. */
MV_API int mv_add_inplace(float* x_dev, const float* y_dev, uint64_t n, void* stream);
/* h = fp32_to_fp16(x) with the reference's rounding (src/gguf_kernels.cpp:242). */
MV_API int mv_fp32_to_fp16(const float* x_dev, uint16_t* h_dev, uint64_t n, void* stream);

/* ------------------------------------------------ paged KV cache (device) */

/* Bytes of one cached token row of kv_dim elements and fp32 scales per row. */
MV_API uint64_t mv_kv_row_bytes(int kv_type, uint64_t kv_dim);
MV_API uint64_t mv_kv_row_scales(int kv_type, uint64_t kv_dim);

/* Writes `rows` tokens of k/v [rows, kv_dim] into the paged cache.  Token r
 * goes to position pos[r] of sequence seq[r] (seq_dev may be NULL: all 0):
 * page block_table[seq*max_pages + pos/page] slot pos%page.  k_pages /
 * v_pages hold n_pages*page rows of mv_kv_row_bytes each; k_scales /
 * v_scales (Q8 types only) n_pages*page*mv_kv_row_scales floats.
 * Replaces PagedKVCache::write (src/llama_model.cpp:22). */
MV_API int mv_kv_append(int kv_type, const float* k_dev, const float* v_dev, uint64_t rows, uint64_t kv_dim,
                 const int32_t* seq_dev, const int32_t* pos_dev, const int32_t* block_table_dev,
                 uint64_t max_pages, uint64_t page, void* k_pages_dev, void* v_pages_dev, float* k_scales_dev,
                 float* v_scales_dev, void* stream);

/* One-query attention for n_seq sequences over a paged cache:
 * q[n_seq, n_head*hd] -> out[n_seq, n_head*hd]; sequence s attends to
 * ctx_len[s] tokens whose pages are block_table[s*max_pages + i].  Per head:
 * softmax(q.k/sqrt(hd)) . v, GQA kv head h/(n_head/n_head_kv).  Split over
 * the context in the reference's order (the per-dimension FMA chain runs over
 * the tokens in sequence): the scores are bit-identical, the output differs
 * from the reference only where the device's correctly rounded exp and tree
 * summed double denominator round differently from the host's expf.
 * Replaces the decode attention loop over PagedKVCache::dot_key/add_value
 * (src/llama_model.cpp:23-55, :256). */
MV_API int mv_paged_attn_decode(int kv_type, const float* q_dev, uint64_t n_seq, uint64_t n_head, uint64_t n_head_kv,
                         uint64_t head_dim, const void* k_pages_dev, const void* v_pages_dev,
                         const float* k_scales_dev, const float* v_scales_dev, const int32_t* block_table_dev,
                         uint64_t max_pages, uint64_t page, const int32_t* ctx_len_dev, uint64_t max_ctx,
                         float* out_dev, void* stream);

/* mv_paged_attn_decode split over the context (split-K): each of four warps
 * per (sequence, head) owns a quarter of the tokens with its own running max,
 * double denominator and partial output, merged once in a fixed order.  Scores
 * are the reference's; the output agrees with it to ~1e-6 of its scale (not
 * bit for bit) at a fraction of the exact path's latency for long contexts.
 * Same arguments; Q8 caches need k_scales/v_scales.  Replaces the same
 * reference loop (src/llama_model.cpp:256). */
MV_API int mv_paged_attn_decode_split(int kv_type, const float* q_dev, uint64_t n_seq, uint64_t n_head,
                                      uint64_t n_head_kv, uint64_t head_dim, const void* k_pages_dev,
                                      const void* v_pages_dev, const float* k_scales_dev, const float* v_scales_dev,
                                      const int32_t* block_table_dev, uint64_t max_pages, uint64_t page,
                                      const int32_t* ctx_len_dev, uint64_t max_ctx, float* out_dev, void* stream);

/* Attention for n_q query rows of ONE sequence (a prefill chunk): every row
 * reads the pages of block_table[0 .. max_pages); row i attends to its first
 * ctx_len[i] tokens (causal: ctx_len[i] = start + i + 1).  Outputs identical
 * to mv_paged_attn_decode given a block table that repeats that row; groups
 * of query rows share each staged K/V tile.
 * Replaces the batched attention loop of LlamaModel::forward_batch_impl
 * (src/llama_model.cpp:248) over PagedKVCache::dot_key/add_value (:23-55). */
MV_API int mv_paged_attn_prefill(int kv_type, const float* q_dev, uint64_t n_q, uint64_t n_head, uint64_t n_head_kv,
                          uint64_t head_dim, const void* k_pages_dev, const void* v_pages_dev,
                          const float* k_scales_dev, const float* v_scales_dev, const int32_t* block_table_dev,
                          uint64_t max_pages, uint64_t page, const int32_t* ctx_len_dev, uint64_t max_ctx,
                          float* out_dev, void* stream);

/* ---------------------------------- host-pointer calls (reference contract) */

/* tensor_matvec with the reference's contract: x and y are HOST pointers,
 * y fully overwritten, synchronous.  src/gguf_kernels.cpp:244-253. */
MV_API int mv_tensor_matvec_host(mv_weight_t w, const float* x_host, float* y_host);
/* tensor_matmul_batch_v06 with host pointers.  src/gguf_kernels.cpp:261-271. */
MV_API int mv_tensor_matmul_batch_host(mv_weight_t w, const float* x_host, float* y_host, uint64_t batch, int act_mode);
/* tensor_read_row_f32 with a host output.  src/gguf_kernels.cpp:226. */
MV_API int mv_tensor_read_row_host(mv_weight_t w, uint64_t row, float* out_host);

/* ------------------------------------------------ internal block formats */

/* Device twins of the reference's internal-format kernels (the non-GGUF blocks
 * of include/memvanta/quant.hpp:8-13: BlockQ8_0 = 36 bytes {float d; int8
 * qs[32]}, BlockQ4_0 = 20 bytes {float d; uint8 qs[16]} with interleaved
 * nibbles), read in place from device memory with the reference's rounding
 * order (bit-identical outputs).  All pointers are device pointers, 4-byte
 * aligned (fp32 x 16-byte aligned); cols % 32 == 0; asynchronous on `stream`. */
/* quantize_q8_0 / quantize_q4_0, src/quant.cpp:44-85 (n % 32 == 0). */
MV_API int mv_int_quantize_q8_0(const float* x_dev, uint64_t n, void* out36_dev, void* stream);
MV_API int mv_int_quantize_q4_0(const float* x_dev, uint64_t n, void* out20_dev, void* stream);
/* matvec_q4_q8 (src/quant_kernels.cpp:68-80): y = A20 . x36. */
MV_API int mv_int_matvec_q4_q8(const void* A20_dev, const void* x36_dev, float* y_dev, uint64_t rows, uint64_t cols,
                               void* stream);
/* matvec_q4_0 / matvec_q8_0 against fp32 x (src/quant.cpp:158-174). */
MV_API int mv_int_matvec_q4_0(const void* A20_dev, const float* x_dev, float* y_dev, uint64_t rows, uint64_t cols,
                              void* stream);
MV_API int mv_int_matvec_q8_0(const void* A36_dev, const float* x_dev, float* y_dev, uint64_t rows, uint64_t cols,
                              void* stream);
/* matmul_q4_0_batch (src/quant_kernels.cpp:82-91): y[b*rows + r]. */
MV_API int mv_int_matmul_q4_0_batch(const void* A20_dev, const float* x_dev, float* y_dev, uint64_t rows,
                                    uint64_t cols, uint64_t batch, void* stream);
/* matvec_f32, the sequential fp32 row dot of src/matmul.cpp:6-8 (row-major A). */
MV_API int mv_matvec_f32(const float* A_dev, const float* x_dev, float* y_dev, uint64_t rows, uint64_t cols,
                         void* stream);

/* ------------------------------------------------------------- model */

/* Device-resident LlamaModel backend: parses the GGUF (mmap), uploads every
 * weight once, builds the RoPE tables on the host exactly as the reference
 * does.  Replaces LlamaModel::LlamaModel / load_config
 * (src/llama_model.cpp:222-235, include/memvanta/llama_model.hpp:102).
 * ctx = 0 keeps the GGUF context length; page_tokens = 0 -> 128. */
MV_API int mv_model_open(const char* gguf_path, uint64_t ctx, uint64_t page_tokens, int kv_type, mv_model_t* out);
MV_API int mv_model_close(mv_model_t m);
/* n_ctx, n_embd, n_ff, n_layer, n_head, n_head_kv, vocab (7 values). */
MV_API int mv_model_config(mv_model_t m, uint64_t* out7);
MV_API int mv_model_reset(mv_model_t m);                       /* LlamaModel::reset, :236 */
MV_API uint64_t mv_model_position(mv_model_t m);               /* LlamaModel::position     */
MV_API uint64_t mv_model_kv_bytes(mv_model_t m);               /* kv_bytes_allocated       */
/* Decode one token; logits_host (vocab floats) may be NULL when
 * compute_logits is 0.  LlamaModel::forward, src/llama_model.cpp:253-259.
 * The decode attention keeps the reference's order bit for bit; with
 * MV_ATTN_SPLIT=1 in the environment at mv_model_open it is split over the
 * context instead (partial softmax states merged in a fixed order, ~1e-6
 * from the reference order per step -- enough for later Q8 activation
 * roundings to move the logits past 2e-2 over tens of steps). */
MV_API int mv_model_forward(mv_model_t m, int32_t token, int compute_logits, float* logits_host);
/* Prefill in chunks of `batch` tokens with Q8 activations (the reference's
 * MEMVANTA_FORCE_Q8_ACT=1 numerics).  LlamaModel::prefill, :260. */
MV_API int mv_model_prefill(mv_model_t m, const int32_t* tokens_host, uint64_t n, uint64_t batch, int compute_logits,
                     float* logits_host);
/* Greedy decode of n tokens starting from `token`, on the device: every step
 * is one captured CUDA graph and the argmax stays in HBM; only the n token ids
 * come back.  Matches forward()+Sampler::sample at temperature 0 (:60-61). */
MV_API int mv_model_generate_greedy(mv_model_t m, int32_t token, uint64_t n, int32_t* out_tokens_host);
/* The model's stream (cudaStream_t) -- for event timing by the caller. */
MV_API void* mv_model_stream(mv_model_t m);
/* 1 when a decode step runs every layer in one persistent kernel (one GPU,
 * Q4_0 layer weights, F16/F32 KV; chosen with MV_DECODE_PERSISTENT=1 in the
 * environment at mv_model_open), 0 when it runs one kernel per operation.
 * Both give identical outputs.  No counterpart in the reference. */
MV_API int mv_model_decode_persistent(mv_model_t m);

/* ------------------------------------- several sequences, one batch */

/* A set of n_seq sequences of up to ctx tokens each (ctx <= the model's
 * context) decoded together with model m's weights (one GPU).  Each sequence
 * has its own paged KV cache; the set's block table maps sequence i's pages
 * into one pool per layer (the layout of mv_paged_attn_decode).  The
 * reference decodes one sequence per LlamaModel; a row of a batched step is
 * that sequence's LlamaModel::forward (src/llama_model.cpp:253-257). */
MV_API int mv_model_seqs_open(mv_model_t m, uint64_t n_seq, uint64_t ctx, mv_seqs_t* out);
MV_API int mv_model_seqs_free(mv_seqs_t s);
/* mv_model_prefill for sequence `seq` of the set, from its position. */
MV_API int mv_model_seqs_prefill(mv_seqs_t s, uint64_t seq, const int32_t* tokens_host, uint64_t n, uint64_t batch,
                                 int compute_logits, float* logits_host);
MV_API int mv_model_seqs_position(mv_seqs_t s, uint64_t seq, uint64_t* pos);
MV_API int mv_model_seqs_reset(mv_seqs_t s, uint64_t seq);
/* One decode step of every sequence of the set: tokens_host[n_seq], one per
 * sequence at its own position; logits_host receives [n_seq][vocab] (may be
 * NULL).  The projections run as one batch of n_seq rows (the weights are
 * read once for all sequences) with the per-row arithmetic of mv_model_forward,
 * the attention through the set's block table. */
MV_API int mv_model_forward_batch(mv_model_t m, mv_seqs_t s, const int32_t* tokens_host, float* logits_host);

/* ---------------------------------------------- tensor parallel model */

/* One process per GPU, `world` ranks of one node (2..8).  The reference runs
 * on one host and has no counterpart; these three calls split the same
 * LlamaModel over NVLink so that every call above returns the results of
 * mv_model_open bit for bit.  Rank r holds q heads [r*H/world, ...), the same
 * share of kv heads and their KV cache, and 1/world of the rows of every
 * other matrix (o, gate, up, down, output); activations stay replicated and
 * each kernel stores its slice into every rank's copy over peer memory.
 * Needs Q4_0 layer weights, heads / kv heads / n_embd / n_ff / vocab divisible
 * by world, and a KV type other than MV_KV_Q8.  prefill_batch bounds the
 * `batch` of mv_model_prefill (0 -> 64) and the batches a call's chunks
 * merge into (up to 512 tokens).  Protocol:
 *   mv_model_open_tp on every rank; mv_model_tp_handle on every rank; gather
 *   the world handles (MV_TP_HANDLE_BYTES each, rank order) on every rank by
 *   any host channel; mv_model_tp_connect on every rank at the same time.
 * Afterwards every rank makes the same calls in the same order, each within
 * the wait bound of the others (default 5 s, mv_model_tp_set_timeout).  A
 * rank that stops answering makes the others' calls fail with MV_ERR_TIMEOUT
 * once the bound runs out; the ranks are then out of step and every model is
 * closed. */
#define MV_TP_HANDLE_BYTES 64
MV_API int mv_model_open_tp(const char* gguf_path, uint64_t ctx, uint64_t page_tokens, int kv_type, int rank,
                            int world, uint64_t prefill_batch, mv_model_t* out);
MV_API int mv_model_tp_handle(mv_model_t m, void* handle_out);
MV_API int mv_model_tp_connect(mv_model_t m, const void* handles);
/* Unmaps the other ranks' blocks (the model is unusable afterwards).  To
 * close: barrier, mv_model_tp_disconnect, barrier, mv_model_close. */
MV_API int mv_model_tp_disconnect(mv_model_t m);
/* Bound, in milliseconds, of every wait for the other ranks (default 5000). */
MV_API int mv_model_tp_set_timeout(mv_model_t m, uint64_t ms);

#ifdef __cplusplus
}
#endif
#endif /* MEMVANTA_B200_H */
