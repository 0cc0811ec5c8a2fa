// capi.cu -- the extern "C" boundary (include/memvanta_b200.h).
//
// Argument checks mirror the reference's std::runtime_error conditions
// (src/gguf_kernels.cpp:245-251, :256-257, :262, :161-163) but return status
// codes; CUDA failures come back as MV_ERR_CUDA with the runtime's message.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/memvanta_b200.h"
#include "kernels.cuh"
#include "weights.cuh"

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
    g_err = msg;
    return code;
}
int cuda_fail(cudaError_t e, const char* what) {
    cudaGetLastError();  // clear a sticky-free launch error so later calls start clean
    return fail(e == cudaErrorMemoryAllocation ? MV_ERR_OOM : MV_ERR_CUDA,
                std::string(what) + ": " + cudaGetErrorString(e));
}

#define CK(call)                                        \
    do {                                                \
        cudaError_t e_ = (call);                        \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call); \
    } while (0)

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

bool type_supported(int t) { return t == 0 || t == 1 || t == 2 || t == 8 || t == 14; }
const char* type_name(int t) {
    switch (t) {
        case 0: return "F32";
        case 1: return "F16";
        case 2: return "Q4_0";
        case 8: return "Q8_0";
        case 14: return "Q6_K";
    }
    return "unknown";
}

uint64_t align256(uint64_t n) { return (n + 255) & ~uint64_t(255); }

// Stream used by the synchronous host-pointer calls: one per thread.
cudaStream_t host_stream() {
    static thread_local cudaStream_t s = nullptr;
    if (!s) cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    return s;
}

// Device buffers reused by the host-pointer calls of one thread (grown on
// demand, never shrunk), so a tensor_matvec-style call costs two copies and a
// launch rather than two allocations as well.
struct HostCallBuffers {
    void* x = nullptr;
    void* y = nullptr;
    size_t nx = 0, ny = 0;
    ~HostCallBuffers() {
        if (x) cudaFree(x);
        if (y) cudaFree(y);
    }
    cudaError_t reserve(size_t bx, size_t by) {
        if (bx > nx) {
            if (x) cudaFree(x);
            x = nullptr;
            nx = 0;
            if (cudaError_t e = cudaMalloc(&x, bx)) return e;
            nx = bx;
        }
        if (by > ny) {
            if (y) cudaFree(y);
            y = nullptr;
            ny = 0;
            if (cudaError_t e = cudaMalloc(&y, by)) return e;
            ny = by;
        }
        return cudaSuccess;
    }
};
HostCallBuffers& host_buffers() {
    static thread_local HostCallBuffers b;
    return b;
}

// Stream-ordered scratch (cudaMallocAsync) comes from the device's default
// pool; keep freed blocks in the pool instead of returning them to the driver
// at every synchronisation.
void keep_pool_memory(int device) {
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
        uint64_t threshold = UINT64_MAX;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
    }
}

int check_weight(const mv_weight_s* w) {
    if (!w) return fail(MV_ERR_INVALID, "null weight handle");
    return MV_OK;
}

// Allocates the planes of `w` (type/rows/cols/nb already set).
int alloc_planes(mv_weight_s* w) {
    const uint64_t nbl = w->rows * w->nb;
    uint64_t q = 0, h = 0, sc = 0, d = 0;
    switch (w->type) {
        case 2: q = nbl * 16; d = w->rows * w->dstride * 2; break;
        case 8: q = nbl * 32; d = nbl * 2; break;
        case 14: q = nbl * 128; h = nbl * 64; sc = nbl * 16; d = nbl * 2; break;
        case 1: q = w->rows * w->cols * 2; break;
        case 0: q = w->rows * w->cols * 4; break;
    }
    const uint64_t oq = 0, oh = align256(oq + q), osc = align256(oh + h), od = align256(osc + sc);
    w->bytes = align256(od + d);
    void* base = nullptr;
    cudaError_t e = cudaMalloc(&base, w->bytes ? w->bytes : 256);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(weight)");
    w->base = base;
    uint8_t* b = static_cast<uint8_t*>(base);
    w->qs = b + oq;
    w->qh = h ? b + oh : nullptr;
    w->sc = sc ? reinterpret_cast<int8_t*>(b + osc) : nullptr;
    w->d = d ? reinterpret_cast<uint16_t*>(b + od) : nullptr;
    if (w->d && w->dstride != w->nb) {
        e = cudaMemset(w->d, 0, d);  // padding scales stay zero
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(scales)");
    }
    return MV_OK;
}

int make_weight(uint64_t nbytes, int type, uint64_t rows, uint64_t cols, mv_weight_s** out) {
    if (!out) return fail(MV_ERR_INVALID, "null output handle");
    *out = nullptr;
    if (!type_supported(type)) return fail(MV_ERR_UNSUPPORTED, "unsupported tensor type " + std::to_string(type));
    if (rows == 0 || cols == 0) return fail(MV_ERR_INVALID, "weight needs rows > 0 and cols > 0");
    const uint64_t per = mvb::ggml_block_elems(type);
    if (cols % per)
        return fail(MV_ERR_INVALID, std::string(type_name(type)) + " matrix row not block aligned (cols % " +
                                        std::to_string(per) + " != 0)");
    const uint64_t expect = rows * (cols / per) * mvb::ggml_block_bytes(type);
    if (nbytes != expect)
        return fail(MV_ERR_INVALID, "nbytes " + std::to_string(nbytes) + " != " + std::to_string(expect) +
                                        " for a " + type_name(type) + " " + std::to_string(rows) + "x" +
                                        std::to_string(cols) + " tensor");
    auto* w = new mv_weight_s();
    w->type = type;
    w->rows = rows;
    w->cols = cols;
    w->nb = cols / per;
    w->dstride = type == 2 ? (w->nb + 7) / 8 * 8 : w->nb;
    cudaGetDevice(&w->device);
    if (int rc = alloc_planes(w)) {
        delete w;
        return rc;
    }
    *out = w;
    return MV_OK;
}

int upload_common(const void* src, bool src_on_device, uint64_t nbytes, int type, uint64_t rows, uint64_t cols,
                  void* stream, mv_weight_t* out) {
    if (!src) return fail(MV_ERR_INVALID, "null source pointer");
    mv_weight_s* w = nullptr;
    if (int rc = make_weight(nbytes, type, rows, cols, &w)) return rc;
    cudaStream_t s = as_stream(stream);
    const uint8_t* raw = static_cast<const uint8_t*>(src);
    void* staging = nullptr;
    auto cleanup = [&](int rc) {
        if (staging) cudaFree(staging);
        if (rc) {
            cudaFree(w->base);
            delete w;
        }
        return rc;
    };
    if (!src_on_device) {
        cudaError_t e = cudaMalloc(&staging, nbytes);
        if (e != cudaSuccess) return cleanup(cuda_fail(e, "cudaMalloc(staging)"));
        e = cudaMemcpyAsync(staging, src, nbytes, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return cleanup(cuda_fail(e, "cudaMemcpyAsync(upload)"));
        raw = static_cast<const uint8_t*>(staging);
    }
    cudaError_t e = mvb::repack_from_ggml(*w, raw, s);
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "repack"));
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "cudaStreamSynchronize(upload)"));
    cleanup(MV_OK);
    *out = w;
    return MV_OK;
}

}  // namespace

namespace mvb {
void set_last_error(const std::string& msg) { g_err = msg; }
}  // namespace mvb

extern "C" {

MV_API const char* mv_last_error(void) { return g_err.c_str(); }
MV_API int mv_version(void) { return 1; }

namespace {
// An empty kernel whose attributes stand for the library's device code.
__global__ void arch_probe_kernel() {}
}  // namespace

MV_API int mv_binary_arch(int* out) {
    if (!out) return fail(MV_ERR_INVALID, "null output");
    cudaFuncAttributes a{};
    CK(cudaFuncGetAttributes(&a, arch_probe_kernel));
    *out = a.binaryVersion;
    return MV_OK;
}

MV_API int mv_init(int device) {
    int n = 0;
    CK(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) return fail(MV_ERR_INVALID, "device " + std::to_string(device) + " out of range");
    CK(cudaSetDevice(device));
    int major = 0;
    CK(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
    if (major != 10)
        return fail(MV_ERR_UNSUPPORTED, "memvanta_b200 is built for sm_100a; device has compute capability " +
                                            std::to_string(major) + ".x");
    keep_pool_memory(device);
    return MV_OK;
}

// ------------------------------------------------------------- weights
MV_API int mv_weight_upload(const void* host_blocks, uint64_t nbytes, int ggml_type, uint64_t rows, uint64_t cols,
                            void* stream, mv_weight_t* out) {
    return upload_common(host_blocks, false, nbytes, ggml_type, rows, cols, stream, out);
}
MV_API int mv_weight_from_device(const void* dev_blocks, uint64_t nbytes, int ggml_type, uint64_t rows, uint64_t cols,
                                 void* stream, mv_weight_t* out) {
    return upload_common(dev_blocks, true, nbytes, ggml_type, rows, cols, stream, out);
}
MV_API int mv_weight_free(mv_weight_t w) {
    if (!w) return MV_OK;
    cudaError_t e = cudaFree(w->base);
    delete w;
    if (e != cudaSuccess) return cuda_fail(e, "cudaFree(weight)");
    return MV_OK;
}
MV_API int mv_weight_info(mv_weight_t w, int* type, uint64_t* rows, uint64_t* cols, uint64_t* bytes) {
    if (int rc = check_weight(w)) return rc;
    if (type) *type = w->type;
    if (rows) *rows = w->rows;
    if (cols) *cols = w->cols;
    if (bytes) *bytes = w->bytes;
    return MV_OK;
}
MV_API int mv_weight_download(mv_weight_t w, void* host_blocks, uint64_t nbytes) {
    if (int rc = check_weight(w)) return rc;
    const uint64_t expect = w->rows * w->nb * mvb::ggml_block_bytes(w->type);
    if (nbytes != expect || !host_blocks) return fail(MV_ERR_INVALID, "download buffer size mismatch");
    cudaStream_t s = host_stream();
    void* raw = nullptr;
    CK(cudaMalloc(&raw, nbytes));
    cudaError_t e = mvb::unpack_to_ggml(*w, static_cast<uint8_t*>(raw), s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(host_blocks, raw, nbytes, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    cudaFree(raw);
    if (e != cudaSuccess) return cuda_fail(e, "download");
    return MV_OK;
}

// ------------------------------------------------------------- matmuls
MV_API int mv_gemv(mv_weight_t w, const float* x, float* y, void* stream) {
    if (int rc = check_weight(w)) return rc;
    if (!x || !y) return fail(MV_ERR_INVALID, "null x or y");
    cudaStream_t s = as_stream(stream);
    if (w->type == 2) {
        if (reinterpret_cast<uintptr_t>(x) % 16) return fail(MV_ERR_INVALID, "x must be 16-byte aligned");
        mvb::GemvQ4Args a{w, x, nullptr, 0.0f, y, mvb::Q4Pro::Plain, mvb::Q4Epi::Store};
        CK(mvb::gemv_q4(a, s));
    } else if (w->type == 14 && w->cols * 4 <= 200 * 1024) {
        CK(mvb::gemv_q6k(*w, x, y, s));
    } else if (w->type == 8 && w->cols * 4 <= 200 * 1024 && reinterpret_cast<uintptr_t>(x) % 16 == 0) {
        CK(mvb::gemv_q8_0(*w, x, y, s));
    } else {
        CK(mvb::matmul_f32act(*w, x, 1, y, s));
    }
    return MV_OK;
}

MV_API int mv_gemm(mv_weight_t w, const float* x, uint64_t batch, float* y, int act_mode, void* stream) {
    if (int rc = check_weight(w)) return rc;
    if (batch == 0) return MV_OK;
    if (!x || !y) return fail(MV_ERR_INVALID, "null x or y");
    if (act_mode != MV_ACT_F32 && act_mode != MV_ACT_Q8) return fail(MV_ERR_INVALID, "unknown act_mode");
    cudaStream_t s = as_stream(stream);
    // The reference routes batch < 2 and every type but Q4_0/Q8_0 to
    // tensor_matmul_batch (fp32 activations), and keeps fp32 activations for
    // Q8_0 even under MEMVANTA_FORCE_Q8_ACT (src/gguf_kernels.cpp:263-266).
    if (batch < 2 || w->type != 2 || act_mode == MV_ACT_F32) {
        CK(mvb::matmul_f32act(*w, x, batch, y, s));
        return MV_OK;
    }
    // Q4_0 with Q8 activations: per-row quantisation into stream-ordered
    // scratch (scales block-major), then the tensor-core GEMM.
    // 64 tokens and more: fp16 operands (gemm_f16.cu), else int8 (gemm_tc.cu)
    const uint64_t ldb = mvb::gemm_tc_ldb(batch);
    const bool f16 = mvb::gemm_f16_preferred(batch);
    int8_t* q = nullptr;
    float* d = nullptr;
    CK(cudaMallocAsync(reinterpret_cast<void**>(&q), batch * w->cols * (f16 ? 2 : 1), s));
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&d), 2 * (w->cols / 32) * ldb * sizeof(float), s);
    uint16_t* qh = f16 ? reinterpret_cast<uint16_t*>(q) : nullptr;
    if (e == cudaSuccess) e = mvb::quantize_q8_rows_t(x, batch, w->cols, q, d, ldb, s, qh);
    if (e == cudaSuccess)
        e = f16 ? mvb::gemm_q4_q8_f16(*w, qh, d, ldb, batch, y, s) : mvb::gemm_q4_q8_tc(*w, q, d, ldb, batch, y, s);
    cudaFreeAsync(q, s);
    if (d) cudaFreeAsync(d, s);
    if (e != cudaSuccess) return cuda_fail(e, "gemm_q4_q8_tc");
    return MV_OK;
}

MV_API int mv_stream_status(void* stream) {
    int status = 0;
    CK(mvb::tc_status(as_stream(stream), &status));
    if (status) return fail(MV_ERR_TIMEOUT, "a tensor-core kernel gave up a bounded wait (site " +
                                                std::to_string(status) + "); its outputs are invalid");
    return MV_OK;
}

MV_API int mv_test_gemm_stall(int skip_commit_stage, uint64_t wait_limit_us) {
    if (skip_commit_stage < -1 || wait_limit_us > 10000000ull) return fail(MV_ERR_INVALID, "bad test stall");
    mvb::gemm_f16_test_stall(skip_commit_stage, wait_limit_us * 1000ull);
    return MV_OK;
}

MV_API int mv_quantize_q8(const float* x, uint64_t rows, uint64_t cols, int8_t* q, float* d, void* stream) {
    if (cols % 32) return fail(MV_ERR_INVALID, "Q8 activation quantization requires cols multiple of 32");
    if (rows && (!x || !q || !d)) return fail(MV_ERR_INVALID, "null pointer");
    CK(mvb::quantize_q8_rows(x, rows, cols, q, d, as_stream(stream)));
    return MV_OK;
}

MV_API int mv_q4_0_block_dots(mv_weight_t w, const float* x, int32_t* isum, void* stream) {
    if (int rc = check_weight(w)) return rc;
    if (w->type != 2) return fail(MV_ERR_UNSUPPORTED, "block dots need a Q4_0 weight");
    CK(mvb::q4_block_dots(*w, x, isum, as_stream(stream)));
    return MV_OK;
}

MV_API int mv_read_rows(mv_weight_t w, const int32_t* rows, uint64_t n, float* out, void* stream) {
    if (int rc = check_weight(w)) return rc;
    if (n && (!rows || !out)) return fail(MV_ERR_INVALID, "null pointer");
    CK(mvb::read_rows(*w, rows, n, out, as_stream(stream)));
    return MV_OK;
}

MV_API int mv_read_row(mv_weight_t w, uint64_t row, float* out, void* stream) {
    if (int rc = check_weight(w)) return rc;
    if (row >= w->rows) return fail(MV_ERR_INVALID, "tensor row out of range");
    cudaStream_t s = as_stream(stream);
    int32_t* d_row = nullptr;
    CK(cudaMallocAsync(reinterpret_cast<void**>(&d_row), sizeof(int32_t), s));
    const int32_t r = (int32_t)row;
    cudaError_t e = cudaMemcpyAsync(d_row, &r, sizeof(r), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = mvb::read_rows(*w, d_row, 1, out, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);  // `r` lives on this stack frame
    cudaFreeAsync(d_row, s);
    if (e != cudaSuccess) return cuda_fail(e, "read_row");
    return MV_OK;
}

// ----------------------------------------------------------------- ops
MV_API int mv_rmsnorm(const float* x, const float* w, uint64_t rows, uint64_t n, float eps, float* out, void* stream) {
    if (rows && (!x || !w || !out || !n)) return fail(MV_ERR_INVALID, "bad rmsnorm arguments");
    CK(mvb::rmsnorm_rows(x, w, rows, n, eps, out, as_stream(stream)));
    return MV_OK;
}
MV_API int mv_rope(float* q, uint64_t n_head, float* k, uint64_t n_head_kv, uint64_t hd, uint64_t rows,
                   const float* cos_t, const float* sin_t, const int32_t* pos, void* stream) {
    if (hd % 2) return fail(MV_ERR_INVALID, "head_dim must be even");
    CK(mvb::rope_rows(q, n_head, k, n_head_kv, hd, rows, cos_t, sin_t, pos, as_stream(stream)));
    return MV_OK;
}
MV_API int mv_silu_mul(const float* g, const float* u, float* out, uint64_t n, void* stream) {
    CK(mvb::silu_mul(g, u, out, n, as_stream(stream)));
    return MV_OK;
}
MV_API int mv_add_inplace(float* x, const float* y, uint64_t n, void* stream) {
    CK(mvb::add_inplace(x, y, n, as_stream(stream)));
    return MV_OK;
}
MV_API int mv_fp32_to_fp16(const float* x, uint16_t* h, uint64_t n, void* stream) {
    CK(mvb::f32_to_f16_ref(x, h, n, as_stream(stream)));
    return MV_OK;
}

// -------------------------------------------------------------- KV cache
MV_API uint64_t mv_kv_row_bytes(int kv_type, uint64_t kv_dim) { return mvb::kv_row_bytes(kv_type, kv_dim); }
MV_API uint64_t mv_kv_row_scales(int kv_type, uint64_t kv_dim) { return mvb::kv_row_scales(kv_type, kv_dim); }

MV_API int mv_kv_append(int kv_type, const float* k, const float* v, uint64_t rows, uint64_t kv_dim,
                        const int32_t* seq, const int32_t* pos, const int32_t* block_table, uint64_t max_pages,
                        uint64_t page, void* k_pages, void* v_pages, float* k_scales, float* v_scales,
                        void* stream) {
    if (kv_type < 0 || kv_type > 3) return fail(MV_ERR_UNSUPPORTED, "unknown KV cache type");
    if (kv_type == 3 && kv_dim % 32) return fail(MV_ERR_INVALID, "Q8_0 KV needs kv_dim % 32 == 0");
    if (kv_type >= 2 && (!k_scales || !v_scales)) return fail(MV_ERR_INVALID, "Q8 KV needs scale arrays");
    if (!page) return fail(MV_ERR_INVALID, "page must be > 0");
    CK(mvb::kv_append(kv_type, k, v, rows, kv_dim, seq, pos, block_table, max_pages, page, k_pages, v_pages,
                      k_scales, v_scales, as_stream(stream)));
    return MV_OK;
}

MV_API int mv_paged_attn_decode(int kv_type, const float* q, uint64_t n_seq, uint64_t n_head, uint64_t n_head_kv,
                                uint64_t hd, const void* k_pages, const void* v_pages, const float* k_scales,
                                const float* v_scales, const int32_t* block_table, uint64_t max_pages, uint64_t page,
                                const int32_t* ctx_len, uint64_t max_ctx, float* out, void* stream) {
    if (kv_type < 0 || kv_type > 3) return fail(MV_ERR_UNSUPPORTED, "unknown KV cache type");
    if (!n_head_kv || n_head % n_head_kv || n_head / n_head_kv > 8)
        return fail(MV_ERR_INVALID, "n_head must be a multiple (<= 8x) of n_head_kv");
    if (hd != 64 && hd != 128 && hd != 256) return fail(MV_ERR_UNSUPPORTED, "head_dim must be 64, 128 or 256");
    if (!page) return fail(MV_ERR_INVALID, "page must be > 0");
    if (n_seq == 0) return MV_OK;
    if (mvb::attn_smem_bytes(hd, max_ctx ? max_ctx : 1, max_pages, kv_type) > 200 * 1024)
        return fail(MV_ERR_INVALID, "max_ctx too large for one attention CTA");
    mvb::AttnArgs a{kv_type, q, n_head * hd, n_seq, n_head, n_head_kv, hd, k_pages, v_pages, k_scales, v_scales,
                    block_table, max_pages, page, ctx_len, max_ctx ? max_ctx : 1, out};
    CK(mvb::paged_attn_decode(a, as_stream(stream)));
    return MV_OK;
}

MV_API int mv_paged_attn_decode_split(int kv_type, const float* q, uint64_t n_seq, uint64_t n_head,
                                      uint64_t n_head_kv, uint64_t hd, const void* k_pages, const void* v_pages,
                                      const float* k_scales, const float* v_scales, const int32_t* block_table,
                                      uint64_t max_pages, uint64_t page, const int32_t* ctx_len, uint64_t max_ctx,
                                      float* out, void* stream) {
    if (kv_type < 0 || kv_type > 3) return fail(MV_ERR_UNSUPPORTED, "unknown KV cache type");
    if (!n_head_kv || n_head % n_head_kv) return fail(MV_ERR_INVALID, "n_head must be a multiple of n_head_kv");
    if (hd != 64 && hd != 128 && hd != 256) return fail(MV_ERR_UNSUPPORTED, "head_dim must be 64, 128 or 256");
    if (!page) return fail(MV_ERR_INVALID, "page must be > 0");
    if (kv_type >= 2 && !(k_scales && v_scales)) return fail(MV_ERR_INVALID, "Q8 caches need k_scales and v_scales");
    if (n_seq == 0) return MV_OK;
    mvb::AttnArgs a{kv_type, q, n_head * hd, n_seq, n_head, n_head_kv, hd, k_pages, v_pages, k_scales, v_scales,
                    block_table, max_pages, page, ctx_len, max_ctx ? max_ctx : 1, out};
    CK(mvb::paged_attn_decode_split(a, as_stream(stream)));
    return MV_OK;
}

MV_API int mv_paged_attn_prefill(int kv_type, const float* q, uint64_t n_q, uint64_t n_head, uint64_t n_head_kv,
                                 uint64_t hd, const void* k_pages, const void* v_pages, const float* k_scales,
                                 const float* v_scales, const int32_t* block_table, uint64_t max_pages, uint64_t page,
                                 const int32_t* ctx_len, uint64_t max_ctx, float* out, void* stream) {
    if (kv_type < 0 || kv_type > 3) return fail(MV_ERR_UNSUPPORTED, "unknown KV cache type");
    if (!n_head_kv || n_head % n_head_kv || n_head / n_head_kv > 8)
        return fail(MV_ERR_INVALID, "n_head must be a multiple (<= 8x) of n_head_kv");
    if (hd != 64 && hd != 128 && hd != 256) return fail(MV_ERR_UNSUPPORTED, "head_dim must be 64, 128 or 256");
    if (!page) return fail(MV_ERR_INVALID, "page must be > 0");
    if (n_q == 0) return MV_OK;
    if (mvb::attn_smem_bytes(hd, max_ctx ? max_ctx : 1, max_pages, kv_type) > 200 * 1024)
        return fail(MV_ERR_INVALID, "max_ctx too large for one attention CTA");
    mvb::AttnArgs a{kv_type, q, n_head * hd, n_q, n_head, n_head_kv, hd, k_pages, v_pages, k_scales, v_scales,
                    block_table, max_pages, page, ctx_len, max_ctx ? max_ctx : 1, out};
    a.one_seq = 1;
    CK(mvb::paged_attn_prefill(a, as_stream(stream)));
    return MV_OK;
}

// ---------------------------------------------------- host-pointer calls
MV_API int mv_tensor_matvec_host(mv_weight_t w, const float* x_host, float* y_host) {
    if (int rc = check_weight(w)) return rc;
    if (!x_host || !y_host) return fail(MV_ERR_INVALID, "null x or y");
    cudaStream_t s = host_stream();
    HostCallBuffers& hb = host_buffers();
    CK(hb.reserve(w->cols * sizeof(float), w->rows * sizeof(float)));
    float* x = static_cast<float*>(hb.x);
    float* y = static_cast<float*>(hb.y);
    CK(cudaMemcpyAsync(x, x_host, w->cols * sizeof(float), cudaMemcpyHostToDevice, s));
    if (int rc = mv_gemv(w, x, y, s)) return rc;
    CK(cudaMemcpyAsync(y_host, y, w->rows * sizeof(float), cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    return MV_OK;
}

MV_API int mv_tensor_matmul_batch_host(mv_weight_t w, const float* x_host, float* y_host, uint64_t batch,
                                       int act_mode) {
    if (int rc = check_weight(w)) return rc;
    if (batch == 0) return MV_OK;
    if (!x_host || !y_host) return fail(MV_ERR_INVALID, "null x or y");
    cudaStream_t s = host_stream();
    HostCallBuffers& hb = host_buffers();
    CK(hb.reserve(batch * w->cols * sizeof(float), batch * w->rows * sizeof(float)));
    float* x = static_cast<float*>(hb.x);
    float* y = static_cast<float*>(hb.y);
    CK(cudaMemcpyAsync(x, x_host, batch * w->cols * sizeof(float), cudaMemcpyHostToDevice, s));
    if (int rc = mv_gemm(w, x, batch, y, act_mode, s)) return rc;
    CK(cudaMemcpyAsync(y_host, y, batch * w->rows * sizeof(float), cudaMemcpyDeviceToHost, s));
    return mv_stream_status(s);
}

MV_API int mv_tensor_read_row_host(mv_weight_t w, uint64_t row, float* out_host) {
    if (int rc = check_weight(w)) return rc;
    if (!out_host) return fail(MV_ERR_INVALID, "null output");
    cudaStream_t s = host_stream();
    HostCallBuffers& hb = host_buffers();
    CK(hb.reserve(sizeof(int32_t), w->cols * sizeof(float)));
    if (int rc = mv_read_row(w, row, static_cast<float*>(hb.y), s)) return rc;
    CK(cudaMemcpyAsync(out_host, hb.y, w->cols * sizeof(float), cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    return MV_OK;
}

}  // extern "C"
