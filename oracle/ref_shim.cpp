// ref_shim.cpp -- C entry points into the reference implementation itself.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the unmodified MemVanta sources (read in place from the reference checkout)
// into oracle/_ref/libmvref.so.  It lets the tests pin the C restatement in
// mv_oracle.c against the reference's own code and lets bench.py time the
// reference's CPU path.  Nothing in the product library links or loads it.
//
// gguf_kernels.cpp is #included (not compiled separately) so that its
// anonymous-namespace helpers -- quantize_q8, dot_q4_q8_block, q6_k_value --
// become reachable for per-block bit-exact checks.
#include "src/gguf_kernels.cpp"

#include "memvanta/llama_model.hpp"
#include "memvanta/quant.hpp"
#include "memvanta/matmul.hpp"

#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>

namespace {
thread_local std::string g_err;
template <class Fn>
int guarded(Fn&& fn) {
    try {
        fn();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}
struct ForceQ8Env {
    bool set;
    explicit ForceQ8Env(int on) : set(on != 0) {
        if (set) setenv("MEMVANTA_FORCE_Q8_ACT", "1", 1); else unsetenv("MEMVANTA_FORCE_Q8_ACT");
    }
    ~ForceQ8Env() { unsetenv("MEMVANTA_FORCE_Q8_ACT"); }
};
}  // namespace

#define API extern "C" __attribute__((visibility("default")))

API const char* mvr_last_error() { return g_err.c_str(); }

// ---- per-block internals (src/gguf_kernels.cpp:122-189, :242; src/gguf.cpp:110) ----
API void mvr_quantize_q8(const float* x, std::size_t cols, std::int8_t* q, float* d) {
    auto a = memvanta::quantize_q8(x, cols);
    std::memcpy(q, a.q.data(), cols);
    std::memcpy(d, a.d.data(), a.d.size() * sizeof(float));
}
API int mvr_dot_q4_q8_block(const void* blk18, const std::int8_t* aq) {
    return memvanta::dot_q4_q8_block(*static_cast<const memvanta::GgufBlockQ4_0*>(blk18), aq);
}
API int mvr_q6_k_value(const void* blk210, std::size_t i) {
    return memvanta::q6_k_value(*static_cast<const memvanta::GgufBlockQ6_K*>(blk210), i);
}
API std::uint16_t mvr_fp32_to_fp16(float f) { return memvanta::fp32_to_fp16(f); }
API float mvr_fp16_to_fp32(std::uint16_t h) { return memvanta::fp16_to_fp32(h); }

// ---- GGUF-layout public kernels (src/gguf_kernels.cpp:224-271) ----
API void* mvr_file_open(const char* path) {
    memvanta::GgufFile* f = nullptr;
    if (guarded([&] { f = new memvanta::GgufFile(path); })) return nullptr;
    return f;
}
API void mvr_file_close(void* f) { delete static_cast<memvanta::GgufFile*>(f); }

static const memvanta::GgufTensor& T(void* f, const char* name) {
    return static_cast<memvanta::GgufFile*>(f)->tensor(name);
}
API int mvr_matvec(void* f, const char* name, const float* x, float* y, unsigned threads) {
    return guarded([&] { memvanta::tensor_matvec(*static_cast<memvanta::GgufFile*>(f), T(f, name), x, y, threads, nullptr); });
}
API int mvr_matmul_batch(void* f, const char* name, const float* x, float* y, std::size_t batch, unsigned threads) {
    return guarded([&] { memvanta::tensor_matmul_batch(*static_cast<memvanta::GgufFile*>(f), T(f, name), x, y, batch, threads, nullptr); });
}
API int mvr_matmul_batch_v06(void* f, const char* name, const float* x, float* y, std::size_t batch, unsigned threads,
                             int force_q8) {
    ForceQ8Env env(force_q8);
    return guarded([&] { memvanta::tensor_matmul_batch_v06(*static_cast<memvanta::GgufFile*>(f), T(f, name), x, y, batch, threads, nullptr); });
}
API int mvr_read_row(void* f, const char* name, std::size_t row, float* out, std::size_t cols) {
    return guarded([&] { memvanta::tensor_read_row_f32(*static_cast<memvanta::GgufFile*>(f), T(f, name), row, out, cols); });
}

// ---- PagedKVCache (src/llama_model.cpp:18-56) ----
API void* mvr_kv_new(std::size_t kv_dim, std::size_t page, int type) {
    return new memvanta::PagedKVCache(kv_dim, page, static_cast<memvanta::KVCacheType>(type));
}
API void mvr_kv_free(void* c) { delete static_cast<memvanta::PagedKVCache*>(c); }
API void mvr_kv_write(void* c, std::size_t pos, const float* k, const float* v) {
    static_cast<memvanta::PagedKVCache*>(c)->write(pos, k, v);
}
API float mvr_kv_dot_key(void* c, std::size_t pos, std::size_t off, const float* q, std::size_t n) {
    return static_cast<memvanta::PagedKVCache*>(c)->dot_key(pos, off, q, n);
}
API void mvr_kv_add_value(void* c, std::size_t pos, std::size_t off, float alpha, float* out, std::size_t n) {
    static_cast<memvanta::PagedKVCache*>(c)->add_value(pos, off, alpha, out, n);
}

// ---- LlamaModel (src/llama_model.cpp:222-263) ----
API void* mvr_model_open(const char* path, unsigned threads, std::size_t ctx, std::size_t page, int kv_type) {
    memvanta::LlamaModel* m = nullptr;
    if (guarded([&] { m = new memvanta::LlamaModel(path, threads, ctx, page, static_cast<memvanta::KVCacheType>(kv_type)); }))
        return nullptr;
    return m;
}
API void mvr_model_free(void* m) { delete static_cast<memvanta::LlamaModel*>(m); }
API void mvr_model_reset(void* m) { static_cast<memvanta::LlamaModel*>(m)->reset(); }
API std::size_t mvr_model_position(void* m) { return static_cast<memvanta::LlamaModel*>(m)->position(); }
API std::size_t mvr_model_vocab(void* m) { return static_cast<memvanta::LlamaModel*>(m)->config().vocab; }
API std::size_t mvr_model_n_ctx(void* m) { return static_cast<memvanta::LlamaModel*>(m)->config().n_ctx; }
API int mvr_model_forward(void* m, int token, int compute_logits, float* logits) {
    return guarded([&] {
        auto* M = static_cast<memvanta::LlamaModel*>(m);
        const auto& l = M->forward(token, compute_logits != 0);
        if (compute_logits && logits) std::memcpy(logits, l.data(), l.size() * sizeof(float));
    });
}
API int mvr_model_prefill(void* m, const int* tokens, std::size_t n, std::size_t batch, int compute_logits,
                          float* logits, int force_q8) {
    ForceQ8Env env(force_q8);
    return guarded([&] {
        auto* M = static_cast<memvanta::LlamaModel*>(m);
        std::vector<int> t(tokens, tokens + n);
        const auto& l = M->prefill(t, batch, compute_logits != 0);
        if (compute_logits && logits) std::memcpy(logits, l.data(), l.size() * sizeof(float));
    });
}
API int mvr_model_forward_q8env(void* m, int token, int compute_logits, float* logits, int force_q8) {
    ForceQ8Env env(force_q8);
    return mvr_model_forward(m, token, compute_logits, logits);
}

// ---- internal formats (src/quant.cpp, src/quant_kernels.cpp, src/matmul.cpp) ----
API void mvr_int_quantize_q8_0(const float* x, std::size_t n, void* out) {
    auto v = memvanta::quantize_q8_0(x, n);
    std::memcpy(out, v.data(), v.size() * sizeof(memvanta::BlockQ8_0));
}
API void mvr_int_quantize_q4_0(const float* x, std::size_t n, void* out) {
    auto v = memvanta::quantize_q4_0(x, n);
    std::memcpy(out, v.data(), v.size() * sizeof(memvanta::BlockQ4_0));
}
API void mvr_int_matvec_q4_q8(const void* A, const void* x, float* y, std::size_t rows, std::size_t cols, unsigned th) {
    memvanta::matvec_q4_q8(static_cast<const memvanta::BlockQ4_0*>(A), static_cast<const memvanta::BlockQ8_0*>(x), y, rows, cols, th);
}
API void mvr_int_matvec_q4_0(const void* A, const float* x, float* y, std::size_t rows, std::size_t cols, unsigned th) {
    memvanta::matvec_q4_0(static_cast<const memvanta::BlockQ4_0*>(A), x, y, rows, cols, th);
}
API void mvr_int_matvec_q8_0(const void* A, const float* x, float* y, std::size_t rows, std::size_t cols, unsigned th) {
    memvanta::matvec_q8_0(static_cast<const memvanta::BlockQ8_0*>(A), x, y, rows, cols, th);
}
API void mvr_int_matmul_q4_0_batch(const void* A, const float* x, float* y, std::size_t rows, std::size_t cols,
                                   std::size_t batch, unsigned th) {
    memvanta::matmul_q4_0_batch(static_cast<const memvanta::BlockQ4_0*>(A), x, y, rows, cols, batch, th);
}
API void mvr_matvec_f32(const float* A, const float* x, float* y, std::size_t rows, std::size_t cols, unsigned th) {
    memvanta::matvec_f32(A, x, y, rows, cols, th);
}
