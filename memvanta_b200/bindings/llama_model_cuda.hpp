// llama_model_cuda.hpp -- the reference-side binding of the device-resident
// model: memvanta::CudaLlamaModel has the public interface of MemVanta's
// memvanta::LlamaModel (include/memvanta/llama_model.hpp:100-116), with the
// weights, the paged KV cache and the activations resident in HBM behind the
// C ABI of include/memvanta_b200.h (mv_model_*).
//
// A caller swaps `LlamaModel` for `CudaLlamaModel` and keeps its code: the
// same constructor arguments, forward / prefill returning the host logits
// vector, generate with the caller's Sampler, reset / position /
// kv_bytes_allocated.  The GGUF file and its tokenizer are also opened on the
// host (the reference's own GgufFile / GgufTokenizer), so gguf() and
// tokenizer() keep working.  `threads` is accepted and only reported back.
// Errors surface as std::runtime_error, as the reference throws them.
#pragma once

#include <cstddef>
#include <string>
#include <vector>

#include "memvanta/gguf.hpp"
#include "memvanta/llama_model.hpp"

struct mv_model_s;

namespace memvanta {

class CudaLlamaModel {
public:
    CudaLlamaModel(const std::string& gguf_path, unsigned threads = 1, std::size_t ctx_override = 0,
                   std::size_t kv_page_tokens = 128, KVCacheType kv_type = KVCacheType::F16);
    ~CudaLlamaModel();
    CudaLlamaModel(const CudaLlamaModel&) = delete;
    CudaLlamaModel& operator=(const CudaLlamaModel&) = delete;

    const LlamaConfig& config() const { return c_; }
    const GgufFile& gguf() const { return file_; }
    const GgufTokenizer& tokenizer() const { return tok_; }
    void reset();
    const std::vector<float>& forward(int token, bool compute_logits = true);
    const std::vector<float>& prefill(const std::vector<int>& tokens, std::size_t batch_size = 64,
                                      bool compute_logits_last = true);
    std::vector<int> generate(const std::vector<int>& prompt, std::size_t n, Sampler& sampler);
    std::size_t position() const;
    std::size_t kv_bytes_allocated() const;
    unsigned threads() const { return threads_; }
    KVCacheType kv_type() const { return kv_type_; }

private:
    GgufFile file_;
    GgufTokenizer tok_;
    LlamaConfig c_;
    unsigned threads_;
    KVCacheType kv_type_;
    mv_model_s* m_ = nullptr;
    std::vector<float> logits_;
};

}  // namespace memvanta
