// llama_model_cuda.cpp -- memvanta::CudaLlamaModel (see llama_model_cuda.hpp):
// MemVanta's LlamaModel interface on the device-resident model of
// libmemvanta_b200 (mv_model_* in include/memvanta_b200.h).
#include "llama_model_cuda.hpp"

#include <algorithm>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "memvanta_b200.h"

namespace memvanta {
namespace {

void check(int rc, const std::string& what) {
    if (rc != MV_OK) throw std::runtime_error(what + ": " + mv_last_error());
}

// KVCacheType {F32, F16, Q8} (include/memvanta/llama_model.hpp:28) onto the
// library's cache types; Q8 is the reference's per-token-scale int8 cache.
int kv_code(KVCacheType t) {
    switch (t) {
        case KVCacheType::F32: return MV_KV_F32;
        case KVCacheType::F16: return MV_KV_F16;
        case KVCacheType::Q8: return MV_KV_Q8;
    }
    throw std::runtime_error("unsupported KV cache type");
}

}  // namespace

CudaLlamaModel::CudaLlamaModel(const std::string& gguf_path, unsigned threads, std::size_t ctx_override,
                               std::size_t kv_page_tokens, KVCacheType kv_type)
    : file_(gguf_path), tok_(file_), threads_(std::max(1u, threads)), kv_type_(kv_type) {
    check(mv_init(0), "mv_init");
    check(mv_model_open(gguf_path.c_str(), ctx_override, kv_page_tokens, kv_code(kv_type), &m_), "mv_model_open");
    std::uint64_t cfg[7] = {};
    check(mv_model_config(m_, cfg), "mv_model_config");
    c_.n_ctx = cfg[0];
    c_.n_embd = cfg[1];
    c_.n_ff = cfg[2];
    c_.n_layer = cfg[3];
    c_.n_head = cfg[4];
    c_.n_head_kv = cfg[5];
    c_.vocab = cfg[6];
    // the same metadata keys and defaults as LlamaModel::load_config (src/llama_model.cpp:226)
    c_.rms_eps = static_cast<float>(file_.get_f64("llama.attention.layer_norm_rms_epsilon").value_or(1e-5));
    c_.rope_theta = static_cast<float>(file_.get_f64("llama.rope.freq_base").value_or(10000.0));
    logits_.assign(c_.vocab, 0.0f);
}

CudaLlamaModel::~CudaLlamaModel() {
    if (m_) mv_model_close(m_);
}

void CudaLlamaModel::reset() { check(mv_model_reset(m_), "reset"); }

std::size_t CudaLlamaModel::position() const { return static_cast<std::size_t>(mv_model_position(m_)); }

std::size_t CudaLlamaModel::kv_bytes_allocated() const { return static_cast<std::size_t>(mv_model_kv_bytes(m_)); }

// LlamaModel::forward (src/llama_model.cpp:253-259): without logits the
// previous logits vector is returned unchanged, as the reference does.
const std::vector<float>& CudaLlamaModel::forward(int token, bool compute_logits) {
    check(mv_model_forward(m_, token, compute_logits ? 1 : 0, compute_logits ? logits_.data() : nullptr), "forward");
    return logits_;
}

// LlamaModel::prefill (src/llama_model.cpp:260): chunks of batch_size tokens,
// logits of the last token only.
const std::vector<float>& CudaLlamaModel::prefill(const std::vector<int>& tokens, std::size_t batch_size,
                                                  bool compute_logits_last) {
    if (tokens.empty()) return logits_;
    std::vector<std::int32_t> ids(tokens.begin(), tokens.end());
    check(mv_model_prefill(m_, ids.data(), ids.size(), std::max<std::size_t>(1, batch_size),
                           compute_logits_last ? 1 : 0, compute_logits_last ? logits_.data() : nullptr),
          "prefill");
    return logits_;
}

// LlamaModel::generate (src/llama_model.cpp:261): reset, prefill all but the
// last prompt token in chunks of 64, then forward + the caller's sampler per
// token, stopping after the tokenizer's end-of-sequence id.
std::vector<int> CudaLlamaModel::generate(const std::vector<int>& prompt, std::size_t n, Sampler& sampler) {
    reset();
    if (prompt.empty()) throw std::runtime_error("prompt cannot be empty");
    if (prompt.size() > 1) prefill(std::vector<int>(prompt.begin(), prompt.end() - 1), 64, false);
    int cur = prompt.back();
    std::vector<int> out;
    out.reserve(n);
    for (std::size_t i = 0; i < n; ++i) {
        const int next = sampler.sample(forward(cur, true));
        out.push_back(next);
        cur = next;
        if (next == tok_.eos_id()) break;
    }
    return out;
}

}  // namespace memvanta
