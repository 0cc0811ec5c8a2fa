// gguf_kernels_cuda.cpp -- the reference-side binding: a drop-in replacement
// for MemVanta's src/gguf_kernels.cpp that routes its public kernel API
// (include/memvanta/gguf_kernels.hpp) to the B200 library through the C ABI
// in include/memvanta_b200.h.
//
// Build it into memvanta_core instead of src/gguf_kernels.cpp and link
// libmemvanta_b200.so; LlamaModel, the benches and the tests then run their
// matmuls on the GPU through their own, unchanged call sites.
//
// Semantics kept from the reference: host pointers in and out, y fully
// overwritten, synchronous, std::runtime_error on the same conditions
// (rank < 2, misaligned rows, unsupported types), the per-tensor profiler.
// The `threads` / `pool` arguments are accepted and ignored.  Weights are
// uploaded to HBM on first use and cached per (file, tensor offset).
#include "memvanta/gguf_kernels.hpp"

#include <atomic>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "memvanta_b200.h"

namespace memvanta {
namespace {

using Clock = std::chrono::steady_clock;

void check(int rc, const std::string& what) {
    if (rc != MV_OK) throw std::runtime_error(what + ": " + mv_last_error());
}

// One device copy per (GgufFile, tensor offset).
mv_weight_t device_weight(const GgufFile& file, const GgufTensor& t) {
    static std::mutex mu;
    static std::map<std::pair<const GgufFile*, std::uint64_t>, mv_weight_t> cache;
    static bool ready = false;
    std::lock_guard<std::mutex> lock(mu);
    if (!ready) {
        check(mv_init(0), "mv_init");
        ready = true;
    }
    auto key = std::make_pair(&file, t.offset);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    mv_weight_t w = nullptr;
    check(mv_weight_upload(file.tensor_data(t), t.nbytes, static_cast<int>(t.type), t.ne(1), t.ne(0), nullptr, &w),
          "upload " + t.name);
    cache.emplace(key, w);
    return w;
}

std::atomic<bool> g_profile_enabled{false};
std::mutex g_profile_mu;
std::vector<KernelProfileEntry> g_profile_entries;

KernelProfileKind classify(const std::string& n) {
    if (n.find(".attn_q.") != std::string::npos) return KernelProfileKind::QProj;
    if (n.find(".attn_k.") != std::string::npos) return KernelProfileKind::KProj;
    if (n.find(".attn_v.") != std::string::npos) return KernelProfileKind::VProj;
    if (n.find(".attn_output.") != std::string::npos) return KernelProfileKind::OProj;
    if (n.find(".ffn_gate.") != std::string::npos) return KernelProfileKind::FfnGate;
    if (n.find(".ffn_up.") != std::string::npos) return KernelProfileKind::FfnUp;
    if (n.find(".ffn_down.") != std::string::npos) return KernelProfileKind::FfnDown;
    if (n == "output.weight") return KernelProfileKind::Output;
    return KernelProfileKind::Other;
}

int layer_of(const std::string& n) {
    if (n.rfind("blk.", 0) != 0) return -1;
    const auto p = n.find('.', 4);
    if (p == std::string::npos) return -1;
    try {
        return std::stoi(n.substr(4, p - 4));
    } catch (...) {
        return -1;
    }
}

void profile(const GgufTensor& t, std::size_t batch, Clock::time_point t0) {
    if (!g_profile_enabled.load(std::memory_order_relaxed)) return;
    const double ms = std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
    KernelProfileEntry e{layer_of(t.name), classify(t.name), t.name, 1, batch, ms};
    std::lock_guard<std::mutex> lock(g_profile_mu);
    for (auto& x : g_profile_entries)
        if (x.layer == e.layer && x.kind == e.kind && x.tensor == e.tensor && x.batch == e.batch) {
            x.calls += 1;
            x.ms += ms;
            return;
        }
    g_profile_entries.push_back(std::move(e));
}

void require_matrix(const GgufTensor& t, const char* what) {
    if (t.dims.size() < 2) throw std::runtime_error(std::string(what) + " requires rank-2 tensor: " + t.name);
}

}  // namespace

void enable_kernel_profiling(bool on) { g_profile_enabled.store(on, std::memory_order_relaxed); }
void reset_kernel_profile() {
    std::lock_guard<std::mutex> lock(g_profile_mu);
    g_profile_entries.clear();
}
std::vector<KernelProfileEntry> kernel_profile_snapshot() {
    std::lock_guard<std::mutex> lock(g_profile_mu);
    return g_profile_entries;
}
const char* kernel_profile_kind_name(KernelProfileKind k) {
    switch (k) {
        case KernelProfileKind::QProj: return "q_proj";
        case KernelProfileKind::KProj: return "k_proj";
        case KernelProfileKind::VProj: return "v_proj";
        case KernelProfileKind::OProj: return "o_proj";
        case KernelProfileKind::FfnGate: return "ffn_gate";
        case KernelProfileKind::FfnUp: return "ffn_up";
        case KernelProfileKind::FfnDown: return "ffn_down";
        case KernelProfileKind::Output: return "output";
        case KernelProfileKind::Other: return "other";
    }
    return "other";
}

void tensor_matvec(const GgufFile& file, const GgufTensor& t, const float* x, float* y, unsigned, WorkerPool*) {
    const auto t0 = Clock::now();
    require_matrix(t, "matvec");
    check(mv_tensor_matvec_host(device_weight(file, t), x, y), "tensor_matvec " + t.name);
    profile(t, 1, t0);
}

void tensor_matmul_batch(const GgufFile& file, const GgufTensor& t, const float* x, float* y, std::size_t batch,
                         unsigned, WorkerPool*) {
    const auto t0 = Clock::now();
    require_matrix(t, "matmul batch");
    check(mv_tensor_matmul_batch_host(device_weight(file, t), x, y, batch, MV_ACT_F32), "tensor_matmul_batch " + t.name);
    profile(t, batch, t0);
}

void tensor_matmul_batch_v06(const GgufFile& file, const GgufTensor& t, const float* x, float* y, std::size_t batch,
                             unsigned, WorkerPool*) {
    const auto t0 = Clock::now();
    require_matrix(t, "hybrid GEMM");
    const char* e = std::getenv("MEMVANTA_FORCE_Q8_ACT");
    const int act = (e && *e == '1') ? MV_ACT_Q8 : MV_ACT_F32;
    check(mv_tensor_matmul_batch_host(device_weight(file, t), x, y, batch, act), "tensor_matmul_batch_v06 " + t.name);
    profile(t, batch, t0);
}

void tensor_read_row_f32(const GgufFile& file, const GgufTensor& t, std::size_t row, float* out, std::size_t cols) {
    if (t.dims.size() < 2 || t.ne(0) != cols || row >= t.ne(1))
        throw std::runtime_error("tensor row shape mismatch: " + t.name);
    check(mv_tensor_read_row_host(device_weight(file, t), row, out), "tensor_read_row_f32 " + t.name);
}

// Small host-side helpers of the same header, unchanged in meaning.
void tensor_vector_to_f32(const GgufFile& file, const GgufTensor& t, float* out, std::size_t n) {
    if (t.elements() != n) throw std::runtime_error("tensor vector size mismatch: " + t.name);
    const std::byte* p = file.tensor_data(t);
    if (t.type == GgmlType::F32) {
        std::memcpy(out, p, n * sizeof(float));
        return;
    }
    if (t.type == GgmlType::F16) {
        const auto* q = reinterpret_cast<const std::uint16_t*>(p);
        for (std::size_t i = 0; i < n; ++i) out[i] = fp16_to_fp32(q[i]);
        return;
    }
    throw std::runtime_error("unsupported vector tensor type " + ggml_type_name(t.type) + ": " + t.name);
}

float dot_f32_simd(const float* a, const float* b, std::size_t n) {
    // eight fma lanes summed left to right: the reference's AVX2 order
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    std::size_t i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; ++l) acc[l] = __builtin_fmaf(a[i + l], b[i + l], acc[l]);
    float s = acc[0];
    for (int l = 1; l < 8; ++l) s += acc[l];
    for (; i < n; ++i) s = __builtin_fmaf(a[i], b[i], s);
    return s;
}

void axpy_f32_simd(float alpha, const float* x, float* y, std::size_t n) {
    for (std::size_t i = 0; i < n; ++i) y[i] = __builtin_fmaf(alpha, x[i], y[i]);
}

std::uint16_t fp32_to_fp16(float f) {
    // round-half-up on the magnitude, as the reference's KV cache stores halves
    std::uint32_t x;
    std::memcpy(&x, &f, 4);
    const std::uint32_t sign = (x >> 16) & 0x8000u;
    std::uint32_t mant = x & 0x7fffffu;
    const int e = static_cast<int>((x >> 23) & 0xffu) - 112;
    if (e >= 31) return static_cast<std::uint16_t>(sign | 0x7c00u);
    if (e > 0) return static_cast<std::uint16_t>(sign | (static_cast<std::uint32_t>(e) << 10) | ((mant + 0x1000u) >> 13));
    if (e < -10) return static_cast<std::uint16_t>(sign);
    mant = (mant | 0x800000u) >> (1 - e);
    return static_cast<std::uint16_t>(sign + ((mant + 0x1000u) >> 13));
}

}  // namespace memvanta
