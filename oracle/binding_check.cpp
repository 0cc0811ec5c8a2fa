// binding_check.cpp -- TEST INFRASTRUCTURE ONLY (built into oracle/_ref by
// oracle/Makefile, run by tests/test_gpu_model.py).  Opens one GGUF twice:
// with the reference's own memvanta::LlamaModel (its CPU kernels, compiled
// from the unmodified MemVanta sources) and with memvanta::CudaLlamaModel
// (memvanta_b200/bindings/llama_model_cuda.cpp, the device-resident model),
// and checks that the swapped class gives the reference's results through the
// reference's own interface: prefill logits within 2e-2 max-abs, identical
// greedy tokens from generate(), equal position() and kv_bytes_allocated().
// The reference's prefill runs with MEMVANTA_FORCE_Q8_ACT=1, the numerics the
// device prefill follows.  Exit code 0: all equal; 1: a mismatch; 3: an error
// (e.g. no GPU).  Usage: binding_check <model.gguf> <vocab>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include "llama_model_cuda.hpp"
int main(int argc, char** argv) {
    setenv("MEMVANTA_FORCE_Q8_ACT", "1", 1);
    try {
        memvanta::LlamaModel ref(argv[1], 8, 256, 16, memvanta::KVCacheType::F16);
        memvanta::CudaLlamaModel gpu(argv[1], 8, 256, 16, memvanta::KVCacheType::F16);
        std::vector<int> prompt;
        const int vocab = argc > 2 ? std::atoi(argv[2]) : 512;
        for (int i = 0; i < 40; ++i) prompt.push_back((i * 1543 + 17) % vocab);
        auto a = ref.prefill(prompt, 16, true);
        auto b = gpu.prefill(prompt, 16, true);
        double md = 0;
        for (size_t i = 0; i < a.size(); ++i) md = std::fmax(md, std::fabs(a[i] - b[i]));
        memvanta::Sampler s1, s2;
        auto ta = ref.generate(prompt, 24, s1);
        auto tb = gpu.generate(prompt, 24, s2);
        std::printf("prefill maxdiff %.3g tokens %zu %zu equal %d pos %zu %zu kv %zu %zu\n", md, ta.size(), tb.size(),
                    int(ta == tb), ref.position(), gpu.position(), ref.kv_bytes_allocated(), gpu.kv_bytes_allocated());
        return (ta == tb && md <= 2e-2) ? 0 : 1;
    } catch (const std::exception& e) {
        std::printf("exception: %s\n", e.what());
        return 3;
    }
}
