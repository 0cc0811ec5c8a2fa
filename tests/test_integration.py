"""The reference-side binding (memvanta_b200/bindings/gguf_kernels_cuda.cpp)
compiles against the reference's own headers and links against the library:
a maintainer can swap it in for src/gguf_kernels.cpp.  CPU only."""
from __future__ import annotations

import os
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("MV_REFERENCE_DIR", "/root/reference")
BINDING = os.path.join(ROOT, "memvanta_b200", "bindings", "gguf_kernels_cuda.cpp")


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "include", "memvanta")), reason="reference checkout absent")
def test_binding_links_with_reference_sources():
    srcs = [os.path.join(REF, "src", f) for f in
            ("gguf.cpp", "mmap_file.cpp", "worker_pool.cpp", "llama_model.cpp")]
    lib_dir = os.path.join(ROOT, "memvanta_b200")
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "libmemvanta_core_cuda.so")
        cmd = ["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-I", os.path.join(REF, "include"),
               "-I", os.path.join(ROOT, "include"), BINDING, *srcs, "-L", lib_dir, "-lmemvanta_b200",
               f"-Wl,-rpath,{lib_dir}", "-Wl,--no-undefined", "-pthread", "-o", out]
        r = subprocess.run(cmd, capture_output=True, text=True)
        assert r.returncode == 0, r.stderr[-2000:]
        # the reference's kernel API is now provided by the binding
        nm = subprocess.run(["nm", "-DC", "--defined-only", out], capture_output=True, text=True).stdout
        for sym in ("memvanta::tensor_matvec", "memvanta::tensor_matmul_batch_v06", "memvanta::tensor_read_row_f32",
                    "memvanta::LlamaModel::forward"):
            assert sym in nm, sym


MODEL_BINDING = os.path.join(ROOT, "memvanta_b200", "bindings", "llama_model_cuda.cpp")

# A caller written against the reference's LlamaModel, with the class swapped:
# the same constructor, prefill / forward / generate / reset / position calls.
CONSUMER = r"""
#include <cstdio>
#include <stdexcept>
#include "llama_model_cuda.hpp"
int main(int argc, char** argv) {
    try {
        memvanta::CudaLlamaModel model(argv[1], 4, 256, 16, memvanta::KVCacheType::F16);
        const auto& logits = model.prefill({1, 2, 3, 4, 5}, 32, true);
        memvanta::Sampler greedy;
        auto toks = model.generate({1, 2, 3}, 4, greedy);
        model.forward(toks.back(), true);
        std::printf("ran %zu %zu %zu\n", logits.size(), model.position(), model.kv_bytes_allocated());
        return 0;
    } catch (const std::runtime_error& e) {
        std::printf("runtime_error: %s\n", e.what());
        return 3;
    }
}
"""


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "include", "memvanta")), reason="reference checkout absent")
def test_model_binding_is_a_drop_in_for_llama_model():
    """memvanta_b200/bindings/llama_model_cuda.cpp compiles against the
    reference's headers, links with its sources and the library, and a caller
    written against LlamaModel's interface builds with CudaLlamaModel in its
    place.  Without a GPU the constructor reports the failure as the
    reference reports errors: a std::runtime_error, not a crash."""
    import sys
    sys.path.insert(0, ROOT)
    from memvanta_b200 import gguf
    srcs = [os.path.join(REF, "src", f) for f in
            ("gguf.cpp", "mmap_file.cpp", "worker_pool.cpp", "llama_model.cpp")]
    lib_dir = os.path.join(ROOT, "memvanta_b200")
    inc = ["-I", os.path.join(REF, "include"), "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(ROOT, "memvanta_b200", "bindings")]
    with tempfile.TemporaryDirectory() as d:
        core = os.path.join(d, "libmemvanta_model_cuda.so")
        r = subprocess.run(["g++", "-std=c++20", "-O1", "-fPIC", "-shared", *inc, MODEL_BINDING, BINDING, *srcs,
                            "-L", lib_dir, "-lmemvanta_b200", f"-Wl,-rpath,{lib_dir}", "-Wl,--no-undefined",
                            "-pthread", "-o", core], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr[-2000:]
        nm = subprocess.run(["nm", "-DC", "--defined-only", core], capture_output=True, text=True).stdout
        for sym in ("memvanta::CudaLlamaModel::forward", "memvanta::CudaLlamaModel::prefill",
                    "memvanta::CudaLlamaModel::generate", "memvanta::CudaLlamaModel::reset"):
            assert sym in nm, sym
        src = os.path.join(d, "consumer.cpp")
        with open(src, "w") as f:
            f.write(CONSUMER)
        exe = os.path.join(d, "consumer")
        r = subprocess.run(["g++", "-std=c++20", "-O1", *inc, src, core, f"-Wl,-rpath,{d}", f"-Wl,-rpath,{lib_dir}",
                            "-pthread", "-o", exe], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr[-2000:]
        path = os.path.join(d, "tiny.gguf")
        gguf.write_random_llama(path, gguf.LlamaShape(n_layer=1, n_embd=256, n_head=4, n_head_kv=4, n_ff=512,
                                                       vocab=512, n_ctx=256, rms_eps=1e-6, rope_theta=10000.0),
                                seed=3)
        run = subprocess.run([exe, path], capture_output=True, text=True, timeout=120)
        import torch
        if torch.cuda.is_available():
            assert run.returncode == 0 and run.stdout.startswith("ran 512 "), run.stdout + run.stderr
        else:
            assert run.returncode == 3 and "mv_init" in run.stdout, run.stdout + run.stderr
