"""The reference-side binding (memvanta_b200/bindings/gguf_kernels_cuda.cpp)
compiles against the reference's own headers and links against the library:
a maintainer can swap it in for src/gguf_kernels.cpp.  CPU only."""
from __future__ import annotations

import os
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = "/root/reference"
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
