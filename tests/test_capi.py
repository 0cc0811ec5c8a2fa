"""CPU-side checks of the C ABI and host logic (no device calls)."""
from __future__ import annotations

import ctypes as C
import os
import re
import subprocess
import tempfile

import numpy as np
import pytest

from memvanta_b200 import _lib, gguf

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "memvanta_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^MV_API\s+[\w\s\*]+?\b(mv_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "mv_gemv" in syms and "mv_gemm" in syms and "mv_model_forward" in syms
    assert len(syms) >= 30


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (mv_\w+)", out))
    assert set(declared_symbols()) <= exported
    # nothing but the ABI leaks out of the library
    assert all(s.startswith("mv_") for s in exported)


def test_python_signatures_cover_header():
    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_library_is_built_for_sm100a_only():
    """The build names one target, sm_100a, in every compile and the link."""
    mk = open(os.path.join(os.path.dirname(_lib.LIB_PATH), "csrc", "Makefile")).read()
    arch = re.search(r"^ARCH := (.*)$", mk, re.M).group(1).strip()
    assert arch == "-gencode arch=compute_100a,code=sm_100a"
    assert "-gencode" not in mk.replace(arch, "")
    assert "$(NVCC) $(NVFLAGS) -c" in mk and "$(NVCC) $(ARCH) -shared" in mk


@pytest.mark.gpu
def test_loaded_device_code_is_sm100(cuda):
    """At run time the kernels the driver loaded are sm_100 code
    (cudaFuncGetAttributes' binaryVersion, through mv_binary_arch)."""
    v = C.c_int(0)
    assert _lib.load().mv_binary_arch(C.byref(v)) == 0
    assert v.value == 100


def test_pure_host_entry_points():
    lib = _lib.load()
    assert lib.mv_version() >= 1
    assert lib.mv_kv_row_bytes(_lib.KV_F16, 4096) == 8192
    assert lib.mv_kv_row_bytes(_lib.KV_Q8, 4096) == 4096
    assert lib.mv_kv_row_scales(_lib.KV_Q8, 4096) == 1
    assert lib.mv_kv_row_scales(_lib.KV_Q8_0, 4096) == 128


def test_gguf_writer_reader_roundtrip():
    rng = np.random.default_rng(3)
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "t.gguf")
        w4 = gguf.gen_q4_0(8, 64, rng)
        w6 = gguf.gen_q6_k(4, 256, rng)
        n = gguf.write_gguf(p, [("general.architecture", "llama"), ("x.f", 1.5), ("x.s", ["a", "b"])],
                            [gguf.TensorSpec("a", [64, 8], gguf.Q4_0, w4), gguf.TensorSpec("b", [256, 4], gguf.Q6_K, w6)])
        assert os.path.getsize(p) == n
        meta, infos = gguf.read_tensor_infos(p)
        assert meta["general.architecture"] == "llama" and meta["x.s"] == ["a", "b"]
        raw = open(p, "rb").read()
        a, b = infos
        assert (a.rows, a.cols, a.ggml_type) == (8, 64, gguf.Q4_0) and a.offset % 32 == 0
        assert raw[a.offset:a.offset + a.nbytes] == w4.tobytes()
        assert raw[b.offset:b.offset + b.nbytes] == w6.tobytes()


def test_generators_follow_config_distributions():
    rng = np.random.default_rng(4)
    w = gguf.gen_q4_0(64, 4096, rng).reshape(-1, 18)
    d = w[:, :2].copy().view(np.float16).astype(np.float32).ravel()
    assert (d >= 0).all() and abs(np.mean(d) - 0.02 * np.sqrt(2 / np.pi)) < 1e-3
    nib = np.concatenate([w[:, 2:] & 15, w[:, 2:] >> 4]).ravel()
    assert nib.min() == 0 and nib.max() == 15 and abs(nib.mean() - 7.5) < 0.05
    q6 = gguf.gen_q6_k(16, 4096, rng).reshape(-1, 210)
    sc = q6[:, 192:208].view(np.int8)
    assert sc.min() == -32 and sc.max() == 31
