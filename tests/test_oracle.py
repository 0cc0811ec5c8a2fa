"""The oracle (oracle/mv_oracle.c) pinned against the reference.

1. Golden fixtures (tests/golden/*.npz, produced by the reference's own code
   by tests/golden/make_golden.py) -- always run, no reference needed.
2. Fresh seeded comparisons with the reference build (oracle/_ref) -- run
   wherever that build exists.
Both demand bit-exact agreement: the oracle restates the reference's
evaluation order and its compiler's FMA contractions.
"""
from __future__ import annotations

import os
import tempfile

import numpy as np
import pytest

from memvanta_b200 import gguf


def bits(a):
    return np.asarray(a, dtype=np.float32).view(np.uint32)


# ------------------------------------------------------------ golden

def test_golden_fp16(oracle, golden):
    g = golden("fp16_cases.npz")
    got = oracle.fp32_to_fp16_array(g["x"])
    assert np.array_equal(got, g["h"])


def test_golden_fp16_to_fp32_exhaustive(oracle):
    h = np.arange(65536, dtype=np.uint16)
    got = np.array([oracle.fp16_to_fp32(int(v)) for v in h], dtype=np.float32)
    want = h.view(np.float16).astype(np.float32)   # IEEE half -> float is exact
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(bits(got)[~nan], bits(want)[~nan])


def test_golden_quant_q8(oracle, golden):
    g = golden("quant_q8.npz")
    q, d = oracle.quantize_q8(g["x"])
    assert np.array_equal(q, g["q"])
    assert np.array_equal(bits(d), bits(g["d"]))
    assert (g["d"][0, 0] == 1.0)                    # all-zero block -> scale 1


def test_golden_blocks(oracle, golden):
    g = golden("blocks.npz")
    for i in range(g["q4"].shape[0]):
        assert oracle.dot_q4_q8_block(g["q4"][i], g["aq"][i]) == g["isum"][i]
    for i in range(g["q6k"].shape[0]):
        assert [oracle.q6_k_value(g["q6k"][i], j) for j in range(256)] == list(g["q6"][i])


GEMV_KEYS = ["q4_0", "q4_0_k11008", "q8_0", "q6_k", "f16", "f32"]


@pytest.mark.parametrize("key", GEMV_KEYS)
def test_golden_matmuls(oracle, golden, key):
    g = golden("gemv.npz")
    t, rows, cols = (int(v) for v in g[f"{key}_meta"])
    w = g[f"{key}_w"]
    assert np.array_equal(bits(oracle.matvec(t, w, rows, cols, g[f"{key}_x"])), bits(g[f"{key}_y"]))
    X = g[f"{key}_X"]
    assert np.array_equal(bits(oracle.matmul_batch_v06(t, w, rows, cols, X, ffn=True)), bits(g[f"{key}_Y"]))
    assert np.array_equal(bits(oracle.matmul_batch_v06(t, w, rows, cols, X, force_q8=True, ffn=True)),
                          bits(g[f"{key}_Yq8"]))
    assert np.array_equal(bits(oracle.read_row(t, w, rows, cols, 5)), bits(g[f"{key}_row5"]))


def test_golden_kv_attention(oracle, golden):
    """Oracle paged attention vs the reference's PagedKVCache dot/add loop.
    The fixture's softmax exponent ran in numpy, so agreement is to float
    rounding rather than bit-exact."""
    g = golden("kv_attention.npz")
    n_head, n_head_kv, hd, page, n_ctx = (int(v) for v in g["meta"])
    kv_dim = n_head_kv * hd
    n_pages = (n_ctx + page - 1) // page
    table = np.arange(n_pages, dtype=np.int32)
    for kvt, tag in [(0, "f32"), (1, "f16"), (2, "q8")]:
        rb = oracle.kv_row_bytes(kvt, kv_dim)
        ns = oracle.kv_row_scales(kvt, kv_dim)
        kp = np.zeros((n_pages * page, rb), np.uint8)
        vp = np.zeros((n_pages * page, rb), np.uint8)
        ks = np.zeros((n_pages * page, max(ns, 1)), np.float32)
        vs = np.zeros((n_pages * page, max(ns, 1)), np.float32)
        for t in range(n_ctx):
            kp[t], s1 = oracle.kv_store(kvt, g["K"][t])
            vp[t], s2 = oracle.kv_store(kvt, g["V"][t])
            ks[t, :ns], vs[t, :ns] = s1, s2
        out = oracle.attn_decode(kvt, g["q"], n_head, n_head_kv, hd, kp, vp, ks if ns else None, vs if ns else None,
                                 table, page, n_ctx)
        np.testing.assert_allclose(out, g[f"{tag}_att"], rtol=2e-5, atol=2e-6)


# ------------------------------------------------- against the reference

@pytest.fixture(scope="module")
def tmpdir_mod():
    with tempfile.TemporaryDirectory() as d:
        yield d


def test_ref_fp16_random(oracle, reference):
    rng = np.random.default_rng(21)
    x = (rng.standard_normal(3000) * 10.0 ** rng.uniform(-9, 5.5, 3000)).astype(np.float32)
    assert all(oracle.fp32_to_fp16(float(v)) == reference.fp32_to_fp16(float(v)) for v in x)


@pytest.mark.parametrize("t,rows,cols", [(gguf.Q4_0, 256, 4096), (gguf.Q4_0, 64, 11008), (gguf.Q8_0, 256, 4096),
                                         (gguf.Q6_K, 128, 4096), (gguf.F16, 64, 1024), (gguf.F32, 64, 1000)])
def test_ref_matmuls_bit_exact(oracle, reference, tmpdir_mod, t, rows, cols):
    rng = np.random.default_rng(1000 + t + cols)
    w = gguf.gen_blocks(t, rows, cols, rng)
    path = os.path.join(tmpdir_mod, f"w{t}_{cols}.gguf")
    name = "blk.3.ffn_up.weight"
    gguf.write_single_tensor(path, name, t, rows, cols, w)
    h = reference.open(path)
    try:
        x = rng.standard_normal(cols).astype(np.float32)
        assert np.array_equal(bits(reference.matvec(h, name, x, rows, threads=3)),
                              bits(oracle.matvec(t, w, rows, cols, x)))
        X = rng.standard_normal((9, cols)).astype(np.float32)
        for fq in (False, True):
            assert np.array_equal(bits(reference.matmul_batch_v06(h, name, X, rows, threads=3, force_q8=fq)),
                                  bits(oracle.matmul_batch_v06(t, w, rows, cols, X, force_q8=fq, ffn=True)))
        assert np.array_equal(bits(reference.matmul_batch(h, name, X[:3], rows)),
                              bits(oracle.matmul_batch(t, w, rows, cols, X[:3])))
    finally:
        reference.close(h)


def test_ref_quant_and_blocks(oracle, reference):
    rng = np.random.default_rng(22)
    x = (rng.standard_normal(8192) * rng.choice([1e-3, 1.0, 1e3], 8192)).astype(np.float32)
    x[:32] = 0.0
    q1, d1 = oracle.quantize_q8(x)
    q2, d2 = reference.quantize_q8(x)
    assert np.array_equal(q1, q2) and np.array_equal(bits(d1), bits(d2))
    blk = gguf.gen_q4_0(1, 32 * 200, rng).reshape(200, 18)
    for i in range(200):
        assert oracle.dot_q4_q8_block(blk[i], q1[32 * i:32 * i + 32]) == reference.dot_q4_q8_block(blk[i], q1[32 * i:32 * i + 32])


def _ref_attention(reference, c, q, n_head, n_head_kv, hd, n_ctx):
    """The reference's decode attention loop (src/llama_model.cpp:256) driven
    through its PagedKVCache::dot_key / add_value."""
    group = n_head // n_head_kv
    root = np.float32(np.sqrt(np.float32(hd)))
    att = np.zeros(n_head * hd, np.float32)
    for h in range(n_head):
        kb, qb = (h // group) * hd, h * hd
        s = np.array([np.float32(reference.kv_dot_key(c, t, kb, q[qb:qb + hd])) / root for t in range(n_ctx)],
                     dtype=np.float32)
        e = np.exp(s - s.max()).astype(np.float32)
        inv = np.float32(1.0 / float(np.sum(e.astype(np.float64))))
        o = np.zeros(hd, np.float32)
        for t in range(n_ctx):
            reference.kv_add_value(c, t, kb, float(np.float32(e[t] * inv)), o)
        att[qb:qb + hd] = o
    return att


@pytest.mark.parametrize("kvt", [0, 1, 2])
def test_ref_kv_attention(oracle, reference, kvt):
    """Oracle kv_store + paged attention vs PagedKVCache write/dot_key/add_value
    with a scattered block table on the oracle side."""
    rng = np.random.default_rng(23 + kvt)
    n_head, n_head_kv, hd, page, n_ctx = 4, 2, 128, 16, 41
    kv_dim = n_head_kv * hd
    c = reference.kv_new(kv_dim, page, kvt)
    try:
        K = rng.standard_normal((n_ctx, kv_dim)).astype(np.float32)
        V = rng.standard_normal((n_ctx, kv_dim)).astype(np.float32)
        q = rng.standard_normal(n_head * hd).astype(np.float32)
        for t in range(n_ctx):
            reference.kv_write(c, t, K[t], V[t])
        want = _ref_attention(reference, c, q, n_head, n_head_kv, hd, n_ctx)
    finally:
        reference.kv_free(c)
    n_pages = (n_ctx + page - 1) // page
    table = rng.permutation(n_pages + 3)[:n_pages].astype(np.int32)   # scattered physical pages
    rb, ns = oracle.kv_row_bytes(kvt, kv_dim), oracle.kv_row_scales(kvt, kv_dim)
    kp = np.zeros(((n_pages + 3) * page, rb), np.uint8)
    vp = np.zeros_like(kp)
    ks = np.zeros(((n_pages + 3) * page, max(ns, 1)), np.float32)
    vs = np.zeros_like(ks)
    for t in range(n_ctx):
        slot = table[t // page] * page + t % page
        kp[slot], s1 = oracle.kv_store(kvt, K[t])
        vp[slot], s2 = oracle.kv_store(kvt, V[t])
        ks[slot, :ns], vs[slot, :ns] = s1, s2
    got = oracle.attn_decode(kvt, q, n_head, n_head_kv, hd, kp, vp, ks if ns else None, vs if ns else None, table,
                             page, n_ctx)
    np.testing.assert_allclose(got, want, rtol=2e-5, atol=2e-6)


def test_ref_internal_formats(oracle, reference):
    rng = np.random.default_rng(24)
    rows, cols = 64, 1024
    A = rng.uniform(-1, 1, (rows, cols)).astype(np.float32)
    A[0, :32] = 0.0
    x = rng.uniform(-1, 1, cols).astype(np.float32)
    a4o, a4r = oracle.int_quantize_q4_0(A), reference.int_quantize_q4_0(A)
    a8o, a8r = oracle.int_quantize_q8_0(A), reference.int_quantize_q8_0(A)
    assert np.array_equal(a4o, a4r) and np.array_equal(a8o, a8r)
    x8 = oracle.int_quantize_q8_0(x)
    assert np.array_equal(bits(oracle.int_matvec_q4_q8(a4o, x8, rows, cols)),
                          bits(reference.int_matvec_q4_q8(a4r, x8, rows, cols, threads=2)))
    assert np.array_equal(bits(oracle.int_matvec_q4_0(a4o, x, rows, cols)),
                          bits(reference.int_matvec_q4_0(a4r, x, rows, cols, threads=2)))
    assert np.array_equal(bits(oracle.int_matvec_q8_0(a8o, x, rows, cols)),
                          bits(reference.int_matvec_q8_0(a8r, x, rows, cols, threads=2)))
    X = rng.uniform(-1, 1, (5, cols)).astype(np.float32)
    assert np.array_equal(bits(oracle.int_matmul_q4_0_batch(a4o, X, rows, cols)),
                          bits(reference.int_matmul_q4_0_batch(a4r, X, rows, cols, threads=2)))
    assert np.array_equal(bits(oracle.matvec_f32(A, x)), bits(reference.matvec_f32(A, x, threads=2)))
