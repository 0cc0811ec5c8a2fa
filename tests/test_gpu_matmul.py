"""Parity of the CUDA matmul path (through the C ABI) with the oracle and the
reference's golden outputs.

Bar (stated per test): per-block int32 dots bit-exact; Q8 activation
quantisation bit-exact; matmul outputs within
|y - ref| <= tol * max(|ref|, rms(ref)) with tol 1e-3 (Q4_0, Q8_0, F16, F32)
and 5e-3 (Q6_K).
"""
from __future__ import annotations

import numpy as np
import pytest

import memvanta_b200 as mv
from memvanta_b200 import gguf
from conftest import rel_err

pytestmark = pytest.mark.gpu

TOL = {gguf.Q4_0: 1e-3, gguf.Q8_0: 1e-3, gguf.F16: 1e-3, gguf.F32: 1e-3, gguf.Q6_K: 5e-3}


def dev(a, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def upload(w, t, rows, cols):
    return mv.Weight.upload(w, t, rows, cols)


def run_gemv(W, x, cuda):
    import torch
    y = torch.empty(W.rows, dtype=torch.float32, device=cuda)
    mv.gemv(W, dev(x, cuda), y)
    return host(y)


def run_gemm(W, X, cuda, act):
    import torch
    Y = torch.empty((X.shape[0], W.rows), dtype=torch.float32, device=cuda)
    mv.gemm(W, dev(X, cuda), Y, act)
    return host(Y)


# ---------------------------------------------------------------- layout

@pytest.mark.parametrize("t,rows,cols", [(gguf.Q4_0, 37, 4096), (gguf.Q8_0, 5, 1024), (gguf.Q6_K, 9, 512),
                                         (gguf.F16, 7, 96), (gguf.F32, 3, 100)])
def test_repack_roundtrip(cuda, t, rows, cols):
    rng = np.random.default_rng(t * 7 + rows)
    w = gguf.gen_blocks(t, rows, cols, rng)
    W = upload(w, t, rows, cols)
    assert np.array_equal(W.download(), w)
    info = W.info()
    assert (info["type"], info["rows"], info["cols"]) == (t, rows, cols)


# ----------------------------------------------------- bit-exact pieces

def test_quantize_q8_golden_bit_exact(cuda, golden):
    g = golden("quant_q8.npz")
    q, d = mv.quantize_q8(dev(g["x"], cuda))
    assert np.array_equal(host(q), g["q"])
    assert np.array_equal(host(d).view(np.uint32), g["d"].view(np.uint32))


def test_quantize_q8_edge_values(cuda, oracle):
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((3, 4096)) * rng.choice([1e-30, 1e-3, 1.0, 1e30], (3, 4096))).astype(np.float32)
    x[0, :64] = 0.0
    x[1, :32] = np.float32(127.0) * (np.arange(32, dtype=np.float32) - 15.5) / np.float32(16.0)   # ties
    x[2, 32:64] = -np.finfo(np.float32).tiny
    q, d = mv.quantize_q8(dev(x, cuda))
    qo, do = oracle.quantize_q8(x)
    assert np.array_equal(host(q), qo)
    assert np.array_equal(host(d).view(np.uint32), do.view(np.uint32))


def test_q4_block_dots_bit_exact(cuda, oracle, golden):
    """Every 32-element block's int32 dot equals the reference's dot_q4_q8_block."""
    rng = np.random.default_rng(6)
    rows, cols = 48, 4096
    w = gguf.gen_q4_0(rows, cols, rng)
    w[:18 * 3] = 0                                    # zero blocks, zero scales
    x = rng.standard_normal(cols).astype(np.float32)
    x[64:96] = 0.0
    W = upload(w, gguf.Q4_0, rows, cols)
    got = host(mv.q4_0_block_dots(W, dev(x, cuda)))
    q, _ = oracle.quantize_q8(x)
    blk = w.reshape(rows, cols // 32, 18)
    want = np.array([[oracle.dot_q4_q8_block(blk[r, b], q[32 * b:32 * b + 32]) for b in range(cols // 32)]
                     for r in range(rows)], dtype=np.int32)
    assert np.array_equal(got, want)
    # the golden per-block cases (extreme nibbles and activations)
    g = golden("blocks.npz")
    for i in range(8):
        Wb = upload(g["q4"][i], gguf.Q4_0, 1, 32)
        xa = g["aq"][i].astype(np.float32)
        qa, _ = oracle.quantize_q8(xa)
        assert host(mv.q4_0_block_dots(Wb, dev(xa, cuda)))[0, 0] == oracle.dot_q4_q8_block(g["q4"][i], qa)


def test_read_row_golden(cuda, golden):
    g = golden("gemv.npz")
    for key in ["q4_0", "q8_0", "q6_k", "f16", "f32"]:
        t, rows, cols = (int(v) for v in g[f"{key}_meta"])
        W = upload(g[f"{key}_w"], t, rows, cols)
        assert np.array_equal(mv.tensor_read_row_f32(W, 5).view(np.uint32), g[f"{key}_row5"].view(np.uint32)), key


# ------------------------------------------------------ golden matmuls

GEMV_KEYS = ["q4_0", "q4_0_k11008", "q8_0", "q6_k", "f16", "f32"]


@pytest.mark.parametrize("key", GEMV_KEYS)
def test_gemv_golden(cuda, golden, key):
    g = golden("gemv.npz")
    t, rows, cols = (int(v) for v in g[f"{key}_meta"])
    W = upload(g[f"{key}_w"], t, rows, cols)
    assert rel_err(run_gemv(W, g[f"{key}_x"], cuda), g[f"{key}_y"]) <= TOL[t]
    # the reference's host-pointer contract gives the same numbers
    assert np.array_equal(mv.tensor_matvec(W, g[f"{key}_x"]), run_gemv(W, g[f"{key}_x"], cuda))


@pytest.mark.parametrize("key", GEMV_KEYS)
def test_gemm_golden(cuda, golden, key):
    g = golden("gemv.npz")
    t, rows, cols = (int(v) for v in g[f"{key}_meta"])
    W = upload(g[f"{key}_w"], t, rows, cols)
    X = g[f"{key}_X"]
    assert rel_err(run_gemm(W, X, cuda, mv.ACT_Q8), g[f"{key}_Yq8"]) <= TOL[t]
    assert rel_err(run_gemm(W, X, cuda, mv.ACT_F32), g[f"{key}_Y"]) <= TOL[t]
    assert rel_err(mv.tensor_matmul_batch_v06(W, X, force_q8=True), g[f"{key}_Yq8"]) <= TOL[t]


# ------------------------------------------------- BASELINE-size parity

def test_config0_q4_gemv_full(cuda, oracle):
    """Config 0: W 4096x4096 Q4_0 (|N(0,0.02)| scales, uniform nibbles), x ~ N(0,1)."""
    rng = np.random.default_rng(1234)
    w = gguf.gen_q4_0(4096, 4096, rng)
    x = rng.standard_normal(4096).astype(np.float32)
    W = upload(w, gguf.Q4_0, 4096, 4096)
    assert rel_err(run_gemv(W, x, cuda), oracle.matvec(gguf.Q4_0, w, 4096, 4096, x)) <= 1e-3


@pytest.mark.parametrize("rows,cols", [(1, 32), (3, 64), (17, 4096), (11008, 4096), (4096, 11008), (5, 352)])
def test_q4_gemv_shapes(cuda, oracle, rows, cols):
    rng = np.random.default_rng(rows * 31 + cols)
    w = gguf.gen_q4_0(rows, cols, rng)
    x = rng.standard_normal(cols).astype(np.float32)
    W = upload(w, gguf.Q4_0, rows, cols)
    assert rel_err(run_gemv(W, x, cuda), oracle.matvec(gguf.Q4_0, w, rows, cols, x)) <= 1e-3


@pytest.mark.parametrize("rows,cols,batch", [(11008, 4096, 32), (4096, 11008, 32), (512, 4096, 128),
                                             (256, 4096, 512), (64, 128, 3), (33, 4096, 9)])
def test_config1_q4_gemm_q8act(cuda, oracle, rows, cols, batch):
    """Config 1 shapes (full weights at B=32; row-sampled at B=128/512 to keep
    the CPU oracle within seconds): Q8 activations vs MEMVANTA_FORCE_Q8_ACT."""
    rng = np.random.default_rng(rows + cols + batch)
    w = gguf.gen_q4_0(rows, cols, rng)
    X = rng.standard_normal((batch, cols)).astype(np.float32)
    W = upload(w, gguf.Q4_0, rows, cols)
    want = oracle.matmul_batch_v06(gguf.Q4_0, w, rows, cols, X, force_q8=True)
    got = run_gemm(W, X, cuda, mv.ACT_Q8)
    assert rel_err(got, want) <= 1e-3
    # the tensor-core GEMM keeps the reference's per-output FMA chain: bit-exact
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def _sms():
    import torch
    return torch.cuda.get_device_properties(0).multi_processor_count


@pytest.mark.parametrize("tile,cols", [("n8", 160), ("n8", 672), ("n16", 160), ("n16", 672), ("n32", 4096),
                                       ("n32b", 672), ("n32b", 1056), ("split", 672), ("split", 4096)])
def test_tc_gemm_tile_widths_bit_exact(cuda, oracle, tile, cols):
    """Every tile width of the tensor-core GEMM (8 tokens on a 16-wide MMA,
    16 and 32 tokens), with block counts that end in a partial pipeline stage
    (nb = 5, 21, 33) and partial row and token tiles; bit-exact against the
    FORCE_Q8 chain.  The shapes make the launcher's wave model pick the width:
    8 tokens for few row tiles (n8), 16 for a little over one row tile per SM
    (n16), 32 for one row tile per SM at 32 and 128 tokens (n32, n32b), and
    for a single token tile over more row tiles than SMs two launches: one
    32-token tile per SM, then the remaining rows in 8-token tiles (split)."""
    sms = _sms()
    rows, batch = {"n8": (300, 70), "n16": (128 * sms + 200, 70), "n32": (128 * sms, 32),
                   "n32b": (128 * sms - 5, 128), "split": (128 * sms + 200, 20)}[tile]
    rng = np.random.default_rng(cols + batch)
    w = gguf.gen_q4_0(rows, cols, rng)
    X = rng.standard_normal((batch, cols)).astype(np.float32)
    W = upload(w, gguf.Q4_0, rows, cols)
    got = run_gemm(W, X, cuda, mv.ACT_Q8)
    mv.stream_status()
    want = oracle.matmul_batch_v06(gguf.Q4_0, w, rows, cols, X, force_q8=True)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("tile", ["nt128", "nt64", "nt32"])
def test_f16_gemm_tile_widths_bit_exact(cuda, oracle, tile):
    """Every token-tile width of the fp16 tensor-core GEMM (64 tokens and
    more), bit-exact against the FORCE_Q8 chain: the launcher's wave model
    takes 128-token tiles when one tile per SM already fills the machine
    (148 row tiles, 128 tokens), 64 at 64 tokens, and 32 for a narrow weight
    (3 row tiles at 100 tokens, ragged rows and tokens)."""
    sms = _sms()
    rows, batch, cols = {"nt128": (128 * sms - 37, 128, 512), "nt64": (128 * sms - 5, 64, 512),
                         "nt32": (300, 100, 1056)}[tile]
    rng = np.random.default_rng(rows + batch)
    w = gguf.gen_q4_0(rows, cols, rng)
    X = rng.standard_normal((batch, cols)).astype(np.float32)
    W = upload(w, gguf.Q4_0, rows, cols)
    got = run_gemm(W, X, cuda, mv.ACT_Q8)
    mv.stream_status()
    want = oracle.matmul_batch_v06(gguf.Q4_0, w, rows, cols, X, force_q8=True)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("batch", [20, 80])
def test_tc_gemm_edge_values(cuda, oracle, batch):
    """Extreme blocks: nibbles all 0 or all 15, activations of one sign at the
    Q8 clamp, zero rows/tokens, a negative fp16 scale -- bit-exact, on the int8
    tensor-core GEMM (20 tokens) and the fp16 one (80 tokens)."""
    rng = np.random.default_rng(77)
    rows, cols = 136, 256
    w = gguf.gen_q4_0(rows, cols, rng).reshape(rows, cols // 32, 18).copy()
    w[0, :, 2:] = 0x00                       # every nibble 0  -> q - 8 = -8
    w[1, :, 2:] = 0xFF                       # every nibble 15 -> q - 8 = 7
    w[2, :, :2] = 0                          # zero scales
    w[3, :, :2] = np.frombuffer(np.float16(-0.03).tobytes(), np.uint8)
    w = w.reshape(-1)
    X = rng.standard_normal((batch, cols)).astype(np.float32)
    X[0] = 1e4
    X[1] = -1e-4
    X[2] = 0.0
    X[3, ::2] = 3.0
    X[3, 1::2] = -3.0
    W = upload(w, gguf.Q4_0, rows, cols)
    got = run_gemm(W, X, cuda, mv.ACT_Q8)
    want = oracle.matmul_batch_v06(gguf.Q4_0, w, rows, cols, X, force_q8=True)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_stream_status_clean(cuda):
    """After normal tensor-core work the bounded-wait status word is clear."""
    rng = np.random.default_rng(5)
    w = gguf.gen_q4_0(256, 512, rng)
    W = upload(w, gguf.Q4_0, 256, 512)
    run_gemm(W, rng.standard_normal((40, 512)).astype(np.float32), cuda, mv.ACT_Q8)
    mv.stream_status()


@pytest.mark.parametrize("stage", [0, 5])
def test_tc_gemm_wait_runs_out_then_next_call_is_clean(cuda, oracle, stage):
    """A bounded wait that runs out, made on purpose through the test hook:
    the fp16 tensor-core GEMM leaves out one stage's MMA commit, so the
    epilogue, converters and producer stop getting that stage; with a 20 ms
    bound one of their waits gives up, every role drains and returns, and
    mv_stream_status reports MV_ERR_TIMEOUT (no fault, the context stays
    usable).  The next launch, without the hook, is bit-exact again."""
    rng = np.random.default_rng(900 + stage)
    rows, cols, batch = 1024, 2048, 96
    w = gguf.gen_q4_0(rows, cols, rng)
    X = rng.standard_normal((batch, cols)).astype(np.float32)
    W = upload(w, gguf.Q4_0, rows, cols)
    mv.stream_status()
    mv.test_gemm_stall(stage, 20000)
    run_gemm(W, X, cuda, mv.ACT_Q8)
    with pytest.raises(mv.MemVantaError) as e:
        mv.stream_status()
    assert e.value.code == mv.MV_ERR_TIMEOUT
    got = run_gemm(W, X, cuda, mv.ACT_Q8)
    mv.stream_status()
    want = oracle.matmul_batch_v06(gguf.Q4_0, w, rows, cols, X, force_q8=True)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_config2_q8_0_and_q6_k(cuda, oracle):
    """Config 2: Q8_0 4096x4096 and a Q6_K 32000x4096 head, batch 1 and 32."""
    rng = np.random.default_rng(2)
    w8 = gguf.gen_q8_0(4096, 4096, rng)
    x = rng.standard_normal(4096).astype(np.float32)
    W8 = upload(w8, gguf.Q8_0, 4096, 4096)
    assert rel_err(run_gemv(W8, x, cuda), oracle.matvec(gguf.Q8_0, w8, 4096, 4096, x)) <= 1e-3
    X = rng.standard_normal((32, 4096)).astype(np.float32)
    assert rel_err(run_gemm(W8, X, cuda, mv.ACT_Q8), oracle.matmul_batch_v06(gguf.Q8_0, w8, 4096, 4096, X, True)) <= 1e-3
    w6 = gguf.gen_q6_k(32000, 4096, rng)
    W6 = upload(w6, gguf.Q6_K, 32000, 4096)
    assert rel_err(run_gemv(W6, x, cuda), oracle.matvec(gguf.Q6_K, w6, 32000, 4096, x)) <= 5e-3
    sub = w6[: 2000 * 16 * 210]                       # B=32 on 2000 rows keeps the oracle fast
    W6s = upload(sub, gguf.Q6_K, 2000, 4096)
    assert rel_err(run_gemm(W6s, X, cuda, mv.ACT_Q8), oracle.matmul_batch(gguf.Q6_K, sub, 2000, 4096, X)) <= 5e-3


def test_zero_and_extreme_inputs(cuda, oracle):
    rng = np.random.default_rng(9)
    w = gguf.gen_q4_0(64, 1024, rng)
    W = upload(w, gguf.Q4_0, 64, 1024)
    x = np.zeros(1024, np.float32)
    assert np.array_equal(run_gemv(W, x, cuda), np.zeros(64, np.float32))
    x = (rng.standard_normal(1024) * 1e4).astype(np.float32)
    assert rel_err(run_gemv(W, x, cuda), oracle.matvec(gguf.Q4_0, w, 64, 1024, x)) <= 1e-3


# ------------------------------------------------------------- errors

def test_error_paths(cuda):
    rng = np.random.default_rng(10)
    w = gguf.gen_q4_0(4, 64, rng)
    with pytest.raises(mv.MemVantaError, match="UNSUPPORTED"):
        mv.Weight.upload(w, 3, 4, 64)                  # Q4_1: the reference cannot matvec it either
    for kq, bb in ((12, 144), (13, 176)):             # Q4_K / Q5_K: sized by the loader, no kernel
        with pytest.raises(mv.MemVantaError, match="UNSUPPORTED"):  # (src/gguf_kernels.cpp:251 throws too)
            mv.Weight.upload(np.zeros(4 * bb, np.uint8), kq, 4, 256)
    with pytest.raises(mv.MemVantaError, match="INVALID"):
        mv.Weight.upload(w[:-1], gguf.Q4_0, 4, 64)     # nbytes mismatch
    with pytest.raises(mv.MemVantaError, match="not block aligned"):
        mv.Weight.upload(np.zeros(4 * 48 * 4, np.uint8), gguf.Q4_0, 4, 48)
    W = upload(w, gguf.Q4_0, 4, 64)
    with pytest.raises(mv.MemVantaError, match="out of range"):
        mv.tensor_read_row_f32(W, 4)
    import torch
    with pytest.raises(mv.MemVantaError, match="multiple of 32"):
        mv.quantize_q8(torch.zeros(40, device=cuda))
    # the library still works after the errors
    assert np.array_equal(W.download(), w)
