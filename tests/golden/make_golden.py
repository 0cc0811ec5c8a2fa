"""Generate the golden fixtures in this directory from the reference itself.

Run in a checkout where oracle/_ref/libmvref.so was built from the reference
sources (``make -C oracle``):

    python tests/golden/make_golden.py

Every array below is an output of the reference's own code (tensor_matvec,
tensor_matmul_batch_v06 with and without MEMVANTA_FORCE_Q8_ACT, the internal
quantize_q8 / dot_q4_q8_block / q6_k_value helpers, PagedKVCache and
LlamaModel) on seeded inputs that are stored next to it, so the fixtures pin
the oracle and the CUDA path without needing the reference at test time.

Kernel calls use threads=2: GCC compiles the reference's single-thread call
path (the row lambda inlined into tensor_matvec) without FMA-contracting the
row sum and its multi-thread path with it, so the two differ in the last bit
of some rows; the oracle restates the multi-thread build.
"""
from __future__ import annotations

import hashlib
import os
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from oracle import Reference, KV_F32, KV_F16, KV_Q8  # noqa: E402
from memvanta_b200 import gguf  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))

# Tiny llama used by the end-to-end fixture: GQA (2 q heads, 1 kv head),
# head_dim 128, Q4_0 layers, Q6_K head.
TINY = gguf.LlamaShape(n_layer=2, n_embd=256, n_head=2, n_head_kv=1, n_ff=512, vocab=256, n_ctx=256,
                       rms_eps=1e-6, rope_theta=10000.0)
TINY_SEED = 77


def sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def fp16_cases(R: Reference):
    rng = np.random.default_rng(11)
    mags = 10.0 ** rng.uniform(-9, 5.5, 4000)
    x = (rng.standard_normal(4000) * mags).astype(np.float32)
    edge = np.array([0.0, -0.0, 1.0, -1.0, 65504.0, 65519.0, 65520.0, 70000.0, 6.1035156e-05, 5.9604645e-08,
                     2.9802322e-08, 2.98e-08, 1e-10, 0.5, 1.0009766, 1.00048828125, 1.000732421875,
                     float("inf"), -float("inf"), 3.0517578e-05], dtype=np.float32)
    x = np.concatenate([edge, x])
    h = np.array([R.fp32_to_fp16(float(v)) for v in x], dtype=np.uint16)
    np.savez_compressed(os.path.join(OUT, "fp16_cases.npz"), x=x, h=h)


def quant_q8(R: Reference):
    rng = np.random.default_rng(12)
    x = rng.standard_normal((4, 1024)).astype(np.float32)
    x[0, :32] = 0.0                                   # all-zero block -> d = 1
    x[1, :32] = np.arange(32, dtype=np.float32) - 15.5  # half-way ties
    x[2, 32:64] *= 1e6
    x[3, 64:96] = 127.0 * 0.5 / 127.0                 # constant block
    qs, ds = [], []
    for r in range(4):
        q, d = R.quantize_q8(x[r])
        qs.append(q)
        ds.append(d)
    np.savez_compressed(os.path.join(OUT, "quant_q8.npz"), x=x, q=np.stack(qs), d=np.stack(ds))


def blocks(R: Reference):
    rng = np.random.default_rng(13)
    b4 = gguf.gen_q4_0(1, 32 * 64, rng).reshape(64, 18)
    aq = rng.integers(-127, 128, size=(64, 32), dtype=np.int8)
    aq[0] = 127
    aq[1] = -127
    b4[0, 2:] = 0x00
    b4[1, 2:] = 0xFF
    isum = np.array([R.dot_q4_q8_block(b4[i], aq[i]) for i in range(64)], dtype=np.int32)
    b6 = gguf.gen_q6_k(1, 256 * 4, rng).reshape(4, 210)
    q6 = np.array([[R.q6_k_value(b6[i], j) for j in range(256)] for i in range(4)], dtype=np.int32)
    np.savez_compressed(os.path.join(OUT, "blocks.npz"), q4=b4, aq=aq, isum=isum, q6k=b6, q6=q6)


def gemv(R: Reference, tmp: str):
    rng = np.random.default_rng(14)
    cases = {}
    for key, t, rows, cols in [("q4_0", gguf.Q4_0, 96, 1024), ("q4_0_k11008", gguf.Q4_0, 8, 11008),
                               ("q8_0", gguf.Q8_0, 64, 1024), ("q6_k", gguf.Q6_K, 48, 1024),
                               ("f16", gguf.F16, 32, 512), ("f32", gguf.F32, 32, 512)]:
        w = gguf.gen_blocks(t, rows, cols, rng)
        x = rng.standard_normal(cols).astype(np.float32)
        X = rng.standard_normal((11 if cols <= 1024 else 3, cols)).astype(np.float32)
        path = os.path.join(tmp, f"{key}.gguf")
        name = "blk.0.ffn_gate.weight"
        gguf.write_single_tensor(path, name, t, rows, cols, w)
        h = R.open(path)
        cases[f"{key}_w"] = w
        cases[f"{key}_meta"] = np.array([t, rows, cols], dtype=np.int64)
        cases[f"{key}_x"] = x
        cases[f"{key}_y"] = R.matvec(h, name, x, rows, threads=2)
        cases[f"{key}_X"] = X
        cases[f"{key}_Y"] = R.matmul_batch_v06(h, name, X, rows, threads=2)  # default fp32-activation prefill
        cases[f"{key}_Yq8"] = R.matmul_batch_v06(h, name, X, rows, threads=2, force_q8=True)
        cases[f"{key}_row5"] = R.read_row(h, name, 5, cols)
        R.close(h)
    np.savez_compressed(os.path.join(OUT, "gemv.npz"), **cases)


def kv_attention(R: Reference):
    """Decode attention through the reference PagedKVCache (src/llama_model.cpp:256)."""
    rng = np.random.default_rng(15)
    n_head, n_head_kv, hd, page, n_ctx = 4, 2, 128, 16, 37
    kv_dim = n_head_kv * hd
    K = rng.standard_normal((n_ctx, kv_dim)).astype(np.float32)
    V = rng.standard_normal((n_ctx, kv_dim)).astype(np.float32)
    q = rng.standard_normal(n_head * hd).astype(np.float32)
    out = {}
    for kvt, tag in [(KV_F32, "f32"), (KV_F16, "f16"), (KV_Q8, "q8")]:
        c = R.kv_new(kv_dim, page, kvt)
        for t in range(n_ctx):
            R.kv_write(c, t, K[t], V[t])
        group = n_head // n_head_kv
        att = np.zeros(n_head * hd, np.float32)
        root = np.float32(np.sqrt(np.float32(hd)))
        for h in range(n_head):
            kb, qb = (h // group) * hd, h * hd
            s = np.array([np.float32(R.kv_dot_key(c, t, kb, q[qb:qb + hd])) / root for t in range(n_ctx)],
                         dtype=np.float32)
            m = s.max()
            e = np.exp(s - m).astype(np.float32)
            den = float(np.sum(e.astype(np.float64)))
            inv = np.float32(1.0 / den)
            o = np.zeros(hd, np.float32)
            for t in range(n_ctx):
                R.kv_add_value(c, t, kb, float(np.float32(e[t] * inv)), o)
            att[qb:qb + hd] = o
        R.kv_free(c)
        out[f"{tag}_att"] = att
    np.savez_compressed(os.path.join(OUT, "kv_attention.npz"), K=K, V=V, q=q,
                        meta=np.array([n_head, n_head_kv, hd, page, n_ctx]), **out)


def tiny_model(R: Reference, tmp: str):
    path = os.path.join(tmp, "tiny.gguf")
    gguf.write_random_llama(path, TINY, seed=TINY_SEED)
    rng = np.random.default_rng(16)
    prompt = rng.integers(0, TINY.vocab, size=45).astype(np.int32)
    res = {"prompt": prompt, "sha256": np.array(sha256(path))}
    for fq in (0, 1):
        m = R.model_open(path, threads=2, ctx=128, page=16, kv_type=KV_F16)
        res[f"prefill_logits_q{fq}"] = R.model_prefill(m, prompt, batch=8, compute_logits=True, force_q8=bool(fq))
        cur = int(np.argmax(res[f"prefill_logits_q{fq}"]))
        toks, logits = [], []
        for _ in range(12):
            l = R.model_forward(m, cur, True, force_q8=bool(fq))
            logits.append(l)
            cur = int(np.argmax(l))
            toks.append(cur)
        res[f"decode_logits_q{fq}"] = np.stack(logits)
        res[f"decode_tokens_q{fq}"] = np.array(toks, dtype=np.int32)
        R.model_free(m)
    np.savez_compressed(os.path.join(OUT, "tiny_model.npz"), **res)


def main():
    R = Reference()
    with tempfile.TemporaryDirectory() as tmp:
        fp16_cases(R)
        quant_q8(R)
        blocks(R)
        gemv(R, tmp)
        kv_attention(R)
        tiny_model(R, tmp)
    for f in sorted(os.listdir(OUT)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(OUT, f)))


if __name__ == "__main__":
    main()
