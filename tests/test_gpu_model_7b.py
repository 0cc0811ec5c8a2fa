"""Config 3 end to end at full size: the random-init OpenLLaMA-7B-shaped Q4_0
Llama (32 layers, d 4096, 32 heads x 128, ffn 11008, vocab 32000, Q6_K head,
F16 paged KV with 16-token pages, ctx 768) against the reference's own
LlamaModel (oracle/_ref, built from the unmodified sources), on the bench's
512-token prompt.

Bar: logits within 2e-2 max-abs, greedy tokens
identical for the first 32 generated tokens.  The prefill runs in batches of
32 (LlamaModel::prefill, src/llama_model.cpp:260) with the reference in its
MEMVANTA_FORCE_Q8_ACT=1 numerics (the int8 prefill GEMM's); decode is
LlamaModel::forward (src/llama_model.cpp:253-259) from position 512, every
step's logits compared.  The reference needs ~30 s of host CPU for this.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

import memvanta_b200 as mv
from memvanta_b200 import gguf

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-2
CTX, PAGE, PROMPT, BATCH, GEN = 768, 16, 512, 32, 32
GGUF_PATH = os.environ.get("MV_BENCH_GGUF", "/tmp/memvanta_b200_rand7b_seed1234.gguf")


def prompt_ids(n, vocab=32000):
    """The bench's prompt ids, (i*1543+17) % vocab -- the reference bench's
    (benchmarks/real_model_bench.cpp:18)."""
    return ((np.arange(n) * 1543 + 17) % vocab).astype(np.int32)


@pytest.fixture(scope="module")
def model_7b():
    if not os.path.exists(GGUF_PATH):
        tmp = GGUF_PATH + f".tmp{os.getpid()}"
        gguf.write_random_llama(tmp, gguf.LLAMA_7B, seed=1234)
        os.replace(tmp, GGUF_PATH)
    return GGUF_PATH


@pytest.fixture(scope="module")
def reference_7b(reference, model_7b):
    """The reference's prefill logits, then GEN greedy steps (logits, tokens)."""
    threads = max(2, len(os.sched_getaffinity(0)))  # the multi-threaded build's numerics
    r = reference.model_open(model_7b, threads=threads, ctx=CTX, page=PAGE, kv_type=mv.KV_F16)
    try:
        pl = reference.model_prefill(r, prompt_ids(PROMPT), batch=BATCH, compute_logits=True, force_q8=True)
        cur, toks, logits = int(np.argmax(pl)), [], []
        for _ in range(GEN):
            lg = reference.model_forward(r, cur, True)
            logits.append(lg)
            cur = int(np.argmax(lg))
            toks.append(cur)
        return pl.copy(), np.stack(logits), toks
    finally:
        reference.model_free(r)


def test_config3_7b_prefill_and_decode_vs_reference(cuda, model_7b, reference_7b):
    pl_ref, lg_ref, tok_ref = reference_7b
    m = mv.LlamaModel(model_7b, ctx_override=CTX, kv_page_tokens=PAGE, kv_type=mv.KV_F16)
    try:
        pl = m.prefill(prompt_ids(PROMPT), batch_size=BATCH).copy()
        err = float(np.max(np.abs(pl - pl_ref)))
        assert err <= LOGIT_TOL, ("prefill logits", err)
        cur, toks = int(np.argmax(pl)), []
        for i in range(GEN):
            lg = m.forward(cur)
            err = float(np.max(np.abs(lg - lg_ref[i])))
            assert err <= LOGIT_TOL, ("decode step", i, err)
            cur = int(np.argmax(lg))
            toks.append(cur)
        assert toks == tok_ref
        # the device-side greedy loop (the timed tg path) gives the same tokens
        m.reset()
        pl2 = m.prefill(prompt_ids(PROMPT), batch_size=BATCH)
        assert np.array_equal(pl2, pl)
        assert list(m.generate_greedy(int(np.argmax(pl2)), GEN)) == tok_ref
    finally:
        m.close()
