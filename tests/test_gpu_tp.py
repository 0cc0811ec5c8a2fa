"""Tensor-parallel LlamaModel (mv_model_open_tp): the model split over 2 or 4
GPUs, one spawned process per rank, must return the single-GPU model's
results bit for bit -- prefill logits (int8 tensor-core GEMMs and the fp32
B=1 path), decode logits and device-side greedy tokens -- for the fused F16
and the Q8_0 KV caches.  A rank that stops calling makes the others fail
with MV_ERR_TIMEOUT after a bounded wait instead of hanging.

The ranks exchange only their peer-memory handles over a gloo group on
127.0.0.1; NVLS is switched off in the children's environment (the library
uses plain peer stores, never multicast).
"""
from __future__ import annotations

import multiprocessing as mp
import os
import socket
import tempfile
import traceback

import numpy as np
import pytest

from memvanta_b200 import gguf

pytestmark = pytest.mark.gpu

SHAPE = gguf.LlamaShape(n_layer=3, n_embd=1024, n_head=8, n_head_kv=4, n_ff=2816, vocab=4096, n_ctx=512,
                        rms_eps=1e-6, rope_theta=10000.0)
PROMPT = [int(t) for t in np.random.default_rng(5).integers(3, 4096, size=75)]
N_DECODE = 6
N_GREEDY = 16


def _gpus() -> int:
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _plan(m, kv_type):
    """The calls every arm makes, in order; returns the results."""
    out = {}
    out["prefill"] = m.prefill(PROMPT, batch_size=32).copy()  # chunks 32, 32, 11 merged into one batch of 75
    cur = int(np.argmax(out["prefill"]))
    dec = []
    for _ in range(N_DECODE):
        l = m.forward(cur).copy()
        dec.append(l)
        cur = int(np.argmax(l))
    out["decode"] = np.stack(dec)
    out["greedy"] = m.generate_greedy(cur, N_GREEDY).copy()
    m.reset()
    out["prefill_b1"] = m.prefill(PROMPT[:9], batch_size=1).copy()  # fp32-activation path
    out["position"] = np.array([m.position()])
    return out


def _single(path, kv_type, outdir):
    try:
        import memvanta_b200 as mv

        mv.init(0)
        m = mv.LlamaModel(path, ctx_override=256, kv_page_tokens=16, kv_type=kv_type)
        np.savez(os.path.join(outdir, "single.npz"), **_plan(m, kv_type))
        m.close()
    except Exception:
        with open(os.path.join(outdir, "single.err"), "w") as f:
            f.write(traceback.format_exc())


def _rank(rank, world, port, path, kv_type, outdir, mode):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import torch.distributed as dist

        import memvanta_b200 as mv

        dist.init_process_group("gloo", rank=rank, world_size=world)
        m = mv.LlamaModel.tensor_parallel(path, device=rank, ctx_override=256, kv_page_tokens=16, kv_type=kv_type,
                                          prefill_batch=128)  # the 75-token prompt merges into one fp16-GEMM batch
        if mode == "parity":
            np.savez(os.path.join(outdir, f"rank{rank}.npz"), **_plan(m, kv_type))
        else:  # failure: rank 1 skips one step; rank 0's step must give up, not hang
            m.set_timeout(500)
            m.prefill(PROMPT[:8], batch_size=8)
            rc = 0
            if rank == 0:
                try:
                    m.forward(PROMPT[8])
                except mv.MemVantaError as e:
                    rc = e.code
            np.savez(os.path.join(outdir, f"rank{rank}.npz"), rc=np.array([rc]))
        m.close()
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(outdir, f"rank{rank}.err"), "w") as f:
            f.write(traceback.format_exc())


def _spawn(target, args_list, timeout=300):
    ctx = mp.get_context("spawn")
    ps = [ctx.Process(target=target, args=a) for a in args_list]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout)
    alive = [p for p in ps if p.is_alive()]
    for p in alive:
        p.kill()
        p.join()
    assert not alive, "a rank did not finish"


def _errors(outdir):
    errs = [f for f in os.listdir(outdir) if f.endswith(".err")]
    return "\n".join(open(os.path.join(outdir, f)).read() for f in errs)


@pytest.fixture(scope="module")
def model_path():
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "tp.gguf")
        gguf.write_random_llama(p, SHAPE, seed=31)
        yield p


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("kv_type", [1, 3], ids=["kv_f16", "kv_q8_0"])
def test_tensor_parallel_bit_exact(model_path, world, kv_type):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    with tempfile.TemporaryDirectory() as outdir:
        _spawn(_single, [(model_path, kv_type, outdir)])
        port = _free_port()
        _spawn(_rank, [(r, world, port, model_path, kv_type, outdir, "parity") for r in range(world)])
        assert not _errors(outdir), _errors(outdir)
        ref = np.load(os.path.join(outdir, "single.npz"))
        for r in range(world):
            got = np.load(os.path.join(outdir, f"rank{r}.npz"))
            for k in ref.files:
                assert np.array_equal(got[k], ref[k]), (r, k)


def test_tensor_parallel_rank_that_stops_gives_timeout(model_path):
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    with tempfile.TemporaryDirectory() as outdir:
        port = _free_port()
        _spawn(_rank, [(r, 2, port, model_path, 1, outdir, "failure") for r in range(2)])
        assert not _errors(outdir), _errors(outdir)
        assert int(np.load(os.path.join(outdir, "rank0.npz"))["rc"][0]) == 6  # MV_ERR_TIMEOUT
