"""Host side of the tensor-parallel model on CPU (gloo, world size 2): every
rank learns that a rank could not open its share and raises, instead of
waiting for a handle that never comes.  Without a GPU, mv_init fails on
every rank, which is the failure exercised here."""
from __future__ import annotations

import multiprocessing as mp
import os
import socket
import tempfile
import traceback

import pytest

from memvanta_b200 import gguf


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, port, path, outdir):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import torch.distributed as dist

        import memvanta_b200 as mv

        dist.init_process_group("gloo", rank=rank, world_size=2)
        try:
            mv.LlamaModel.tensor_parallel(path, device=rank, ctx_override=64)
            res = "opened"
        except RuntimeError as e:
            res = "raised: " + str(e)
        dist.barrier()
        dist.destroy_process_group()
        with open(os.path.join(outdir, f"rank{rank}.txt"), "w") as f:
            f.write(res)
    except Exception:
        with open(os.path.join(outdir, f"rank{rank}.txt"), "w") as f:
            f.write("error: " + traceback.format_exc())


def test_open_failure_reaches_every_rank():
    import torch

    if torch.cuda.is_available():
        pytest.skip("exercises the no-GPU failure path")
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m.gguf")
        gguf.write_random_llama(path, gguf.LlamaShape(n_layer=1, n_embd=256, n_head=2, n_head_kv=2, n_ff=512,
                                                      vocab=64, n_ctx=64), seed=3)
        port = _free_port()
        ctx = mp.get_context("spawn")
        ps = [ctx.Process(target=_rank, args=(r, port, path, d)) for r in range(2)]
        for p in ps:
            p.start()
        for p in ps:
            p.join(120)
        alive = [p for p in ps if p.is_alive()]
        for p in alive:
            p.kill()
            p.join()
        assert not alive, "a rank hung"
        for r in range(2):
            res = open(os.path.join(d, f"rank{r}.txt")).read()
            assert res.startswith("raised: tensor-parallel open failed on rank(s)"), res
            assert "(0," in res and "(1," in res, res
