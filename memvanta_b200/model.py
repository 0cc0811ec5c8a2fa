"""LlamaModel: the device-resident decoder behind the C ABI (mv_model_*).

Mirrors the reference's public class (include/memvanta/llama_model.hpp:100-113):
``LlamaModel(path, threads, ctx, page_tokens, kv_type)``, ``forward``,
``prefill``, ``generate``, ``reset``, ``position``, ``kv_bytes_allocated``.
``threads`` is accepted for signature compatibility and ignored (the GPU
parallelises internally).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from ._lib import KV_F16, check, load

HANDLE_BYTES = 64  # MV_TP_HANDLE_BYTES


class LlamaModel:
    tp_rank, tp_world, _group = 0, 1, None

    def __init__(self, gguf_path: str | os.PathLike, threads: int = 1, ctx_override: int = 0,
                 kv_page_tokens: int = 128, kv_type: int = KV_F16):
        self._m = None
        h = C.c_void_p()
        check(load().mv_model_open(os.fspath(gguf_path).encode(), ctx_override, kv_page_tokens, kv_type,
                                   C.byref(h)))
        self._m = h
        self._read_config()

    def _read_config(self) -> None:
        cfg = (C.c_uint64 * 7)()
        check(load().mv_model_config(self._m, cfg))
        self.n_ctx, self.n_embd, self.n_ff, self.n_layer, self.n_head, self.n_head_kv, self.vocab = list(cfg)
        self._logits = np.empty(self.vocab, np.float32)

    @classmethod
    def tensor_parallel(cls, gguf_path: str | os.PathLike, group=None, device: int | None = None,
                        ctx_override: int = 0, kv_page_tokens: int = 128, kv_type: int = KV_F16,
                        prefill_batch: int = 512, timeout_ms: int | None = None) -> "LlamaModel":
        """The same model split over the ranks of a torch.distributed group,
        one process per GPU of one node (mv_model_open_tp).  Every rank calls
        this, then makes the same calls in the same order; every call returns
        what the single-GPU model returns, bit for bit.  The group only
        carries the peer-memory handles (any backend); the data path is the
        library's own kernels over NVLink."""
        import torch.distributed as dist

        rank, world = dist.get_rank(group), dist.get_world_size(group)
        if device is None:
            device = int(os.environ.get("LOCAL_RANK", rank))
        lib = load()
        self = cls.__new__(cls)
        self._m = None
        h = C.c_void_p()
        rc = lib.mv_init(device)
        if rc == 0:
            rc = lib.mv_model_open_tp(os.fspath(gguf_path).encode(), ctx_override, kv_page_tokens, kv_type,
                                      rank, world, prefill_batch, C.byref(h))
        handle = (C.c_char * HANDLE_BYTES)()
        if rc == 0:
            self._m = h
            rc = lib.mv_model_tp_handle(h, handle)
        msg = lib.mv_last_error().decode() if rc else ""
        # every rank learns whether every other rank opened its share
        got = [None] * world
        dist.all_gather_object(got, (rc, msg, bytes(handle)), group=group)
        bad = [(r, g[0], g[1]) for r, g in enumerate(got) if g[0]]
        if bad:
            self.close(barrier=False)
            raise RuntimeError(f"tensor-parallel open failed on rank(s) {bad}")
        self.tp_rank, self.tp_world, self._group = rank, world, group
        if timeout_ms is not None:
            check(lib.mv_model_tp_set_timeout(h, int(timeout_ms)))
        buf = b"".join(g[2] for g in got)
        check(lib.mv_model_tp_connect(h, buf))
        self._read_config()
        return self

    def set_timeout(self, ms: int) -> None:
        """Bound of every wait for the other ranks (tensor parallel only)."""
        check(load().mv_model_tp_set_timeout(self._m, int(ms)))

    def config(self) -> dict:
        return {"n_ctx": self.n_ctx, "n_embd": self.n_embd, "n_ff": self.n_ff, "n_layer": self.n_layer,
                "n_head": self.n_head, "n_head_kv": self.n_head_kv, "vocab": self.vocab}

    def reset(self) -> None:
        check(load().mv_model_reset(self._m))

    def position(self) -> int:
        return load().mv_model_position(self._m)

    def kv_bytes_allocated(self) -> int:
        return load().mv_model_kv_bytes(self._m)

    @property
    def stream(self) -> int:
        return load().mv_model_stream(self._m) or 0

    @property
    def decode_persistent(self) -> bool:
        """Whether a decode step runs every layer in one persistent kernel
        (MV_DECODE_PERSISTENT=1 at open)."""
        return bool(load().mv_model_decode_persistent(self._m))

    def forward(self, token: int, compute_logits: bool = True, out: np.ndarray | None = None) -> np.ndarray:
        """One decode step (src/llama_model.cpp:253-259); returns host logits."""
        out = self._logits if out is None else out
        check(load().mv_model_forward(self._m, int(token), int(compute_logits),
                                      out.ctypes.data_as(C.c_void_p) if compute_logits else None))
        return out

    def prefill(self, tokens, batch_size: int = 64, compute_logits_last: bool = True) -> np.ndarray:
        """Chunked prefill (src/llama_model.cpp:260) with Q8 activations."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        check(load().mv_model_prefill(self._m, t.ctypes.data_as(C.c_void_p), t.size, batch_size,
                                      int(compute_logits_last),
                                      self._logits.ctypes.data_as(C.c_void_p) if compute_logits_last else None))
        return self._logits

    def generate_greedy(self, token: int, n: int) -> np.ndarray:
        """n greedy steps from `token`, argmax on the device."""
        out = np.empty(n, np.int32)
        check(load().mv_model_generate_greedy(self._m, int(token), n, out.ctypes.data_as(C.c_void_p)))
        return out

    def generate(self, prompt, n: int, eos_id: int | None = None) -> list:
        """LlamaModel::generate at temperature 0 (src/llama_model.cpp:261)."""
        prompt = list(prompt)
        if not prompt:
            raise ValueError("prompt cannot be empty")
        self.reset()
        if len(prompt) > 1:
            self.prefill(prompt[:-1], 64, False)
        cur, out = prompt[-1], []
        for _ in range(n):
            nxt = int(np.argmax(self.forward(cur, True)))
            out.append(nxt)
            cur = nxt
            if eos_id is not None and nxt == eos_id:
                break
        return out

    def open_sequences(self, n_seq: int, ctx: int) -> "SequenceSet":
        """A set of n_seq sequences (own KV caches, one block table) decoded
        together with this model's weights (mv_model_seqs_open)."""
        return SequenceSet(self, n_seq, ctx)

    def close(self, barrier: bool = True) -> None:
        """Frees the model.  Tensor parallel: every rank's block is mapped by
        the others, so the ranks first wait for one another."""
        if self._m:
            if barrier and self.tp_world > 1:
                import torch.distributed as dist

                if dist.is_initialized():
                    dist.barrier(group=self._group)  # every rank idle
                    load().mv_model_tp_disconnect(self._m)
                    dist.barrier(group=self._group)  # nobody maps a block any more
            load().mv_model_close(self._m)
            self._m = None

    def __del__(self):
        try:
            self.close(barrier=False)
        except Exception:
            pass


class SequenceSet:
    """Several sequences decoded as one batch (mv_model_forward_batch): each
    has its own paged KV cache and position; ``forward(tokens)`` advances every
    sequence by one token and returns [n_seq, vocab] logits."""

    def __init__(self, model: LlamaModel, n_seq: int, ctx: int):
        self._s = None
        self.model, self.n_seq = model, int(n_seq)
        h = C.c_void_p()
        check(load().mv_model_seqs_open(model._m, self.n_seq, int(ctx), C.byref(h)))
        self._s = h
        self._logits = np.empty((self.n_seq, model.vocab), np.float32)

    def prefill(self, seq: int, tokens, batch_size: int = 64, compute_logits_last: bool = True) -> np.ndarray:
        """LlamaModel.prefill for one sequence of the set; its last logits."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty(self.model.vocab, np.float32)
        check(load().mv_model_seqs_prefill(self._s, int(seq), t.ctypes.data_as(C.c_void_p), t.size, batch_size,
                                           int(compute_logits_last),
                                           out.ctypes.data_as(C.c_void_p) if compute_logits_last else None))
        return out

    def forward(self, tokens) -> np.ndarray:
        """One decode token of every sequence; [n_seq, vocab] host logits."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        if t.size != self.n_seq:
            raise ValueError(f"need {self.n_seq} tokens, got {t.size}")
        check(load().mv_model_forward_batch(self.model._m, self._s, t.ctypes.data_as(C.c_void_p),
                                            self._logits.ctypes.data_as(C.c_void_p)))
        return self._logits

    def position(self, seq: int) -> int:
        p = C.c_uint64()
        check(load().mv_model_seqs_position(self._s, int(seq), C.byref(p)))
        return p.value

    def reset(self, seq: int) -> None:
        check(load().mv_model_seqs_reset(self._s, int(seq)))

    def close(self) -> None:
        if self._s:
            load().mv_model_seqs_free(self._s)
            self._s = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
