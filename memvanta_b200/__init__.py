"""memvanta_b200 -- B200 (sm_100a) implementation of MemVanta's GGUF
block-quantized matmul hot path, behind a C ABI (include/memvanta_b200.h).

This module is the Python host side over that ABI.  Its names mirror the
reference's C++ API so tests read like the reference's own:

* ``tensor_matvec``, ``tensor_matmul_batch``, ``tensor_matmul_batch_v06``,
  ``tensor_read_row_f32`` -- include/memvanta/gguf_kernels.hpp:25-30, with the
  reference's host-pointer contract (numpy in, numpy out);
* ``LlamaModel`` with ``forward`` / ``prefill`` / ``generate`` / ``reset`` /
  ``position`` / ``kv_bytes_allocated`` -- include/memvanta/llama_model.hpp:100-113.

Device-pointer entry points (``gemv``, ``gemm``, ``quantize_q8``, ...) take
torch CUDA tensors and run asynchronously on the given (or current) stream;
torch only provides device memory and streams here.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from ._lib import (F32, F16, Q4_0, Q8_0, Q6_K, ACT_F32, ACT_Q8, KV_F32, KV_F16, KV_Q8, KV_Q8_0,  # noqa: F401
                   MV_ERR_TIMEOUT, MemVantaError, check, load)

__all__ = [
    "init", "Weight", "tensor_matvec", "tensor_matmul_batch", "tensor_matmul_batch_v06", "tensor_read_row_f32",
    "gemv", "gemm", "quantize_q8", "q4_0_block_dots", "read_rows", "rmsnorm", "rope", "silu_mul", "add_inplace",
    "fp32_to_fp16", "kv_row_bytes", "kv_row_scales", "kv_append", "paged_attn_decode", "paged_attn_prefill", "LlamaModel",
    "SequenceSet",
    "MemVantaError",
]


def init(device: int = 0) -> None:
    check(load().mv_init(device))


def _np_ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def _t_ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(stream):
    if stream is None:
        import torch
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)
    if isinstance(stream, int):
        return C.c_void_p(stream)
    return C.c_void_p(stream.cuda_stream)


class Weight:
    """One GGUF tensor resident in HBM (planar repack of its blocks)."""

    def __init__(self, handle, ggml_type: int, rows: int, cols: int):
        self._h = handle
        self.type, self.rows, self.cols = ggml_type, rows, cols

    @classmethod
    def upload(cls, blocks, ggml_type: int, rows: int, cols: int, stream=None) -> "Weight":
        """blocks: the tensor's raw GGML bytes (numpy uint8 / bytes / memoryview)."""
        buf = np.ascontiguousarray(np.frombuffer(blocks, dtype=np.uint8) if not isinstance(blocks, np.ndarray)
                                   else blocks.view(np.uint8).reshape(-1))
        h = C.c_void_p()
        s = C.c_void_p(0) if stream is None else _stream(stream)
        check(load().mv_weight_upload(_np_ptr(buf), buf.nbytes, ggml_type, rows, cols, s, C.byref(h)))
        return cls(h, ggml_type, rows, cols)

    @property
    def handle(self):
        return self._h

    def info(self) -> dict:
        t, r, c, b = C.c_int(), C.c_uint64(), C.c_uint64(), C.c_uint64()
        check(load().mv_weight_info(self._h, C.byref(t), C.byref(r), C.byref(c), C.byref(b)))
        return {"type": t.value, "rows": r.value, "cols": c.value, "device_bytes": b.value}

    def download(self) -> np.ndarray:
        from .gguf import tensor_nbytes
        n = tensor_nbytes(self.type, self.rows * self.cols)
        out = np.empty(n, np.uint8)
        check(load().mv_weight_download(self._h, _np_ptr(out), n))
        return out

    def free(self) -> None:
        if self._h:
            check(load().mv_weight_free(self._h))
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


# ------------------------------------------------ reference host contract

def tensor_matvec(w: Weight, x: np.ndarray) -> np.ndarray:
    """memvanta::tensor_matvec (src/gguf_kernels.cpp:244-253): host x -> host y."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.size != w.cols:
        raise ValueError(f"x has {x.size} elements, tensor has {w.cols} columns")
    y = np.empty(w.rows, np.float32)
    check(load().mv_tensor_matvec_host(w.handle, _np_ptr(x), _np_ptr(y)))
    return y


def tensor_matmul_batch_v06(w: Weight, x: np.ndarray, force_q8: bool = False) -> np.ndarray:
    """memvanta::tensor_matmul_batch_v06 (src/gguf_kernels.cpp:261-271);
    force_q8 selects the MEMVANTA_FORCE_Q8_ACT=1 path."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, w.cols)
    y = np.empty((x.shape[0], w.rows), np.float32)
    check(load().mv_tensor_matmul_batch_host(w.handle, _np_ptr(x), _np_ptr(y), x.shape[0],
                                             ACT_Q8 if force_q8 else ACT_F32))
    return y


def tensor_matmul_batch(w: Weight, x: np.ndarray) -> np.ndarray:
    """memvanta::tensor_matmul_batch (src/gguf_kernels.cpp:255-259): fp32 activations."""
    return tensor_matmul_batch_v06(w, x, force_q8=False)


def tensor_read_row_f32(w: Weight, row: int) -> np.ndarray:
    """memvanta::tensor_read_row_f32 (src/gguf_kernels.cpp:226)."""
    out = np.empty(w.cols, np.float32)
    check(load().mv_tensor_read_row_host(w.handle, row, _np_ptr(out)))
    return out


# ------------------------------------------- device-pointer entry points

def gemv(w: Weight, x, y, stream=None) -> None:
    check(load().mv_gemv(w.handle, _t_ptr(x), _t_ptr(y), _stream(stream)))


def gemm(w: Weight, x, y, act_mode: int = ACT_Q8, stream=None) -> None:
    check(load().mv_gemm(w.handle, _t_ptr(x), x.shape[0] if x.dim() > 1 else 1, _t_ptr(y), act_mode,
                         _stream(stream)))


def stream_status(stream=None) -> None:
    """Synchronise the stream; raise MV_ERR_TIMEOUT if a tensor-core kernel
    gave up a bounded device-side wait since the last check."""
    check(load().mv_stream_status(_stream(stream)))


def test_gemm_stall(skip_commit_stage: int, wait_limit_us: int = 0) -> None:
    """Test hook: the next fp16 tensor-core GEMM launch leaves out one MMA
    commit and bounds its waits by wait_limit_us (mv_test_gemm_stall)."""
    check(load().mv_test_gemm_stall(skip_commit_stage, wait_limit_us))


def quantize_q8(x, stream=None):
    import torch
    rows, cols = (1, x.numel()) if x.dim() == 1 else tuple(x.shape)
    q = torch.empty((rows, cols), dtype=torch.int8, device=x.device)
    d = torch.empty((rows, cols // 32), dtype=torch.float32, device=x.device)
    check(load().mv_quantize_q8(_t_ptr(x), rows, cols, _t_ptr(q), _t_ptr(d), _stream(stream)))
    return q, d


# ---- internal (non-GGUF) block formats: device twins of quant.hpp / matmul.hpp
# Tensors are torch CUDA tensors; blocks are uint8 tensors of 20 (Q4_0) or 36
# (Q8_0) bytes per 32 elements.

def int_quantize_q8_0(x, stream=None):
    """quantize_q8_0 (src/quant.cpp:44-62) -> uint8[n/32*36]."""
    import torch
    out = torch.empty(x.numel() // 32 * 36, dtype=torch.uint8, device=x.device)
    check(load().mv_int_quantize_q8_0(_t_ptr(x), x.numel(), _t_ptr(out), _stream(stream)))
    return out


def int_quantize_q4_0(x, stream=None):
    """quantize_q4_0 (src/quant.cpp:64-85) -> uint8[n/32*20]."""
    import torch
    out = torch.empty(x.numel() // 32 * 20, dtype=torch.uint8, device=x.device)
    check(load().mv_int_quantize_q4_0(_t_ptr(x), x.numel(), _t_ptr(out), _stream(stream)))
    return out


def int_matvec_q4_q8(A20, x36, rows: int, cols: int, stream=None):
    import torch
    y = torch.empty(rows, dtype=torch.float32, device=A20.device)
    check(load().mv_int_matvec_q4_q8(_t_ptr(A20), _t_ptr(x36), _t_ptr(y), rows, cols, _stream(stream)))
    return y


def int_matvec_q4_0(A20, x, rows: int, cols: int, stream=None):
    import torch
    y = torch.empty(rows, dtype=torch.float32, device=A20.device)
    check(load().mv_int_matvec_q4_0(_t_ptr(A20), _t_ptr(x), _t_ptr(y), rows, cols, _stream(stream)))
    return y


def int_matvec_q8_0(A36, x, rows: int, cols: int, stream=None):
    import torch
    y = torch.empty(rows, dtype=torch.float32, device=A36.device)
    check(load().mv_int_matvec_q8_0(_t_ptr(A36), _t_ptr(x), _t_ptr(y), rows, cols, _stream(stream)))
    return y


def int_matmul_q4_0_batch(A20, x, rows: int, cols: int, batch: int, stream=None):
    import torch
    y = torch.empty((batch, rows), dtype=torch.float32, device=A20.device)
    check(load().mv_int_matmul_q4_0_batch(_t_ptr(A20), _t_ptr(x), _t_ptr(y), rows, cols, batch, _stream(stream)))
    return y


def matvec_f32(A, x, stream=None):
    import torch
    rows, cols = A.shape
    y = torch.empty(rows, dtype=torch.float32, device=A.device)
    check(load().mv_matvec_f32(_t_ptr(A), _t_ptr(x), _t_ptr(y), rows, cols, _stream(stream)))
    return y


def q4_0_block_dots(w: Weight, x, stream=None):
    import torch
    isum = torch.empty((w.rows, w.cols // 32), dtype=torch.int32, device=x.device)
    check(load().mv_q4_0_block_dots(w.handle, _t_ptr(x), _t_ptr(isum), _stream(stream)))
    return isum


def read_rows(w: Weight, rows, stream=None):
    import torch
    out = torch.empty((rows.numel(), w.cols), dtype=torch.float32, device=rows.device)
    check(load().mv_read_rows(w.handle, _t_ptr(rows), rows.numel(), _t_ptr(out), _stream(stream)))
    return out


def rmsnorm(x, w, eps: float, stream=None):
    import torch
    out = torch.empty_like(x)
    rows = 1 if x.dim() == 1 else x.shape[0]
    check(load().mv_rmsnorm(_t_ptr(x), _t_ptr(w), rows, x.shape[-1], eps, _t_ptr(out), _stream(stream)))
    return out


def rope(q, n_head: int, k, n_head_kv: int, head_dim: int, cos_t, sin_t, pos, stream=None) -> None:
    """In place on q [rows, n_head*hd] and k [rows, n_head_kv*hd]."""
    check(load().mv_rope(_t_ptr(q), n_head, _t_ptr(k), n_head_kv, head_dim, pos.numel(), _t_ptr(cos_t),
                         _t_ptr(sin_t), _t_ptr(pos), _stream(stream)))


def silu_mul(g, u, stream=None):
    import torch
    out = torch.empty_like(g)
    check(load().mv_silu_mul(_t_ptr(g), _t_ptr(u), _t_ptr(out), g.numel(), _stream(stream)))
    return out


def add_inplace(x, y, stream=None) -> None:
    check(load().mv_add_inplace(_t_ptr(x), _t_ptr(y), x.numel(), _stream(stream)))


def fp32_to_fp16(x, stream=None):
    import torch
    h = torch.empty(x.shape, dtype=torch.int16, device=x.device)
    check(load().mv_fp32_to_fp16(_t_ptr(x), _t_ptr(h), x.numel(), _stream(stream)))
    return h


def kv_row_bytes(kv_type: int, kv_dim: int) -> int:
    return load().mv_kv_row_bytes(kv_type, kv_dim)


def kv_row_scales(kv_type: int, kv_dim: int) -> int:
    return load().mv_kv_row_scales(kv_type, kv_dim)


def kv_append(kv_type, k, v, pos, block_table, max_pages, page, k_pages, v_pages, k_scales=None, v_scales=None,
              seq=None, stream=None) -> None:
    rows, kv_dim = k.shape
    check(load().mv_kv_append(kv_type, _t_ptr(k), _t_ptr(v), rows, kv_dim, _t_ptr(seq), _t_ptr(pos),
                              _t_ptr(block_table), max_pages, page, _t_ptr(k_pages), _t_ptr(v_pages),
                              _t_ptr(k_scales), _t_ptr(v_scales), _stream(stream)))


def paged_attn_decode(kv_type, q, n_head, n_head_kv, head_dim, k_pages, v_pages, block_table, max_pages, page,
                      ctx_len, max_ctx, k_scales=None, v_scales=None, out=None, stream=None):
    import torch
    n_seq = q.shape[0]
    if out is None:
        out = torch.empty((n_seq, n_head * head_dim), dtype=torch.float32, device=q.device)
    check(load().mv_paged_attn_decode(kv_type, _t_ptr(q), n_seq, n_head, n_head_kv, head_dim, _t_ptr(k_pages),
                                      _t_ptr(v_pages), _t_ptr(k_scales), _t_ptr(v_scales), _t_ptr(block_table),
                                      max_pages, page, _t_ptr(ctx_len), max_ctx, _t_ptr(out), _stream(stream)))
    return out


def paged_attn_decode_split(kv_type, q, n_head, n_head_kv, head_dim, k_pages, v_pages, block_table, max_pages,
                            page, ctx_len, max_ctx, k_scales=None, v_scales=None, out=None, stream=None):
    """paged_attn_decode split over the context (not bit-exact: ~1e-6)."""
    import torch
    n_seq = q.shape[0]
    if out is None:
        out = torch.empty((n_seq, n_head * head_dim), dtype=torch.float32, device=q.device)
    check(load().mv_paged_attn_decode_split(kv_type, _t_ptr(q), n_seq, n_head, n_head_kv, head_dim, _t_ptr(k_pages),
                                            _t_ptr(v_pages), _t_ptr(k_scales), _t_ptr(v_scales),
                                            _t_ptr(block_table), max_pages, page, _t_ptr(ctx_len), max_ctx,
                                            _t_ptr(out), _stream(stream)))
    return out


def paged_attn_prefill(kv_type, q, n_head, n_head_kv, head_dim, k_pages, v_pages, block_table, max_pages, page,
                       ctx_len, max_ctx, k_scales=None, v_scales=None, out=None, stream=None):
    """Attention of the query rows of one sequence (a prefill chunk): every
    row reads block-table row 0; row i sees ctx_len[i] tokens."""
    import torch
    n_q = q.shape[0]
    if out is None:
        out = torch.empty((n_q, n_head * head_dim), dtype=torch.float32, device=q.device)
    check(load().mv_paged_attn_prefill(kv_type, _t_ptr(q), n_q, n_head, n_head_kv, head_dim, _t_ptr(k_pages),
                                       _t_ptr(v_pages), _t_ptr(k_scales), _t_ptr(v_scales), _t_ptr(block_table),
                                       max_pages, page, _t_ptr(ctx_len), max_ctx, _t_ptr(out), _stream(stream)))
    return out


from .model import LlamaModel, SequenceSet  # noqa: E402
