"""ctypes front-end for the test oracles.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arms, never by the product package.

* ``Oracle`` wraps ``_bin/libmvoracle.so`` -- the C restatement of the
  reference's arithmetic in ``mv_oracle.c``.
* ``Reference`` wraps ``_ref/libmvref.so`` -- the reference's own code
  compiled from its unmodified sources (see Makefile); present wherever it was
  built (it travels with the repository snapshot as a build product).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_bin", "libmvoracle.so")
REF_SO = os.path.join(HERE, "_ref", "libmvref.so")
REF_REAL_BENCH = os.path.join(HERE, "_ref", "memvanta_real_bench")
REF_KERNEL_BENCH = os.path.join(HERE, "_ref", "memvanta_kernel_bench")

F32, F16, Q4_0, Q8_0, Q6_K = 0, 1, 2, 8, 14
KV_F32, KV_F16, KV_Q8, KV_Q8_0 = 0, 1, 2, 3

_f = np.float32
_p = C.c_void_p
_sz = C.c_size_t


def build(ref_root: str | None = None) -> None:
    """Build the oracle (and, when the reference checkout exists, oracle/_ref)."""
    args = ["make", "-s", "-C", HERE]
    if ref_root:
        args.append(f"REF={ref_root}")
    subprocess.run(args, check=True)


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class Oracle:
    """The C restatement (mv_oracle.c)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        self.L = L
        L.mvo_fp16_to_fp32.restype = C.c_float
        L.mvo_fp16_to_fp32.argtypes = [C.c_uint16]
        L.mvo_fp32_to_fp16.restype = C.c_uint16
        L.mvo_fp32_to_fp16.argtypes = [C.c_float]
        L.mvo_quantize_q8.argtypes = [_p, _sz, _p, _p]
        L.mvo_quantize_q8_rows.argtypes = [_p, _sz, _sz, _p, _p]
        L.mvo_dot_q4_q8_block.restype = C.c_int32
        L.mvo_dot_q4_q8_block.argtypes = [_p, _p]
        L.mvo_q6_k_value.restype = C.c_int
        L.mvo_q6_k_value.argtypes = [_p, _sz]
        L.mvo_matvec.restype = C.c_int
        L.mvo_matvec.argtypes = [C.c_int, _p, _sz, _sz, _p, _p]
        L.mvo_matmul_batch.restype = C.c_int
        L.mvo_matmul_batch.argtypes = [C.c_int, _p, _sz, _sz, _p, _sz, _p]
        L.mvo_matmul_batch_v06.restype = C.c_int
        L.mvo_matmul_batch_v06.argtypes = [C.c_int, _p, _sz, _sz, _p, _sz, _p, C.c_int, C.c_int]
        L.mvo_read_row.restype = C.c_int
        L.mvo_read_row.argtypes = [C.c_int, _p, _sz, _sz, _sz, _p]
        L.mvo_rmsnorm.argtypes = [_p, _p, _sz, C.c_float, _p]
        L.mvo_rope_tables.argtypes = [_sz, _sz, C.c_float, _p, _p]
        L.mvo_rope.argtypes = [_p, _sz, _p, _sz, _sz, _p, _p]
        L.mvo_silu_mul.argtypes = [_p, _p, _p, _sz]
        L.mvo_kv_store.argtypes = [C.c_int, _p, _sz, _p, _p]
        L.mvo_kv_row_bytes.restype = _sz
        L.mvo_kv_row_bytes.argtypes = [C.c_int, _sz]
        L.mvo_kv_row_scales.restype = _sz
        L.mvo_kv_row_scales.argtypes = [C.c_int, _sz]
        L.mvo_attn_decode.argtypes = [C.c_int, _p, _sz, _sz, _sz, _p, _p, _p, _p, _p, _sz, _sz, _p]
        L.mvo_dot_f32.restype = C.c_float
        L.mvo_dot_f32.argtypes = [_p, _p, _sz]
        for n in ("mvo_int_quantize_q8_0", "mvo_int_quantize_q4_0"):
            getattr(L, n).argtypes = [_p, _sz, _p]
        L.mvo_int_matvec_q4_q8.argtypes = [_p, _p, _p, _sz, _sz]
        L.mvo_int_matvec_q4_0.argtypes = [_p, _p, _p, _sz, _sz]
        L.mvo_int_matvec_q8_0.argtypes = [_p, _p, _p, _sz, _sz]
        L.mvo_int_matmul_q4_0_batch.argtypes = [_p, _p, _p, _sz, _sz, _sz]
        L.mvo_matvec_f32.argtypes = [_p, _p, _p, _sz, _sz]

    # scalar helpers
    def fp16_to_fp32(self, h: int) -> float:
        return self.L.mvo_fp16_to_fp32(h)

    def fp32_to_fp16(self, f: float) -> int:
        return self.L.mvo_fp32_to_fp16(f)

    def fp32_to_fp16_array(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=_f)
        out = np.empty(x.shape, dtype=np.uint16)
        # mvo_kv_store(F16) is the reference's per-element conversion loop
        self.L.mvo_kv_store(KV_F16, _ptr(x.reshape(-1)), x.size, _ptr(out.reshape(-1)), None)
        return out

    def quantize_q8(self, x: np.ndarray):
        x = np.ascontiguousarray(x, dtype=_f)
        rows, cols = (1, x.size) if x.ndim == 1 else x.shape
        q = np.empty((rows, cols), np.int8)
        d = np.empty((rows, cols // 32), _f)
        self.L.mvo_quantize_q8_rows(_ptr(x), rows, cols, _ptr(q), _ptr(d))
        return (q[0], d[0]) if x.ndim == 1 else (q, d)

    def dot_q4_q8_block(self, blk18: np.ndarray, aq: np.ndarray) -> int:
        return self.L.mvo_dot_q4_q8_block(_ptr(np.ascontiguousarray(blk18)), _ptr(np.ascontiguousarray(aq)))

    def q6_k_value(self, blk210: np.ndarray, i: int) -> int:
        return self.L.mvo_q6_k_value(_ptr(np.ascontiguousarray(blk210)), i)

    def matvec(self, t: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
        y = np.empty(rows, _f)
        x = np.ascontiguousarray(x, dtype=_f)
        if self.L.mvo_matvec(t, _ptr(np.ascontiguousarray(w)), rows, cols, _ptr(x), _ptr(y)):
            raise RuntimeError("oracle matvec: unsupported type or shape")
        return y

    def matmul_batch(self, t, w, rows, cols, x) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=_f)
        b = x.shape[0]
        y = np.empty((b, rows), _f)
        if self.L.mvo_matmul_batch(t, _ptr(np.ascontiguousarray(w)), rows, cols, _ptr(x), b, _ptr(y)):
            raise RuntimeError("oracle matmul_batch: unsupported type or shape")
        return y

    def matmul_batch_v06(self, t, w, rows, cols, x, force_q8=False, ffn=False) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=_f)
        b = x.shape[0]
        y = np.empty((b, rows), _f)
        if self.L.mvo_matmul_batch_v06(t, _ptr(np.ascontiguousarray(w)), rows, cols, _ptr(x), b, _ptr(y),
                                       int(force_q8), int(ffn)):
            raise RuntimeError("oracle matmul_batch_v06: unsupported type or shape")
        return y

    def read_row(self, t, w, rows, cols, row) -> np.ndarray:
        out = np.empty(cols, _f)
        if self.L.mvo_read_row(t, _ptr(np.ascontiguousarray(w)), rows, cols, row, _ptr(out)):
            raise RuntimeError("oracle read_row: bad row or type")
        return out

    def rmsnorm(self, x, w, eps) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=_f)
        o = np.empty_like(x)
        self.L.mvo_rmsnorm(_ptr(x), _ptr(np.ascontiguousarray(w, dtype=_f)), x.size, eps, _ptr(o))
        return o

    def rope_tables(self, n_ctx, hd, theta):
        c = np.empty((n_ctx, hd // 2), _f)
        s = np.empty((n_ctx, hd // 2), _f)
        self.L.mvo_rope_tables(n_ctx, hd, theta, _ptr(c), _ptr(s))
        return c, s

    def rope(self, q, n_head, k, n_head_kv, hd, cos_row, sin_row):
        q = np.array(q, dtype=_f, copy=True)
        k = np.array(k, dtype=_f, copy=True)
        self.L.mvo_rope(_ptr(q), n_head, _ptr(k), n_head_kv, hd, _ptr(np.ascontiguousarray(cos_row, dtype=_f)),
                        _ptr(np.ascontiguousarray(sin_row, dtype=_f)))
        return q, k

    def silu_mul(self, g, u):
        g = np.ascontiguousarray(g, dtype=_f)
        o = np.empty_like(g)
        self.L.mvo_silu_mul(_ptr(g), _ptr(np.ascontiguousarray(u, dtype=_f)), _ptr(o), g.size)
        return o

    def kv_row_bytes(self, kv_type, kv_dim):
        return self.L.mvo_kv_row_bytes(kv_type, kv_dim)

    def kv_row_scales(self, kv_type, kv_dim):
        return self.L.mvo_kv_row_scales(kv_type, kv_dim)

    def kv_store(self, kv_type, v):
        v = np.ascontiguousarray(v, dtype=_f)
        raw = np.zeros(self.kv_row_bytes(kv_type, v.size), np.uint8)
        sc = np.zeros(max(1, self.kv_row_scales(kv_type, v.size)), _f)
        self.L.mvo_kv_store(kv_type, _ptr(v), v.size, _ptr(raw), _ptr(sc))
        return raw, sc[: self.kv_row_scales(kv_type, v.size)]

    def attn_decode(self, kv_type, q, n_head, n_head_kv, hd, k_pages, v_pages, k_scales, v_scales, block_table,
                    page, n_ctx):
        out = np.empty(n_head * hd, _f)
        self.L.mvo_attn_decode(kv_type, _ptr(np.ascontiguousarray(q, dtype=_f)), n_head, n_head_kv, hd,
                               _ptr(k_pages), _ptr(v_pages), _ptr(k_scales), _ptr(v_scales),
                               _ptr(np.ascontiguousarray(block_table, dtype=np.int32)), page, n_ctx, _ptr(out))
        return out

    # internal formats
    def int_quantize_q8_0(self, x):
        x = np.ascontiguousarray(x, dtype=_f)
        out = np.empty(x.size // 32 * 36, np.uint8)
        self.L.mvo_int_quantize_q8_0(_ptr(x), x.size, _ptr(out))
        return out

    def int_quantize_q4_0(self, x):
        x = np.ascontiguousarray(x, dtype=_f)
        out = np.empty(x.size // 32 * 20, np.uint8)
        self.L.mvo_int_quantize_q4_0(_ptr(x), x.size, _ptr(out))
        return out

    def int_matvec_q4_q8(self, A20, x36, rows, cols):
        y = np.empty(rows, _f)
        self.L.mvo_int_matvec_q4_q8(_ptr(A20), _ptr(x36), _ptr(y), rows, cols)
        return y

    def int_matvec_q4_0(self, A20, x, rows, cols):
        y = np.empty(rows, _f)
        self.L.mvo_int_matvec_q4_0(_ptr(A20), _ptr(np.ascontiguousarray(x, dtype=_f)), _ptr(y), rows, cols)
        return y

    def int_matvec_q8_0(self, A36, x, rows, cols):
        y = np.empty(rows, _f)
        self.L.mvo_int_matvec_q8_0(_ptr(A36), _ptr(np.ascontiguousarray(x, dtype=_f)), _ptr(y), rows, cols)
        return y

    def int_matmul_q4_0_batch(self, A20, x, rows, cols):
        x = np.ascontiguousarray(x, dtype=_f)
        y = np.empty((x.shape[0], rows), _f)
        self.L.mvo_int_matmul_q4_0_batch(_ptr(A20), _ptr(x), _ptr(y), rows, cols, x.shape[0])
        return y

    def matvec_f32(self, A, x):
        A = np.ascontiguousarray(A, dtype=_f)
        y = np.empty(A.shape[0], _f)
        self.L.mvo_matvec_f32(_ptr(A), _ptr(np.ascontiguousarray(x, dtype=_f)), _ptr(y), A.shape[0], A.shape[1])
        return y


class Reference:
    """The reference's own code (oracle/_ref/libmvref.so)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (needs the reference checkout at build time)")
        L = C.CDLL(path)
        self.L = L
        L.mvr_last_error.restype = C.c_char_p
        L.mvr_quantize_q8.argtypes = [_p, _sz, _p, _p]
        L.mvr_dot_q4_q8_block.restype = C.c_int
        L.mvr_dot_q4_q8_block.argtypes = [_p, _p]
        L.mvr_q6_k_value.restype = C.c_int
        L.mvr_q6_k_value.argtypes = [_p, _sz]
        L.mvr_fp32_to_fp16.restype = C.c_uint16
        L.mvr_fp32_to_fp16.argtypes = [C.c_float]
        L.mvr_fp16_to_fp32.restype = C.c_float
        L.mvr_fp16_to_fp32.argtypes = [C.c_uint16]
        L.mvr_file_open.restype = _p
        L.mvr_file_open.argtypes = [C.c_char_p]
        L.mvr_file_close.argtypes = [_p]
        L.mvr_matvec.restype = C.c_int
        L.mvr_matvec.argtypes = [_p, C.c_char_p, _p, _p, C.c_uint]
        L.mvr_matmul_batch.restype = C.c_int
        L.mvr_matmul_batch.argtypes = [_p, C.c_char_p, _p, _p, _sz, C.c_uint]
        L.mvr_matmul_batch_v06.restype = C.c_int
        L.mvr_matmul_batch_v06.argtypes = [_p, C.c_char_p, _p, _p, _sz, C.c_uint, C.c_int]
        L.mvr_read_row.restype = C.c_int
        L.mvr_read_row.argtypes = [_p, C.c_char_p, _sz, _p, _sz]
        L.mvr_kv_new.restype = _p
        L.mvr_kv_new.argtypes = [_sz, _sz, C.c_int]
        L.mvr_kv_free.argtypes = [_p]
        L.mvr_kv_write.argtypes = [_p, _sz, _p, _p]
        L.mvr_kv_dot_key.restype = C.c_float
        L.mvr_kv_dot_key.argtypes = [_p, _sz, _sz, _p, _sz]
        L.mvr_kv_add_value.argtypes = [_p, _sz, _sz, C.c_float, _p, _sz]
        L.mvr_model_open.restype = _p
        L.mvr_model_open.argtypes = [C.c_char_p, C.c_uint, _sz, _sz, C.c_int]
        L.mvr_model_free.argtypes = [_p]
        L.mvr_model_reset.argtypes = [_p]
        L.mvr_model_position.restype = _sz
        L.mvr_model_position.argtypes = [_p]
        L.mvr_model_vocab.restype = _sz
        L.mvr_model_vocab.argtypes = [_p]
        L.mvr_model_n_ctx.restype = _sz
        L.mvr_model_n_ctx.argtypes = [_p]
        L.mvr_model_forward.restype = C.c_int
        L.mvr_model_forward.argtypes = [_p, C.c_int, C.c_int, _p]
        L.mvr_model_forward_q8env.restype = C.c_int
        L.mvr_model_forward_q8env.argtypes = [_p, C.c_int, C.c_int, _p, C.c_int]
        L.mvr_model_prefill.restype = C.c_int
        L.mvr_model_prefill.argtypes = [_p, _p, _sz, _sz, C.c_int, _p, C.c_int]
        for n in ("mvr_int_quantize_q8_0", "mvr_int_quantize_q4_0"):
            getattr(L, n).argtypes = [_p, _sz, _p]
        L.mvr_int_matvec_q4_q8.argtypes = [_p, _p, _p, _sz, _sz, C.c_uint]
        L.mvr_int_matvec_q4_0.argtypes = [_p, _p, _p, _sz, _sz, C.c_uint]
        L.mvr_int_matvec_q8_0.argtypes = [_p, _p, _p, _sz, _sz, C.c_uint]
        L.mvr_int_matmul_q4_0_batch.argtypes = [_p, _p, _p, _sz, _sz, _sz, C.c_uint]
        L.mvr_matvec_f32.argtypes = [_p, _p, _p, _sz, _sz, C.c_uint]

    def _check(self, rc):
        if rc:
            raise RuntimeError(self.L.mvr_last_error().decode())

    def quantize_q8(self, x):
        x = np.ascontiguousarray(x, dtype=_f)
        q = np.empty(x.size, np.int8)
        d = np.empty(x.size // 32, _f)
        self.L.mvr_quantize_q8(_ptr(x), x.size, _ptr(q), _ptr(d))
        return q, d

    def dot_q4_q8_block(self, blk18, aq) -> int:
        return self.L.mvr_dot_q4_q8_block(_ptr(np.ascontiguousarray(blk18)), _ptr(np.ascontiguousarray(aq)))

    def q6_k_value(self, blk210, i) -> int:
        return self.L.mvr_q6_k_value(_ptr(np.ascontiguousarray(blk210)), i)

    def fp32_to_fp16(self, f: float) -> int:
        return self.L.mvr_fp32_to_fp16(f)

    def fp16_to_fp32(self, h: int) -> float:
        return self.L.mvr_fp16_to_fp32(h)

    # GGUF file-level kernels
    def open(self, path: str):
        h = self.L.mvr_file_open(os.fspath(path).encode())
        if not h:
            raise RuntimeError(self.L.mvr_last_error().decode())
        return h

    def close(self, h):
        self.L.mvr_file_close(h)

    def matvec(self, h, name, x, rows, threads=1):
        x = np.ascontiguousarray(x, dtype=_f)
        y = np.empty(rows, _f)
        self._check(self.L.mvr_matvec(h, name.encode(), _ptr(x), _ptr(y), threads))
        return y

    def matmul_batch(self, h, name, x, rows, threads=1):
        x = np.ascontiguousarray(x, dtype=_f)
        y = np.empty((x.shape[0], rows), _f)
        self._check(self.L.mvr_matmul_batch(h, name.encode(), _ptr(x), _ptr(y), x.shape[0], threads))
        return y

    def matmul_batch_v06(self, h, name, x, rows, threads=1, force_q8=False):
        x = np.ascontiguousarray(x, dtype=_f)
        y = np.empty((x.shape[0], rows), _f)
        self._check(self.L.mvr_matmul_batch_v06(h, name.encode(), _ptr(x), _ptr(y), x.shape[0], threads,
                                                int(force_q8)))
        return y

    def read_row(self, h, name, row, cols):
        out = np.empty(cols, _f)
        self._check(self.L.mvr_read_row(h, name.encode(), row, _ptr(out), cols))
        return out

    # KV cache
    def kv_new(self, kv_dim, page, kv_type):
        return self.L.mvr_kv_new(kv_dim, page, kv_type)

    def kv_free(self, c):
        self.L.mvr_kv_free(c)

    def kv_write(self, c, pos, k, v):
        self.L.mvr_kv_write(c, pos, _ptr(np.ascontiguousarray(k, dtype=_f)), _ptr(np.ascontiguousarray(v, dtype=_f)))

    def kv_dot_key(self, c, pos, off, q):
        q = np.ascontiguousarray(q, dtype=_f)
        return self.L.mvr_kv_dot_key(c, pos, off, _ptr(q), q.size)

    def kv_add_value(self, c, pos, off, alpha, out):
        self.L.mvr_kv_add_value(c, pos, off, alpha, _ptr(out), out.size)

    # LlamaModel
    def model_open(self, path, threads=1, ctx=0, page=128, kv_type=KV_F16):
        m = self.L.mvr_model_open(os.fspath(path).encode(), threads, ctx, page, kv_type)
        if not m:
            raise RuntimeError(self.L.mvr_last_error().decode())
        return m

    def model_free(self, m):
        self.L.mvr_model_free(m)

    def model_reset(self, m):
        self.L.mvr_model_reset(m)

    def model_vocab(self, m):
        return self.L.mvr_model_vocab(m)

    def model_forward(self, m, token, compute_logits=True, force_q8=False):
        out = np.empty(self.model_vocab(m), _f)
        self._check(self.L.mvr_model_forward_q8env(m, token, int(compute_logits), _ptr(out), int(force_q8)))
        return out

    def model_prefill(self, m, tokens, batch=32, compute_logits=True, force_q8=False):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty(self.model_vocab(m), _f)
        self._check(self.L.mvr_model_prefill(m, _ptr(t), t.size, batch, int(compute_logits), _ptr(out),
                                             int(force_q8)))
        return out

    # internal formats
    def int_quantize_q8_0(self, x):
        x = np.ascontiguousarray(x, dtype=_f)
        out = np.empty(x.size // 32 * 36, np.uint8)
        self.L.mvr_int_quantize_q8_0(_ptr(x), x.size, _ptr(out))
        return out

    def int_quantize_q4_0(self, x):
        x = np.ascontiguousarray(x, dtype=_f)
        out = np.empty(x.size // 32 * 20, np.uint8)
        self.L.mvr_int_quantize_q4_0(_ptr(x), x.size, _ptr(out))
        return out

    def int_matvec_q4_q8(self, A20, x36, rows, cols, threads=1):
        y = np.empty(rows, _f)
        self.L.mvr_int_matvec_q4_q8(_ptr(A20), _ptr(x36), _ptr(y), rows, cols, threads)
        return y

    def int_matvec_q4_0(self, A20, x, rows, cols, threads=1):
        y = np.empty(rows, _f)
        self.L.mvr_int_matvec_q4_0(_ptr(A20), _ptr(np.ascontiguousarray(x, dtype=_f)), _ptr(y), rows, cols, threads)
        return y

    def int_matvec_q8_0(self, A36, x, rows, cols, threads=1):
        y = np.empty(rows, _f)
        self.L.mvr_int_matvec_q8_0(_ptr(A36), _ptr(np.ascontiguousarray(x, dtype=_f)), _ptr(y), rows, cols, threads)
        return y

    def int_matmul_q4_0_batch(self, A20, x, rows, cols, threads=1):
        x = np.ascontiguousarray(x, dtype=_f)
        y = np.empty((x.shape[0], rows), _f)
        self.L.mvr_int_matmul_q4_0_batch(_ptr(A20), _ptr(x), _ptr(y), rows, cols, x.shape[0], threads)
        return y

    def matvec_f32(self, A, x, threads=1):
        A = np.ascontiguousarray(A, dtype=_f)
        y = np.empty(A.shape[0], _f)
        self.L.mvr_matvec_f32(_ptr(A), _ptr(np.ascontiguousarray(x, dtype=_f)), _ptr(y), A.shape[0], A.shape[1], threads)
        return y
