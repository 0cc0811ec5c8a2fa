"""ctypes binding of libmemvanta_b200.so (the C ABI in include/memvanta_b200.h).

The shared library is built in-tree (memvanta_b200/libmemvanta_b200.so).  There
is no fallback: if the library is missing or cannot be loaded every call
raises, so a GPU run can never silently take a CPU path.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmemvanta_b200.so")

MV_OK, MV_ERR_INVALID, MV_ERR_UNSUPPORTED, MV_ERR_CUDA, MV_ERR_OOM, MV_ERR_IO, MV_ERR_TIMEOUT, MV_ERR_NOT_BUILT = range(8)
ERR_NAMES = {1: "MV_ERR_INVALID", 2: "MV_ERR_UNSUPPORTED", 3: "MV_ERR_CUDA", 4: "MV_ERR_OOM", 5: "MV_ERR_IO",
             6: "MV_ERR_TIMEOUT", 7: "MV_ERR_NOT_BUILT"}
F32, F16, Q4_0, Q8_0, Q6_K = 0, 1, 2, 8, 14
ACT_F32, ACT_Q8 = 0, 1
KV_F32, KV_F16, KV_Q8, KV_Q8_0 = 0, 1, 2, 3

_p = C.c_void_p
_u64 = C.c_uint64
_i = C.c_int
_f = C.c_float

# name -> (restype, argtypes); every symbol the header declares
SIGNATURES = {
    "mv_init": (_i, [_i]),
    "mv_last_error": (C.c_char_p, []),
    "mv_version": (_i, []),
    "mv_binary_arch": (_i, [C.POINTER(_i)]),
    "mv_stream_status": (_i, [_p]),
    "mv_test_gemm_stall": (_i, [_i, _u64]),
    "mv_weight_upload": (_i, [_p, _u64, _i, _u64, _u64, _p, C.POINTER(_p)]),
    "mv_weight_from_device": (_i, [_p, _u64, _i, _u64, _u64, _p, C.POINTER(_p)]),
    "mv_weight_free": (_i, [_p]),
    "mv_weight_info": (_i, [_p, C.POINTER(_i), C.POINTER(_u64), C.POINTER(_u64), C.POINTER(_u64)]),
    "mv_weight_download": (_i, [_p, _p, _u64]),
    "mv_gemv": (_i, [_p, _p, _p, _p]),
    "mv_gemm": (_i, [_p, _p, _u64, _p, _i, _p]),
    "mv_gemm_q8_noalloc": (_i, [_p, _p, _u64, _p, _p]),
    "mv_quantize_q8": (_i, [_p, _u64, _u64, _p, _p, _p]),
    "mv_q4_0_block_dots": (_i, [_p, _p, _p, _p]),
    "mv_read_row": (_i, [_p, _u64, _p, _p]),
    "mv_read_rows": (_i, [_p, _p, _u64, _p, _p]),
    "mv_rmsnorm": (_i, [_p, _p, _u64, _u64, _f, _p, _p]),
    "mv_rope": (_i, [_p, _u64, _p, _u64, _u64, _u64, _p, _p, _p, _p]),
    "mv_silu_mul": (_i, [_p, _p, _p, _u64, _p]),
    "mv_add_inplace": (_i, [_p, _p, _u64, _p]),
    "mv_fp32_to_fp16": (_i, [_p, _p, _u64, _p]),
    "mv_kv_row_bytes": (_u64, [_i, _u64]),
    "mv_kv_row_scales": (_u64, [_i, _u64]),
    "mv_kv_append": (_i, [_i, _p, _p, _u64, _u64, _p, _p, _p, _u64, _u64, _p, _p, _p, _p, _p]),
    "mv_paged_attn_decode": (_i, [_i, _p, _u64, _u64, _u64, _u64, _p, _p, _p, _p, _p, _u64, _u64, _p, _u64, _p,
                                  _p]),
    "mv_paged_attn_decode_split": (_i, [_i, _p, _u64, _u64, _u64, _u64, _p, _p, _p, _p, _p, _u64, _u64, _p, _u64,
                                        _p, _p]),
    "mv_paged_attn_prefill": (_i, [_i, _p, _u64, _u64, _u64, _u64, _p, _p, _p, _p, _p, _u64, _u64, _p, _u64, _p,
                                   _p]),
    "mv_tensor_matvec_host": (_i, [_p, _p, _p]),
    "mv_tensor_matmul_batch_host": (_i, [_p, _p, _p, _u64, _i]),
    "mv_tensor_read_row_host": (_i, [_p, _u64, _p]),
    "mv_model_open": (_i, [C.c_char_p, _u64, _u64, _i, C.POINTER(_p)]),
    "mv_model_close": (_i, [_p]),
    "mv_model_config": (_i, [_p, C.POINTER(_u64)]),
    "mv_model_reset": (_i, [_p]),
    "mv_model_position": (_u64, [_p]),
    "mv_model_kv_bytes": (_u64, [_p]),
    "mv_model_forward": (_i, [_p, C.c_int32, _i, _p]),
    "mv_model_prefill": (_i, [_p, _p, _u64, _u64, _i, _p]),
    "mv_model_generate_greedy": (_i, [_p, C.c_int32, _u64, _p]),
    "mv_model_stream": (_p, [_p]),
    "mv_model_decode_persistent": (_i, [_p]),
    "mv_model_seqs_open": (_i, [_p, _u64, _u64, C.POINTER(_p)]),
    "mv_model_seqs_free": (_i, [_p]),
    "mv_model_seqs_prefill": (_i, [_p, _u64, _p, _u64, _u64, _i, _p]),
    "mv_model_seqs_position": (_i, [_p, _u64, C.POINTER(_u64)]),
    "mv_model_seqs_reset": (_i, [_p, _u64]),
    "mv_model_forward_batch": (_i, [_p, _p, _p, _p]),
    "mv_int_quantize_q8_0": (_i, [_p, _u64, _p, _p]),
    "mv_int_quantize_q4_0": (_i, [_p, _u64, _p, _p]),
    "mv_int_matvec_q4_q8": (_i, [_p, _p, _p, _u64, _u64, _p]),
    "mv_int_matvec_q4_0": (_i, [_p, _p, _p, _u64, _u64, _p]),
    "mv_int_matvec_q8_0": (_i, [_p, _p, _p, _u64, _u64, _p]),
    "mv_int_matmul_q4_0_batch": (_i, [_p, _p, _p, _u64, _u64, _u64, _p]),
    "mv_matvec_f32": (_i, [_p, _p, _p, _u64, _u64, _p]),
    "mv_model_open_tp": (_i, [C.c_char_p, _u64, _u64, _i, _i, _i, _u64, C.POINTER(_p)]),
    "mv_model_tp_handle": (_i, [_p, _p]),
    "mv_model_tp_connect": (_i, [_p, _p]),
    "mv_model_tp_set_timeout": (_i, [_p, _u64]),
    "mv_model_tp_disconnect": (_i, [_p]),
}


class MemVantaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERR_NAMES.get(code, code)}: {msg}")
        self.code = code


_lock = threading.Lock()
_lib = None


def load(path: str = LIB_PATH) -> C.CDLL:
    """Load (once) and return the library with every signature declared."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(path):
                raise FileNotFoundError(
                    f"{path} is missing: build it with `python -m memvanta_b200.build` (no CPU fallback exists)")
            lib = C.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
        return _lib


def check(rc: int) -> None:
    if rc != MV_OK:
        raise MemVantaError(rc, load().mv_last_error().decode(errors="replace"))
