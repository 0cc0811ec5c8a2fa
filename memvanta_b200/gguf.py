"""GGUF v3 writer, minimal reader and seeded block generators.

The generators draw the synthetic weights the benchmark configurations are
defined on (Q4_0 / Q8_0 / Q6_K blocks with the scale distributions named
there); the writer emits files the reference's ``GgufFile`` parser and this
package's C++ loader both accept.  Block layouts follow the GGML formats the
reference reads (src/gguf_kernels.cpp:21-31):

* Q4_0 -- 18 bytes ``{fp16 d; u8 qs[16]}``; element i<16 is ``qs[i]&15``,
  element 16+i is ``qs[i]>>4``; value ``(q-8)*d``.
* Q8_0 -- 34 bytes ``{fp16 d; i8 qs[32]}``.
* Q6_K -- 210 bytes ``{u8 ql[128]; u8 qh[64]; i8 scales[16]; fp16 d}`` per
  256 elements.
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass, field
from typing import BinaryIO, Iterable, Sequence

import numpy as np

# GGML tensor types (include/memvanta/gguf.hpp:18-26 of the reference).
F32, F16, Q4_0, Q8_0, Q6_K = 0, 1, 2, 8, 14
TYPE_NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q8_0: "Q8_0", Q6_K: "Q6_K"}
# (elements per block, bytes per block)
BLOCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q6_K: (256, 210)}

# GGUF metadata value types.
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)


def tensor_nbytes(ggml_type: int, elements: int) -> int:
    per, size = BLOCK[ggml_type]
    if elements % per:
        raise ValueError(f"{TYPE_NAMES[ggml_type]} element count {elements} is not a multiple of {per}")
    return elements // per * size


# ---------------------------------------------------------------- generators

def _abs_normal_f16(rng: np.random.Generator, n: int, sigma: float) -> np.ndarray:
    return np.abs(rng.standard_normal(n, dtype=np.float32) * np.float32(sigma)).astype(np.float16)


def gen_q4_0(rows: int, cols: int, rng: np.random.Generator, sigma: float = 0.02) -> np.ndarray:
    """Q4_0 rows: per block d = fp16(|N(0, sigma)|) and 16 bytes of uniform nibbles."""
    nb = rows * (cols // 32)
    out = np.frombuffer(bytearray(rng.bytes(nb * 18)), dtype=np.uint8).reshape(nb, 18)
    out[:, 0:2] = _abs_normal_f16(rng, nb, sigma).view(np.uint8).reshape(nb, 2)
    return out.reshape(-1)


def gen_q8_0(rows: int, cols: int, rng: np.random.Generator, sigma: float = 0.02) -> np.ndarray:
    """Q8_0 rows: d = fp16(|N(0, sigma)|), int8 values uniform in -127..127."""
    nb = rows * (cols // 32)
    out = np.empty((nb, 34), dtype=np.uint8)
    out[:, 0:2] = _abs_normal_f16(rng, nb, sigma).view(np.uint8).reshape(nb, 2)
    out[:, 2:] = rng.integers(-127, 128, size=(nb, 32), dtype=np.int8).view(np.uint8)
    return out.reshape(-1)


def gen_q6_k(rows: int, cols: int, rng: np.random.Generator, sigma: float = 0.002) -> np.ndarray:
    """Q6_K rows: uniform ql/qh bytes (6-bit values uniform in 0..63, minus 32),
    int8 sub-scales uniform in -32..31, d = fp16(|N(0, sigma)|)."""
    nb = rows * (cols // 256)
    out = np.empty((nb, 210), dtype=np.uint8)
    out[:, 0:192] = np.frombuffer(rng.bytes(nb * 192), dtype=np.uint8).reshape(nb, 192)
    out[:, 192:208] = rng.integers(-32, 32, size=(nb, 16), dtype=np.int8).view(np.uint8)
    out[:, 208:210] = _abs_normal_f16(rng, nb, sigma).view(np.uint8).reshape(nb, 2)
    return out.reshape(-1)


def gen_f16(rows: int, cols: int, rng: np.random.Generator, sigma: float = 0.02) -> np.ndarray:
    return (rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(sigma)).astype(np.float16).view(np.uint8)


def gen_f32(rows: int, cols: int, rng: np.random.Generator, sigma: float = 0.02) -> np.ndarray:
    return (rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(sigma)).view(np.uint8)


def gen_blocks(ggml_type: int, rows: int, cols: int, rng: np.random.Generator) -> np.ndarray:
    return {Q4_0: gen_q4_0, Q8_0: gen_q8_0, Q6_K: gen_q6_k, F16: gen_f16, F32: gen_f32}[ggml_type](rows, cols, rng)


# ------------------------------------------------------------------- writer

def _s(x: str) -> bytes:
    b = x.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, value) -> bytes:
    if isinstance(value, bool):
        return _s(key) + struct.pack("<IB", _BOOL, int(value))
    if isinstance(value, int):
        return _s(key) + struct.pack("<II", _U32, value)
    if isinstance(value, float):
        return _s(key) + struct.pack("<If", _F32, value)
    if isinstance(value, str):
        return _s(key) + struct.pack("<I", _STR) + _s(value)
    if isinstance(value, (list, tuple)) and all(isinstance(v, str) for v in value):
        return _s(key) + struct.pack("<IIQ", _ARR, _STR, len(value)) + b"".join(_s(v) for v in value)
    raise TypeError(f"unsupported metadata value for {key}: {type(value)}")


@dataclass
class TensorSpec:
    name: str
    dims: Sequence[int]          # GGML order: ne0 (cols), ne1 (rows)
    ggml_type: int
    data: object = None          # bytes-like, or a callable returning one (streamed)

    def nbytes(self) -> int:
        n = 1
        for d in self.dims:
            n *= int(d)
        return tensor_nbytes(self.ggml_type, n)


def write_gguf(path: str | os.PathLike, metadata: Iterable[tuple[str, object]], tensors: Sequence[TensorSpec],
               alignment: int = 32) -> int:
    """Write a GGUF v3 file; tensor data are produced one at a time so a
    multi-GB model never has to sit in memory at once.  Returns the file size."""
    meta = list(metadata)
    if not any(k == "general.alignment" for k, _ in meta):
        meta.append(("general.alignment", alignment))
    offsets, off = [], 0
    for t in tensors:
        off = (off + alignment - 1) // alignment * alignment
        offsets.append(off)
        off += t.nbytes()
    head = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(meta)))
    for k, v in meta:
        head += _kv(k, v)
    for t, o in zip(tensors, offsets):
        head += _s(t.name) + struct.pack("<I", len(t.dims)) + struct.pack(f"<{len(t.dims)}Q", *t.dims)
        head += struct.pack("<IQ", t.ggml_type, o)
    data_start = (len(head) + alignment - 1) // alignment * alignment
    head += bytes(data_start - len(head))
    with open(path, "wb") as f:
        f.write(head)
        pos = 0
        for t, o in zip(tensors, offsets):
            if o > pos:
                f.write(bytes(o - pos))
                pos = o
            data = t.data() if callable(t.data) else t.data
            buf = memoryview(np.ascontiguousarray(data).view(np.uint8).reshape(-1)) if isinstance(data, np.ndarray) else memoryview(data)
            if buf.nbytes != t.nbytes():
                raise ValueError(f"tensor {t.name}: {buf.nbytes} bytes, expected {t.nbytes()}")
            f.write(buf)
            pos += buf.nbytes
        return data_start + pos


# ------------------------------------------------------------- llama model

@dataclass
class LlamaShape:
    n_layer: int = 32
    n_embd: int = 4096
    n_head: int = 32
    n_head_kv: int = 32
    n_ff: int = 11008
    vocab: int = 32000
    n_ctx: int = 2048
    rms_eps: float = 1e-6
    rope_theta: float = 10000.0
    layer_type: int = Q4_0
    embd_type: int = Q4_0
    output_type: int | None = Q6_K      # None -> tied to token_embd (no output.weight)
    extra: dict = field(default_factory=dict)


# OpenLLaMA-7B-shaped configuration.
LLAMA_7B = LlamaShape()


def write_random_llama(path: str | os.PathLike, shape: LlamaShape = LLAMA_7B, seed: int = 1234) -> int:
    """Random-init Llama GGUF: Q4_0 (or shape.layer_type) projections with
    |N(0,0.02)| scales, F32 norms 1+U(-0.02,0.02), Q6_K output head, and a
    placeholder vocabulary so the reference's tokenizer loads."""
    rng = np.random.default_rng(seed)
    D, F, L = shape.n_embd, shape.n_ff, shape.n_layer
    hd = D // shape.n_head
    KV = shape.n_head_kv * hd
    meta = [
        ("general.architecture", "llama"),
        ("general.name", f"memvanta-b200 random llama L{L} D{D} F{F}"),
        ("llama.context_length", shape.n_ctx),
        ("llama.embedding_length", D),
        ("llama.feed_forward_length", F),
        ("llama.block_count", L),
        ("llama.attention.head_count", shape.n_head),
        ("llama.attention.head_count_kv", shape.n_head_kv),
        ("llama.attention.layer_norm_rms_epsilon", float(shape.rms_eps)),
        ("llama.rope.freq_base", float(shape.rope_theta)),
        ("tokenizer.ggml.model", "llama"),
        ("tokenizer.ggml.tokens", [f"<t{i}>" for i in range(shape.vocab)]),
        ("tokenizer.ggml.bos_token_id", 1),
        ("tokenizer.ggml.eos_token_id", 2),
    ]
    # One child generator per tensor keeps every tensor's bytes independent
    # of the order in which tensors are produced.
    seeds = iter(rng.integers(0, 2**63 - 1, size=16 + 16 * L))

    def mat(t, rows, cols):
        s = int(next(seeds))
        return lambda: gen_blocks(t, rows, cols, np.random.default_rng(s))

    def norm(n):
        s = int(next(seeds))
        return lambda: (1.0 + np.random.default_rng(s).uniform(-0.02, 0.02, n)).astype(np.float32)

    ts = [TensorSpec("token_embd.weight", [D, shape.vocab], shape.embd_type, mat(shape.embd_type, shape.vocab, D))]
    for i in range(L):
        p = f"blk.{i}."
        ts += [
            TensorSpec(p + "attn_norm.weight", [D], F32, norm(D)),
            TensorSpec(p + "attn_q.weight", [D, D], shape.layer_type, mat(shape.layer_type, D, D)),
            TensorSpec(p + "attn_k.weight", [D, KV], shape.layer_type, mat(shape.layer_type, KV, D)),
            TensorSpec(p + "attn_v.weight", [D, KV], shape.layer_type, mat(shape.layer_type, KV, D)),
            TensorSpec(p + "attn_output.weight", [D, D], shape.layer_type, mat(shape.layer_type, D, D)),
            TensorSpec(p + "ffn_norm.weight", [D], F32, norm(D)),
            TensorSpec(p + "ffn_gate.weight", [D, F], shape.layer_type, mat(shape.layer_type, F, D)),
            TensorSpec(p + "ffn_up.weight", [D, F], shape.layer_type, mat(shape.layer_type, F, D)),
            TensorSpec(p + "ffn_down.weight", [F, D], shape.layer_type, mat(shape.layer_type, D, F)),
        ]
    ts.append(TensorSpec("output_norm.weight", [D], F32, norm(D)))
    if shape.output_type is not None:
        ts.append(TensorSpec("output.weight", [D, shape.vocab], shape.output_type,
                             mat(shape.output_type, shape.vocab, D)))
    return write_gguf(path, meta, ts)


def write_single_tensor(path: str | os.PathLike, name: str, ggml_type: int, rows: int, cols: int,
                        data: np.ndarray) -> int:
    """A GGUF holding one matrix; used to drive the reference's tensor_* kernels."""
    return write_gguf(path, [("general.architecture", "none")], [TensorSpec(name, [cols, rows], ggml_type, data)])


# ------------------------------------------------------------------- reader

@dataclass
class TensorInfo:
    name: str
    dims: list
    ggml_type: int
    offset: int          # absolute file offset
    nbytes: int

    @property
    def cols(self) -> int:
        return int(self.dims[0])

    @property
    def rows(self) -> int:
        return int(self.dims[1]) if len(self.dims) > 1 else 1


def read_tensor_infos(path: str | os.PathLike) -> tuple[dict, list]:
    """Parse a GGUF header: (metadata, [TensorInfo]).  Test-side helper."""
    with open(path, "rb") as f:
        def rd(fmt):
            n = struct.calcsize(fmt)
            return struct.unpack(fmt, f.read(n))

        def rs():
            (n,) = rd("<Q")
            return f.read(n).decode()

        scal = {_U8: "<B", _I8: "<b", _U16: "<H", _I16: "<h", _U32: "<I", _I32: "<i", _F32: "<f",
                _BOOL: "<B", _U64: "<Q", _I64: "<q", _F64: "<d"}

        def rv(t):
            if t == _STR:
                return rs()
            if t == _ARR:
                et, n = rd("<IQ")
                return [rv(et) for _ in range(n)]
            return rd(scal[t])[0]

        if f.read(4) != b"GGUF":
            raise ValueError("not a GGUF file")
        ver, nt, nkv = rd("<IQQ")
        meta = {}
        for _ in range(nkv):
            k = rs()
            (t,) = rd("<I")
            meta[k] = rv(t)
        raw = []
        for _ in range(nt):
            name = rs()
            (nd,) = rd("<I")
            dims = list(rd(f"<{nd}Q"))
            t, rel = rd("<IQ")
            raw.append((name, dims, t, rel))
        align = int(meta.get("general.alignment", 32))
        start = (f.tell() + align - 1) // align * align
    infos = []
    for name, dims, t, rel in raw:
        n = 1
        for d in dims:
            n *= d
        infos.append(TensorInfo(name, dims, t, start + rel, tensor_nbytes(t, n)))
    return meta, infos
