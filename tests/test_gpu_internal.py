"""Device twins of the reference's internal-format kernels (quant.hpp /
matmul.hpp: 20-byte Q4_0 and 36-byte Q8_0 blocks, fp32 scales, interleaved
nibbles) against the oracle, which is pinned to the reference's own build in
test_oracle.py::test_ref_internal_formats.  Integer work and every fp32
rounding follow the reference's order, so the bar is bit-exact."""
from __future__ import annotations

import numpy as np
import pytest

import memvanta_b200 as mv

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def _x(rng, n, zero_blocks=()):
    x = rng.normal(0, 1, n).astype(np.float32)
    x[::37] = 0.5 * np.round(x[::37] * 14)  # exact halves: ties of nearbyint
    for b in zero_blocks:
        x[32 * b:32 * b + 32] = 0.0
    return x


@pytest.mark.parametrize("n", [32, 4096, 11008])
def test_int_quantize_bit_exact(cuda, oracle, n):
    import torch
    rng = np.random.default_rng(n)
    x = _x(rng, n, zero_blocks=(0,))
    xt = torch.from_numpy(x).to(cuda)
    assert np.array_equal(mv.int_quantize_q8_0(xt).cpu().numpy(), oracle.int_quantize_q8_0(x))
    assert np.array_equal(mv.int_quantize_q4_0(xt).cpu().numpy(), oracle.int_quantize_q4_0(x))


@pytest.mark.parametrize("rows,cols", [(1, 32), (37, 256), (300, 4096), (64, 11008)])
def test_int_matvecs_bit_exact(cuda, oracle, rows, cols):
    import torch
    rng = np.random.default_rng(rows * 7 + cols)
    A = (rng.normal(0, 0.05, (rows, cols))).astype(np.float32)
    A[0, :32] = 0.0  # a zero block
    x = _x(rng, cols)
    a20, a36, x36 = oracle.int_quantize_q4_0(A), oracle.int_quantize_q8_0(A), oracle.int_quantize_q8_0(x)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    y = mv.int_matvec_q4_q8(dev(a20), dev(x36), rows, cols).cpu().numpy()
    assert np.array_equal(bits(y), bits(oracle.int_matvec_q4_q8(a20, x36, rows, cols)))
    y = mv.int_matvec_q4_0(dev(a20), dev(x), rows, cols).cpu().numpy()
    assert np.array_equal(bits(y), bits(oracle.int_matvec_q4_0(a20, x, rows, cols)))
    y = mv.int_matvec_q8_0(dev(a36), dev(x), rows, cols).cpu().numpy()
    assert np.array_equal(bits(y), bits(oracle.int_matvec_q8_0(a36, x, rows, cols)))


def test_int_matmul_q4_0_batch_bit_exact(cuda, oracle):
    import torch
    rng = np.random.default_rng(3)
    rows, cols, batch = 45, 1024, 5
    A = rng.normal(0, 0.05, (rows, cols)).astype(np.float32)
    X = rng.normal(0, 1, (batch, cols)).astype(np.float32)
    a20 = oracle.int_quantize_q4_0(A)
    y = mv.int_matmul_q4_0_batch(torch.from_numpy(a20).to(cuda), torch.from_numpy(X).to(cuda), rows, cols, batch)
    assert np.array_equal(bits(y.cpu().numpy()), bits(oracle.int_matmul_q4_0_batch(a20, X, rows, cols)))


@pytest.mark.parametrize("rows,cols", [(1, 1), (33, 77), (128, 4096)])
def test_matvec_f32_bit_exact(cuda, oracle, rows, cols):
    import torch
    rng = np.random.default_rng(rows + cols)
    A = rng.normal(0, 1, (rows, cols)).astype(np.float32)
    x = rng.normal(0, 1, cols).astype(np.float32)
    y = mv.matvec_f32(torch.from_numpy(A).to(cuda), torch.from_numpy(x).to(cuda)).cpu().numpy()
    assert np.array_equal(bits(y), bits(oracle.matvec_f32(A, x)))


def test_int_entry_points_reject_bad_sizes(cuda):
    import torch
    x = torch.zeros(33, device=cuda)
    with pytest.raises(mv.MemVantaError):
        mv.int_quantize_q8_0(x)
