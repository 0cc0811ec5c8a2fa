"""mv_gemm_q8_noalloc: the Q8-activation batched matmul for callers that may
not allocate device memory (a framework whose own pool owns the GPU's memory,
a fixed memory budget, a latency-critical loop).  Both entry points run the
same bit-exact tensor-core GEMM on the same quantised activations, so its
output must equal the allocating entry point's, mv_gemm(..., MV_ACT_Q8), bit
for bit, on two calls in a row -- the second call reuses the library's fixed
scratch array the first one left behind -- and equal the oracle's
MEMVANTA_FORCE_Q8_ACT=1 matmul (tensor_matmul_batch_v06).  This file is
collected last so a failure here leaves every other test already run."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import memvanta_b200 as mv
from memvanta_b200 import gguf

pytestmark = pytest.mark.gpu


def _noalloc(W, X, Y, stream):
    lib = mv.load()
    return lib.mv_gemm_q8_noalloc(W.handle, C.c_void_p(X.data_ptr()), X.shape[0], C.c_void_p(Y.data_ptr()),
                                  C.c_void_p(stream.cuda_stream))


def _pool_reserved(dev):
    """Bytes the device's default memory pool (cudaMallocAsync) holds."""
    from cuda.bindings import runtime as rt
    err, pool = rt.cudaDeviceGetDefaultMemPool(dev)
    assert err == rt.cudaError_t.cudaSuccess
    err, v = rt.cudaMemPoolGetAttribute(pool, rt.cudaMemPoolAttr.cudaMemPoolAttrReservedMemCurrent)
    assert err == rt.cudaError_t.cudaSuccess
    return int(v)


@pytest.mark.parametrize("rows,cols,batch", [(11008, 4096, 32), (4096, 11008, 96), (64, 128, 3)])
def test_noalloc_matches_mv_gemm_on_two_calls(cuda, oracle, rows, cols, batch):
    import torch
    rng = np.random.default_rng(rows + cols + batch)
    w = gguf.gen_q4_0(rows, cols, rng)
    W = mv.Weight.upload(w, mv.Q4_0, rows, cols)
    stream = torch.cuda.current_stream()
    for call in range(2):
        x = rng.standard_normal((batch, cols)).astype(np.float32)
        X = torch.from_numpy(x).to(cuda)
        want = torch.empty((batch, rows), dtype=torch.float32, device=cuda)
        mv.gemm(W, X, want, mv.ACT_Q8, stream)
        got = torch.full((batch, rows), float("nan"), dtype=torch.float32, device=cuda)
        torch.cuda.synchronize()
        # mv_gemm's stream-ordered scratch went back to the pool: nothing the
        # no-allocation call could take from it is held outside the pool, and
        # the pool itself must not grow across the call
        pool_before = _pool_reserved(cuda.index)
        free_before = torch.cuda.mem_get_info()[0]
        rc = _noalloc(W, X, got, stream)
        assert rc == 0, mv.load().mv_last_error().decode()
        torch.cuda.synchronize()
        assert _pool_reserved(cuda.index) == pool_before, call
        if call == 1:  # the first call on a device may load the module holding the array
            assert torch.cuda.mem_get_info()[0] == free_before
        g, r = got.cpu().numpy(), want.cpu().numpy()
        assert np.array_equal(g, r), (call, float(np.nanmax(np.abs(g - r))))
        if call == 0 and rows * cols <= 11008 * 4096 and batch >= 2:
            # and both are the reference's FORCE_Q8 prefill matmul
            ref = oracle.matmul_batch_v06(gguf.Q4_0, w, rows, cols, x, force_q8=True)
            assert np.array_equal(g, ref.reshape(g.shape))
    W.free()


def test_noalloc_rejects_oversize_and_wrong_type(cuda):
    import torch
    rng = np.random.default_rng(1)
    W = mv.Weight.upload(gguf.gen_q4_0(8, 11008, rng), mv.Q4_0, 8, 11008)
    X = torch.zeros((1024, 11008), dtype=torch.float32, device=cuda)   # 12.7 MB of scratch > 8 MiB
    Y = torch.empty((1024, 8), dtype=torch.float32, device=cuda)
    assert _noalloc(W, X, Y, torch.cuda.current_stream()) == mv._lib.MV_ERR_INVALID
    assert b"8388608" in mv.load().mv_last_error()
    W8 = mv.Weight.upload(gguf.gen_q8_0(8, 128, rng), mv.Q8_0, 8, 128)
    X8 = torch.zeros((4, 128), dtype=torch.float32, device=cuda)
    Y8 = torch.empty((4, 8), dtype=torch.float32, device=cuda)
    assert _noalloc(W8, X8, Y8, torch.cuda.current_stream()) == mv._lib.MV_ERR_UNSUPPORTED
