"""dc_qmatmul_skinny_noalloc, the allocation-free entry point for callers that cannot allocate device memory (a
plug-in whose host owns all device memory, a loop that cannot take cudaMalloc's device synchronisation): its output
matches the existing skinny matmul entry point's (dc_qmatmul_form, form 1) on two calls in a row, it allocates no
device memory after its first call, and it rejects requests beyond its static scratch limit with a clear error.

The file name sorts it after the other test files, so a run that stops at the first failure has run them already."""
import ctypes

import numpy as np
import pytest

from conftest import f16_of, to_dev

pytestmark = pytest.mark.gpu


def _inputs(M, N, K, bits, seed, dev, host=False):
    from decision_js_b200 import synth
    X, codes, S = synth.config1_inputs(seed=seed, M=M, N=N, K=K, bits=bits)
    d = [to_dev(X, dev), to_dev(codes, dev), to_dev(S, dev)]
    return (d, (X, codes, S)) if host else d


def _close(got, ref):
    # the matmul tolerance of tests/test_gpu_kernels.py (about one f16 ulp)
    tol = 4e-3 * np.abs(ref) + 1e-3 * np.abs(ref).max()
    assert (np.abs(got - ref) <= tol).all()


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("M,N,K,splits", [(1, 768, 768, 0), (16, 1024, 2048, 4), (100, 384, 320, 3),
                                          (64, 3072, 1024, 0)])
def test_noalloc_matches_skinny_entry_point(ctx, dev, pkg, oracle, bits, M, N, K, splits):
    import torch
    from decision_js_b200._lib import lib
    L = lib()
    for call in range(2):  # two calls in a row, each against the existing entry point and the oracle
        (X, W, S), (hX, hW, hS) = _inputs(M, N, K, bits, 31 * call + M + bits, dev, host=True)
        ref = torch.empty((M, N), dtype=torch.int16, device=dev)
        got = torch.full((M, N), -1, dtype=torch.int16, device=dev)
        torch.cuda.synchronize()
        ctx.call("qmatmul_form", X, W, S, ref, M, N, K, bits, 1, splits)
        ctx.sync(60000)
        rc = L.dc_qmatmul_skinny_noalloc(None, X.data_ptr(), W.data_ptr(), S.data_ptr(), got.data_ptr(), M, N, K,
                                         bits, splits)
        assert rc == 0, L.dc_last_error().decode()
        torch.cuda.synchronize()
        _close(f16_of(got), f16_of(ref))
        _close(f16_of(got), oracle.qmatmul(hX, hW, hS, N, K, bits).view(np.float16).astype(np.float32))


def test_noalloc_allocates_nothing(dev, pkg):
    """After the first call on the device (which resolves the static array), further calls leave the device's free
    memory unchanged: nothing is allocated, by this library or by torch."""
    import torch
    from decision_js_b200._lib import lib
    L = lib()
    M, N, K = 8, 2048, 4096
    X, W, S = _inputs(M, N, K, 8, 5, dev)
    Y = torch.empty((M, N), dtype=torch.int16, device=dev)
    args = (X.data_ptr(), W.data_ptr(), S.data_ptr(), Y.data_ptr(), M, N, K, 8, 8)
    assert L.dc_qmatmul_skinny_noalloc(None, *args) == 0, L.dc_last_error().decode()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        assert L.dc_qmatmul_skinny_noalloc(None, *args) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0


def test_noalloc_rejects_over_the_limit(dev, pkg):
    import torch
    from decision_js_b200._lib import DC_EINVAL, lib
    L = lib()
    M, N, K = 128, 16384, 8192
    X, W, S = _inputs(M, 128, K, 8, 1, dev)  # pointers only: the call is refused before any launch
    Y = torch.empty((1,), dtype=torch.int16, device=dev)
    rc = L.dc_qmatmul_skinny_noalloc(None, X.data_ptr(), W.data_ptr(), S.data_ptr(), Y.data_ptr(), M, N, K, 8, 64)
    assert rc == DC_EINVAL
    msg = L.dc_last_error().decode()
    assert "static" in msg and "limit" in msg
