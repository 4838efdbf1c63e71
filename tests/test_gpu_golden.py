"""The GPU kernels on the reference's own quantizer output (tests/golden/quant_golden.npz, written by
tests/golden/make_golden.py from scripts/export_common.py:64-97).

The fixture's codes hold what the reference's exporter writes and the synthetic inputs may not: q8 codes 1 and
255 (saturated -127 / +127), q4 nibble 0 (code -8) and 15, an all-zero block with scale 1, and scales near the
f16 subnormal range. Dequantization and the embedding gather must reproduce the reference's dequantized weight
bit for bit; the matmuls and the readout over the same tables are checked against the oracle with the tolerances
of the other kernel tests.
"""
import os

import numpy as np
import pytest

from conftest import f16_of, rel_err, to_dev

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
G = np.load(os.path.join(HERE, "golden", "quant_golden.npz"))
N, K = G["w"].shape  # 48 x 256


def _table(bits):
    codes = np.ascontiguousarray(G[f"q{bits}_codes"].reshape(N, -1))
    scales = np.ascontiguousarray(G[f"q{bits}_scales"].view(np.float16))
    # the reference's dequantized weight, rounded once to f16; -0.0 of the exporter's copy canonicalised (the stored
    # code is Z, which unpacks to +0)
    want = (G[f"q{bits}_deq"] + np.float32(0.0)).astype(np.float16).view(np.uint16)
    return codes, scales, want


def test_fixture_holds_the_extremes():
    c8 = G["q8_codes"]
    c4 = G["q4_codes"].reshape(N, -1)
    assert c8.min() == 1 and c8.max() == 255
    nib = np.concatenate([c4 & 15, c4 >> 4])
    assert nib.min() == 0 and nib.max() == 15


@pytest.mark.parametrize("bits", [8, 4])
def test_dequant_reference_codes_bit_exact(ctx, dev, bits):
    import torch
    codes, scales, want = _table(bits)
    out = torch.full((N, K), -1, dtype=torch.int16, device=dev)
    ctx.call("dequant", to_dev(codes, dev), to_dev(scales, dev), out, N, K, bits)
    ctx.sync(60000)
    got = out.cpu().numpy().view(np.uint16)
    got = np.where(got == 0x8000, 0, got)  # sign of zero canonicalised on both sides
    want = np.where(want == 0x8000, 0, want)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("bits", [8, 4])
def test_gather_reference_codes_bit_exact(ctx, dev, bits):
    """Every row of the reference-quantized table, some twice, in shuffled order."""
    import torch
    codes, scales, want = _table(bits)
    ids = np.random.default_rng(bits).permutation(np.concatenate([np.arange(N), np.arange(0, N, 3)])).astype(np.int32)
    T = ids.size
    dX = torch.full((T, K), -1, dtype=torch.int16, device=dev)
    ctx.call("gather", to_dev(ids, dev), to_dev(codes, dev), to_dev(scales, dev), dX, T, K, bits)
    ctx.sync(60000)
    got = dX.cpu().numpy().view(np.uint16)
    got = np.where(got == 0x8000, 0, got)
    want = np.where(want == 0x8000, 0, want)[ids]
    assert np.array_equal(got, want)


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("form,M", [(5, 1), (5, 16), (1, 40), (4, 100), (0, 300), (2, 300), (3, 520), (6, 300),
                                    (7, 520)])
def test_qmatmul_reference_codes(ctx, dev, oracle, bits, form, M):
    """Every matmul form over the reference-quantized weight (48 rows: one ragged weight tile)."""
    import torch
    codes, scales, _ = _table(bits)
    X = np.random.default_rng(M + bits).standard_normal((M, K)).astype(np.float16)
    Y = torch.full((M, N), -1, dtype=torch.int16, device=dev)
    ctx.call("qmatmul_form", to_dev(X, dev), to_dev(codes, dev), to_dev(scales, dev), Y, M, N, K, bits, form, 0)
    ctx.sync(60000)
    got = f16_of(Y)
    ref = oracle.qmatmul(X, codes, scales, N, K, bits).view(np.float16).astype(np.float32)
    tol = 4e-3 * np.abs(ref) + 1e-3 * np.abs(ref).max()
    assert (np.abs(got - ref) <= tol).all(), rel_err(got, ref)


@pytest.mark.parametrize("bits", [8, 4])
def test_leaf_logits_reference_codes(ctx, dev, oracle, bits):
    """The readout over the reference-quantized table as a tied embedding (H = 256, every row read)."""
    import torch
    codes, scales, _ = _table(bits)
    rng = np.random.default_rng(31 + bits)
    T, L = 20, 6
    X = rng.standard_normal((T, K)).astype(np.float16)
    W = (1 + 0.1 * rng.standard_normal(K)).astype(np.float16)
    leaves = rng.integers(0, T, L).astype(np.int32)
    ids = np.arange(L * 8, dtype=np.int32).reshape(L, 8) % N
    out = torch.empty((L, 8), dtype=torch.float32, device=dev)
    ctx.call("leaf_logits", to_dev(X, dev), to_dev(leaves, dev), to_dev(W, dev), to_dev(ids, dev), to_dev(codes, dev),
             to_dev(scales, dev), out, L, K, 8, bits, 1e-6)
    ctx.sync(60000)
    assert rel_err(out.cpu().numpy(), oracle.leaf_logits(X, leaves, W, ids, codes, scales, bits, 1e-6)) < 1e-4
