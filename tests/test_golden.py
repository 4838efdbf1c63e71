"""The oracle and this package's quantizers, pinned against the reference's own quantizer outputs
(tests/golden/quant_golden.npz, written by tests/golden/make_golden.py from scripts/export_common.py:64-97)."""
import os

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
G = np.load(os.path.join(HERE, "golden", "quant_golden.npz"))


@pytest.mark.parametrize("bits", [8, 4])
def test_oracle_dequant_matches_reference(oracle, bits):
    """deq = f16((code - Z) * scale): the oracle's dequantisation equals the reference's dequantized weight
    (f32 codes x scale) rounded once to f16, bit for bit. The exporter's in-memory copy holds -0.0 where round()
    of a tiny negative weight gave -0; the stored code is Z and the engine's unpacking (code - Z) * scale gives
    +0 there (src/kernels.ts:296), so zeros compare with their sign canonicalised."""
    codes = G[f"q{bits}_codes"].reshape(-1)
    scales = G[f"q{bits}_scales"]
    N, K = G["w"].shape
    got = oracle.dequant(codes, scales, N, K, bits)
    want = (G[f"q{bits}_deq"] + np.float32(0.0)).astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("bits", [8, 4])
def test_numpy_dequant_matches_reference(pkg, bits):
    from decision_js_b200 import synth
    N, K = G["w"].shape
    got = synth.dequantize(G[f"q{bits}_codes"].reshape(-1), G[f"q{bits}_scales"].view(np.float16), N, K, bits)
    want = (G[f"q{bits}_deq"] + np.float32(0.0)).astype(np.float16).view(np.uint16)
    assert np.array_equal(got.view(np.uint16), want)


def test_quantize8_matches_reference(pkg):
    from decision_js_b200 import synth
    codes, scales = synth.quantize8(torch.from_numpy(G["w"]))
    assert np.array_equal(codes.reshape(-1), G["q8_codes"].reshape(-1))
    assert np.array_equal(scales.view(np.uint16).reshape(-1), G["q8_scales"].reshape(-1))


def test_quantize4_matches_reference(pkg):
    from decision_js_b200 import synth
    codes, scales = synth.quantize4(torch.from_numpy(G["w"]))
    assert np.array_equal(codes.reshape(-1), G["q4_codes"].reshape(-1))
    assert np.array_equal(scales.view(np.uint16).reshape(-1), G["q4_scales"].reshape(-1))


def test_golden_edge_blocks_present():
    """The fixture holds the edge cases it claims: an all-zero block (scale 1, codes all Z), a saturated +-127 q8
    code, and a q4 block using both extremes."""
    s8 = G["q8_scales"].view(np.float16)
    assert s8[0, 0] == 1.0 and np.all(G["q8_codes"][0, :32] == 128)
    assert G["q8_codes"].max() == 255 and G["q8_codes"].min() == 1
    c4 = G["q4_codes"].reshape(48, -1)
    nib = np.concatenate([c4 & 15, c4 >> 4])
    assert nib.min() == 0 and nib.max() == 15
