"""Generates the golden quantization fixtures from the reference's own quantizers.

    python tests/golden/make_golden.py /path/to/decision.js

Imports quantize8 / quantize4 from the reference's scripts/export_common.py (lines 64-97) and records, for
seeded weights with edge-case blocks (an all-zero block, a single outlier, saturating extremes, tiny values):
the weight, the codes and f16 scales the reference writes to weights.bin, and the dequantized f32 weight the
reference computes with (codes x scale). tests/test_golden.py pins the oracle's dequantisation and this
package's quantizers against them. The fixture is small and committed; the reference is not needed to run
the tests.
"""
import os
import sys

import numpy as np
import torch


def weights():
    g = torch.Generator().manual_seed(20241201)
    w = torch.randn(48, 256, generator=g) * 0.02
    w[0, 0:32] = 0.0                                        # all-zero block
    w[1, 32:64] = 0.0
    w[1, 40] = 0.5                                          # one outlier in a zero block
    w[2, 64:96] = torch.linspace(-1.0, 1.0, 32)             # full range, exact extremes
    w[3, 96:128] = 1e-6 * torch.randn(32, generator=g)      # scale near the f16 subnormal range
    w[4, 128:160] = torch.tensor([(-1) ** i * 3.0 for i in range(32)])  # alternating saturating values
    w[5] = torch.randn(256, generator=g) * 2.0              # large row
    return w


def main(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "scripts"))
    from export_common import quantize4, quantize8  # the reference's own code

    w = weights()
    q8c, q8s, q8d = quantize8(w)
    q4c, q4s, q4d = quantize4(w)
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "quant_golden.npz")
    np.savez_compressed(out, w=w.numpy().astype(np.float32),
                        q8_codes=q8c, q8_scales=q8s.view(np.uint16), q8_deq=q8d.numpy().astype(np.float32),
                        q4_codes=q4c, q4_scales=q4s.view(np.uint16), q4_deq=q4d.numpy().astype(np.float32))
    print(out, os.path.getsize(out), "bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/decision.js")
    main(sys.argv[1])
