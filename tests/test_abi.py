"""The C ABI without a GPU: the library loads, exports every entry point include/*.h declares, and the calls that
need no device behave (errors, device count, manifest validation)."""
import ctypes
import glob
import json
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        names |= set(re.findall(r"DC_API\s+[\w\s\*]+?\b(dc_\w+)\s*\(", open(h).read()))
    return names


def test_header_declares_entry_points():
    names = _declared()
    assert {"dc_init", "dc_qmatmul", "dc_attention", "dc_load_weights", "dc_forward_encoder",
            "dc_forward_decoder"} <= names


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.lib()
    for name in _declared():
        assert hasattr(lib, name), name
    # and the binding declares signatures for all of them
    from decision_js_b200._lib import symbols
    assert _declared() <= set(symbols())


def test_no_device_calls_fail_cleanly(pkg):
    from decision_js_b200._lib import DC_ECUDA, DC_EINVAL, lib
    n = ctypes.c_int(-1)
    assert lib().dc_device_count(ctypes.byref(n)) == 0
    if n.value == 0:
        h = ctypes.c_void_p()
        rc = lib().dc_init(0, ctypes.byref(h))
        assert rc == DC_ECUDA and not h.value
        assert lib().dc_last_error().decode().startswith("decision.js:")
    assert lib().dc_qmatmul(None, None, None, None, None, 1, 1, 32, 8, 0) == DC_EINVAL
    assert lib().dc_static_weights(None, 1) == DC_EINVAL


def _write(tmp, manifest, blob=b""):
    os.makedirs(tmp, exist_ok=True)
    with open(os.path.join(tmp, "manifest.json"), "w") as f:
        f.write(manifest if isinstance(manifest, str) else json.dumps(manifest))
    with open(os.path.join(tmp, "weights.bin"), "wb") as f:
        f.write(blob)
    return str(tmp).encode()


def test_check_weights_accepts_synthetic_model(pkg, tmp_path):
    from decision_js_b200 import synth
    synth.write_encoder(str(tmp_path), layers=1, vocab=256)
    assert pkg.lib().dc_check_weights(str(tmp_path).encode()) == 0


def test_check_weights_failures(pkg, tmp_path):
    """Host-side fault injection on the loader (the reference throws on a short range read, src/gpu.ts:66, and on a
    bad manifest): truncated weights.bin -> DC_EIO, malformed JSON / dtype / shape / scales -> DC_EFORMAT."""
    from decision_js_b200._lib import DC_EFORMAT, DC_EIO, lib
    good = {"format": "d1.js/1", "config": {}, "bytes": 1024 + 64,
            "tensors": {"w": {"dtype": "q8", "shape": [4, 256], "offset": 0, "bytes": 1024, "scales": 1024,
                              "scales_bytes": 64}}}
    blob = bytes(1024 + 64)
    assert lib().dc_check_weights(_write(tmp_path / "ok", good, blob)) == 0
    assert lib().dc_check_weights(_write(tmp_path / "trunc", good, blob[:1000])) == DC_EIO
    assert "weights.bin" in lib().dc_last_error().decode()
    assert lib().dc_check_weights(_write(tmp_path / "json", "{not json", blob)) == DC_EFORMAT
    bad = json.loads(json.dumps(good))
    bad["tensors"]["w"]["dtype"] = "q3"
    assert lib().dc_check_weights(_write(tmp_path / "dtype", bad, blob)) == DC_EFORMAT
    bad = json.loads(json.dumps(good))
    bad["tensors"]["w"]["bytes"] = 1000
    assert lib().dc_check_weights(_write(tmp_path / "bytes", bad, blob)) == DC_EFORMAT
    bad = json.loads(json.dumps(good))
    bad["tensors"]["w"]["scales_bytes"] = 32
    assert lib().dc_check_weights(_write(tmp_path / "scales", bad, blob)) == DC_EFORMAT
    bad = json.loads(json.dumps(good))
    bad["tensors"]["w"]["shape"] = [4, 250]
    bad["tensors"]["w"]["bytes"] = 1000
    assert lib().dc_check_weights(_write(tmp_path / "k32", bad, blob)) == DC_EFORMAT
    assert lib().dc_check_weights(str(tmp_path / "missing").encode()) == DC_EIO


def test_decision_load_missing_dir(pkg, tmp_path):
    with pytest.raises(pkg.DecisionError) as e:
        pkg.Decision.load(str(tmp_path / "nothing"))
    assert str(e.value).startswith("decision.js:")
