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
    assert lib().dc_selftest_wait(None, 0) == DC_EINVAL and "limit_us" in lib().dc_last_error().decode()
    assert lib().dc_selftest_wait(None, 1000) == DC_EINVAL and "null context" in lib().dc_last_error().decode()


def test_misaligned_pointers_rejected_before_device_use(pkg):
    """The kernels move rows in 16-byte vectors; every entry point checks its pointers' alignment on the host before
    it touches the context, so a misaligned view is DC_EINVAL with a message instead of a device fault. The pointers
    here are never dereferenced: the calls return before any device work (the context is null)."""
    from decision_js_b200._lib import DC_EINVAL, lib
    A, B = 0x10000, 0x10002  # 16-byte aligned; 2 bytes past a boundary
    f = lib()
    calls = {
        "qmatmul": lambda p: f.dc_qmatmul(None, A, A, A, p, 4, 128, 256, 8, 0),
        "qmatmul X": lambda p: f.dc_qmatmul(None, p, A, A, A, 4, 128, 256, 8, 0),
        "qmatmul_form": lambda p: f.dc_qmatmul_form(None, A, p, A, A, 4, 128, 256, 8, 5, 0),
        "dequant": lambda p: f.dc_dequant(None, A, A, p, 128, 256, 8),
        "dequant codes": lambda p: f.dc_dequant(None, p, A, A, 128, 256, 8),
        "add_rmsnorm": lambda p: f.dc_add_rmsnorm(None, A, p, A, A, 4, 256, 1, 1e-6),
        "add_rmsnorm W": lambda p: f.dc_add_rmsnorm(None, A, None, p, A, 4, 256, 0, 1e-6),
        "sandwich": lambda p: f.dc_sandwich(None, A, A, A, p, A, 4, 256, 1e-6, 1.0),
        "qkv_norm_rope": lambda p: f.dc_qkv_norm_rope(None, p, A, A, A, 4, 8, 2, 128, 1e-6, 1e4, 0),
        "qkv_norm_rope kn": lambda p: f.dc_qkv_norm_rope(None, A, A, p, A, 4, 8, 2, 128, 1e-6, 1e4, 0),
        "attention": lambda p: f.dc_attention(None, A, A, p, 4, 8, 2, 128, 0.1),
        "attention_form": lambda p: f.dc_attention_form(None, p, A, A, 4, 8, 2, 128, 0.1, 0),
        "glu": lambda p: f.dc_glu(None, p, A, 4, 256, 0),
        "gather": lambda p: f.dc_gather(None, A, A, A, p, 4, 256, 8),
        "gather codes": lambda p: f.dc_gather(None, A, 0x10004, A, A, 4, 256, 8),
        "pool": lambda p: f.dc_pool(None, p, A, None, A, 2, 256, 0),
        "leaf_logits": lambda p: f.dc_leaf_logits(None, A, A, A, A, A, 0x10001, A, 2, 256, 4, 8, 1e-6),
        "short_conv": lambda p: f.dc_short_conv(None, A, A, A, p, 4, 256),
        "short_conv taps": lambda p: f.dc_short_conv(None, A, A, p, A, 4, 256),
        "ple_mix": lambda p: f.dc_ple_mix(None, A, p, A, A, 4, 512, 1e-6),
        "readout": lambda p: f.dc_readout(None, p, A, A, A, 4, 256, 8, 4),
    }
    for name, call in calls.items():
        assert call(B) == DC_EINVAL, name
        assert "aligned" in f.dc_last_error().decode(), (name, f.dc_last_error())
        # the same call with aligned pointers passes the checks and stops at the null context
        if name in ("gather codes", "leaf_logits"):
            continue
        assert call(A) == DC_EINVAL, name
        assert "null context" in f.dc_last_error().decode(), (name, f.dc_last_error())
    # q4 codes only need 4 bytes (one word of 8 codes): 4 past a boundary passes the checks
    assert f.dc_gather(None, A, 0x10004, A, A, 4, 256, 4) == DC_EINVAL
    assert "null context" in f.dc_last_error().decode()
    assert f.dc_qmatmul_skinny_noalloc(None, A, A, 0x10001, A, 4, 128, 256, 8, 1) == DC_EINVAL
    assert "aligned" in f.dc_last_error().decode()


def test_width_limits_checked_on_host(pkg):
    """Shapes past what a kernel's shared memory holds are refused on the host with the limit in the message (pool:
    9 H floats per CTA; readout: H floats)."""
    from decision_js_b200._lib import DC_EINVAL, lib
    A, f = 0x10000, lib()
    assert f.dc_pool(None, A, A, None, A, 2, 6408, 0) == DC_EINVAL
    assert "6400" in f.dc_last_error().decode()
    assert f.dc_pool(None, A, A, None, A, 2, 6400, 0) == DC_EINVAL
    assert "null context" in f.dc_last_error().decode()
    assert f.dc_leaf_logits(None, A, A, A, A, A, A, A, 2, 16416, 4, 8, 1e-6) == DC_EINVAL
    assert "bad arguments" in f.dc_last_error().decode()
    assert f.dc_ple_mix(None, A, A, A, A, 4, 1032, 1e-6) == DC_EINVAL
    assert "1024" in f.dc_last_error().decode()
    assert f.dc_short_conv(None, A, A, A, A, 4, 100) == DC_EINVAL
    assert "multiple of 8" in f.dc_last_error().decode()


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
    bad = json.loads(json.dumps(good))
    bad["tensors"]["w"]["scales"] = 1023  # f16 scales at an odd byte
    bad["bytes"] = 1023 + 64
    assert lib().dc_check_weights(_write(tmp_path / "odd_scales", bad, blob)) == DC_EFORMAT
    assert "aligned" in lib().dc_last_error().decode()
    bad = json.loads(json.dumps(good))
    bad["tensors"]["n"] = {"dtype": "f16", "shape": [8], "offset": 1032, "bytes": 16}  # not on a 16-byte boundary
    assert lib().dc_check_weights(_write(tmp_path / "f16_off", bad, blob)) == DC_EFORMAT
    assert "16-byte" in lib().dc_last_error().decode()
    ok = json.loads(json.dumps(good))
    ok["tensors"]["n"] = {"dtype": "f16", "shape": [8], "offset": 1024 + 32, "bytes": 16}
    assert lib().dc_check_weights(_write(tmp_path / "f16_ok", ok, blob)) == 0
    assert lib().dc_check_weights(str(tmp_path / "missing").encode()) == DC_EIO


def test_decision_load_missing_dir(pkg, tmp_path):
    with pytest.raises(pkg.DecisionError) as e:
        pkg.Decision.load(str(tmp_path / "nothing"))
    assert str(e.value).startswith("decision.js:")
