"""ctypes binding of libdecisioncuda.so (include/decision_cuda.h). Loading fails loudly when the library is
missing: there is no fallback path."""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdecisioncuda.so")

DC_OK, DC_EINVAL, DC_ENOMEM, DC_ECUDA, DC_ETIMEOUT, DC_EFORMAT, DC_EIO = range(7)
ACT_SILU, ACT_GELU_TANH, ACT_GELU_ERF = 0, 1, 2
K_QGEMM, K_QGEMV, K_ATTN, K_NORM, K_OTHER = range(5)


class DecisionError(RuntimeError):
    """A failed library call: `code` is the DC_E* status, the message starts with "decision.js:" like the
    reference's errors."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


_vp, _i, _f, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
_SIGS = {
    "dc_last_error": ([], ctypes.c_char_p),
    "dc_init": ([_i, ctypes.POINTER(_vp)], _i),
    "dc_destroy": ([_vp], _i),
    "dc_device_count": ([ctypes.POINTER(_i)], _i),
    "dc_alloc": ([_vp, _sz, ctypes.POINTER(_vp)], _i),
    "dc_free": ([_vp, _vp], _i),
    "dc_upload": ([_vp, _vp, _vp, _sz], _i),
    "dc_download": ([_vp, _vp, _vp, _sz], _i),
    "dc_memset": ([_vp, _vp, _i, _sz], _i),
    "dc_sync": ([_vp, _i], _i),
    "dc_stream": ([_vp], _vp),
    "dc_static_weights": ([_vp, _i], _i),
    "dc_selftest_wait": ([_vp, _i], _i),
    "dc_profile": ([_vp, _i], _i),
    "dc_profile_read": ([_vp, _i, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_longlong),
                         ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)], _i),
    "dc_qmatmul": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i], _i),
    "dc_qmatmul_form": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i], _i),
    "dc_dequant": ([_vp, _vp, _vp, _vp, _i, _i, _i], _i),
    "dc_qmatmul_f16": ([_vp, _vp, _vp, _vp, _i, _i, _i, _i], _i),
    "dc_qmatmul_skinny_noalloc": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i], _i),
    "dc_add_rmsnorm": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _f], _i),
    "dc_sandwich": ([_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _f, _f], _i),
    "dc_qkv_norm_rope": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _f, _i], _i),
    "dc_attention": ([_vp, _vp, _vp, _vp, _i, _i, _i, _i, _f], _i),
    "dc_attention_form": ([_vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _i], _i),
    "dc_glu": ([_vp, _vp, _vp, _i, _i, _i], _i),
    "dc_gather": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i], _i),
    "dc_pool": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i], _i),
    "dc_leaf_logits": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f], _i),
    "dc_short_conv": ([_vp, _vp, _vp, _vp, _vp, _i, _i], _i),
    "dc_ple_mix": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _f], _i),
    "dc_readout": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i], _i),
    "dc_attention_ex": ([_vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, ctypes.c_long, _i, _i], _i),
    "dc_forward_laya": ([_vp, _vp, _vp, _vp, _vp, _i, _vp, _vp, _i, _vp], _i),
    "dc_forward_omni": ([_vp, _vp, _vp, _vp, _vp, _i, _vp, _vp, _i, _vp], _i),
    "dc_forward_d3": ([_vp, _vp, _vp, _vp, _i, _vp, _i, _vp, _i, _vp], _i),
    "dc_gdn": ([_vp, _vp, ctypes.c_long, ctypes.c_long, _i, _vp, _vp, _vp, _vp, _vp, _i, _f, _vp, _i], _i),
    "dc_add_rows": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i], _i),
    "dc_bias_act": ([_vp, _vp, _vp, _i, _i, _i], _i),
    "dc_add_layernorm": ([_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _f], _i),
    "dc_gather_rows": ([_vp, _vp, _vp, _vp, _i, _i, _i], _i),
    "dc_score": ([_vp, _vp, _vp, _vp, _vp, _i, _i], _i),
    "dc_qk_rope": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, ctypes.c_long, _i, _i, _f, _f], _i),
    "dc_load_weights": ([_vp, ctypes.c_char_p, ctypes.POINTER(_vp)], _i),
    "dc_check_weights": ([ctypes.c_char_p], _i),
    "dc_model_free": ([_vp], _i),
    "dc_model_kind": ([_vp, ctypes.c_char_p, _sz], _i),
    "dc_model_config_f": ([_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)], _i),
    "dc_model_tensor": ([_vp, ctypes.c_char_p, ctypes.POINTER(_vp), ctypes.POINTER(_vp), ctypes.POINTER(_i),
                         ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64)], _i),
    "dc_forward_encoder": ([_vp, _vp, _vp, _i, _i, _vp], _i),
    "dc_forward_decoder": ([_vp, _vp, _vp, _vp, _i, _vp, _vp, _i, _i, _vp], _i),
    "dc_forward_encoder_device": ([_vp, _vp, _vp, _i, _i, _vp], _i),
    "dc_forward_decoder_device": ([_vp, _vp, _vp, _vp, _i, _vp, _vp, _i, _i, _vp], _i),
    "dc_model_context": ([_vp, ctypes.POINTER(_vp)], _i),
    "dc_eg2_head": ([_vp, _vp, _i, _vp, _i, _vp, _i, _vp, _i, _vp], _i),
}

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library, with every entry point's signature declared."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise DecisionError(DC_ECUDA, f"decision.js: {LIB_PATH} is not built (run __graft_entry__.build())")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def symbols() -> list[str]:
    return list(_SIGS)


def check(rc: int) -> None:
    if rc != DC_OK:
        raise DecisionError(rc, lib().dc_last_error().decode() or f"decision.js: error {rc}")


def ptr(x) -> int | None:
    """A device or host address from a torch tensor, numpy array, int or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if hasattr(x, "ctypes"):
        return x.ctypes.data
    raise TypeError(type(x))


class Context:
    """One dc_ctx: a CUDA device, its stream and scratch."""

    def __init__(self, device: int = 0):
        h = ctypes.c_void_p()
        check(lib().dc_init(device, ctypes.byref(h)))
        self.h = h
        self.device = device

    def close(self):
        if self.h:
            lib().dc_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream(self) -> int:
        return lib().dc_stream(self.h) or 0

    def sync(self, timeout_ms: int = -1):
        check(lib().dc_sync(self.h, timeout_ms))

    def call(self, name: str, *args):
        """Calls dc_<name>(ctx, *args), converting tensors / arrays to addresses, and raises on failure."""
        conv = [ptr(a) if not isinstance(a, (float, bool)) else a for a in args]
        check(getattr(lib(), "dc_" + name)(self.h, *conv))

    def profile(self, enable: bool):
        check(lib().dc_profile(self.h, int(enable)))

    def profile_read(self, kind: int):
        ms, n, fl, by = ctypes.c_double(), ctypes.c_longlong(), ctypes.c_double(), ctypes.c_double()
        check(lib().dc_profile_read(self.h, kind, ctypes.byref(ms), ctypes.byref(n), ctypes.byref(fl),
                                    ctypes.byref(by)))
        return {"ms": ms.value, "launches": n.value, "flops": fl.value, "bytes": by.value}


def device_count() -> int:
    n = ctypes.c_int()
    check(lib().dc_device_count(ctypes.byref(n)))
    return n.value
