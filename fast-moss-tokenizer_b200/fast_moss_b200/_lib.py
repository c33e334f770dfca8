"""ctypes binding of libfast_moss_b200.so (the C ABI in include/fast_moss_b200.h).

The library is required: importing a kernel wrapper without it raises
immediately, and no operation falls back to another implementation when the
library is missing.  Status codes become the exception classes the
reference raises for the same situations (ValueError for bad input,
RuntimeError otherwise).
"""

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libfast_moss_b200.so")

OK = 0
ERR_VALUE = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_TIMEOUT = 4

F32 = 0
BF16 = 1

ACT_SILU = 0
ACT_GELU_ERF = 1
ACT_GELU_TANH = 2

LINEAR_BIAS = 0
LINEAR_BIAS_ACT = 1


class UnsupportedError(ValueError):
    """Valid input that the B200 kernels do not cover (caller may fall back to
    the upstream module, as the reference's guards do)."""


_vp = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float
_pi64 = ctypes.POINTER(ctypes.c_int64)

_SIGNATURES = {
    "moss_version": (_i, []),
    "moss_last_error": (ctypes.c_char_p, []),
    "moss_check_device_error": (_i, [_vp]),
    "moss_test_bounded_wait": (_i, [_i64, _i, _vp]),
    "moss_scale_add": (_i, [_vp, _i, _vp, _i, _vp, _vp, _i64, _i64, _vp]),
    "moss_layer_norm": (_i, [_vp, _vp, _vp, _f, _i64, _i64, _vp, _vp, _vp, _vp]),
    "moss_residual_layer_norm": (
        _i, [_vp, _i, _vp, _i, _vp, _vp, _vp, _f, _i64, _i64, _vp, _vp, _vp, _vp, _vp]),
    "moss_residual_layer_norm_out": (
        _i, [_vp, _i, _vp, _i, _vp, _vp, _vp, _f, _i64, _i64, _vp, _vp, _i, _vp, _vp, _vp]),
    "moss_rotate": (_i, [_vp, _vp, _i, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _pi64, _pi64,
                         _vp]),
    "moss_rope": (_i, [_vp, _vp, _i, _vp, _i, _f, _vp, _vp, _i64, _i64, _i64, _i64, _pi64, _pi64,
                       _vp]),
    "moss_rope_kv": (_i, [_vp, _vp, _vp, _i, _vp, _i, _f, _vp, _vp, _vp, _vp, _i64, _i64, _i64,
                          _i64, _i64, _pi64, _pi64, _pi64, _vp]),
    "moss_qkv_rope": (_i, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i, _f, _vp, _vp, _vp, _vp,
                           _i64, _vp]),
    "moss_history_attention": (_i, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64,
                                    _f, _vp, _vp]),
    "moss_history_attention_qkv": (_i, [_vp, _vp, _f, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                                        _i64, _i64, _f, _vp, _vp]),
    "moss_gated_act": (_i, [_vp, _vp, _vp, _i, _i64, _i64, _i, _i, _vp]),
    "moss_linear_pack_weight": (_i, [_vp, _i64, _i64, _vp, _vp]),
    "moss_linear": (_i, [_vp, _i64, _i64, _vp, _i64, _vp, _i, _i, _vp, _vp]),
    "moss_linear_cluster": (_i, [_i64, _i64, _i64]),
    "moss_lfq_prepare": (_i, [_vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp]),
    "moss_lfq_select": (_i, [_vp, _vp, _vp, _vp, _vp, _pi64, _i64, _i64, _i64, _i64, _i, _vp, _vp,
                             _vp]),
    "moss_lfq_decode": (_i, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp]),
    "moss_lfq_rvq_encode": (_i, [_vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp,
                                 _vp, _vp, _vp, _vp]),
    "moss_rvq_packed_floats": (_i64, [_i64, _i64, _i64]),
    "moss_rvq_prepare_codebooks": (_i, [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp]),
    "moss_rvq_encode": (_i, [_vp, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp]),
    "moss_rvq_encode_kernel": (_i, [_vp, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp,
                                    _i, _vp]),
    "moss_rvq_encode_static": (_i, [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _vp]),
    "moss_rvq_encode_ffma": (_i, [_vp, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp,
                                  _vp]),
    "moss_rvq_decode": (_i, [_vp, _i64, _vp, _i64, _i64, _i64, _vp, _vp]),
}

EXPORTED = tuple(_SIGNATURES)

_lib = None


def load():
    """Loads the native library (once) and declares every entry point."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"fast_moss_b200 native library not built ({LIB_PATH}); run "
                "`python fast-moss-tokenizer_b200/build.py` (needs nvcc)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(status, what):
    """Raises the exception that matches a non-OK status."""
    if status == OK:
        return
    msg = load().moss_last_error().decode(errors="replace")
    if status == ERR_VALUE:
        raise ValueError(msg)
    if status == ERR_UNSUPPORTED:
        raise UnsupportedError(msg)
    raise RuntimeError(f"{what}: {msg}")


def call(name, *args):
    """Calls entry point `name` and raises on a non-OK status."""
    check(getattr(load(), name)(*args), name)


def strides(values):
    arr = (ctypes.c_int64 * len(values))(*[int(v) for v in values])
    return arr
