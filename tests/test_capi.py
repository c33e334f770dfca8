"""CPU: the C-ABI library loads, exports every declared symbol, and rejects
bad arguments with the documented status codes before touching the GPU."""

import ctypes
import os
import re

import pytest

from conftest import REPO

HEADER = os.path.join(REPO, "include", "fast_moss_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^MOSS_API\s+[\w\s\*]+?\b(moss_\w+)\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    from fast_moss_b200 import _lib

    return _lib.load()


def test_header_declares_the_api():
    syms = declared_symbols()
    assert len(syms) >= 16
    assert "moss_rvq_encode" in syms and "moss_residual_layer_norm" in syms


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_python_binding_covers_the_header():
    from fast_moss_b200 import _lib

    assert sorted(_lib.EXPORTED) == declared_symbols()


def test_library_is_sm100a_only():
    from fast_moss_b200 import _lib

    blob = open(_lib.LIB_PATH, "rb").read()
    assert b"sm_100a" in blob


def test_version(lib):
    assert lib.moss_version() == 100


def test_bad_arguments_map_to_value_errors(lib):
    from fast_moss_b200 import _lib

    # negative sizes / zero channels are rejected before any CUDA call
    assert lib.moss_scale_add(None, 0, None, 0, None, None, -1, 4, None) == _lib.ERR_VALUE
    assert lib.moss_scale_add(None, 0, None, 0, None, None, 8, 0, None) == _lib.ERR_VALUE
    assert lib.moss_scale_add(None, 7, None, 0, None, None, 8, 4, None) == _lib.ERR_VALUE
    assert b"dtype" in lib.moss_last_error()
    # odd head dim
    s = _lib.strides([0, 0, 0, 1])
    assert lib.moss_rotate(None, None, 1, None, None, None, None, 1, 1, 1, 3, s, s,
                           None) == _lib.ERR_VALUE
    # unsupported widths are distinguished from invalid ones
    assert lib.moss_layer_norm(ctypes.c_void_p(16), None, None, 1e-5, 4, 6, ctypes.c_void_p(16),
                               None, None, None) == _lib.ERR_UNSUPPORTED
    assert lib.moss_rvq_encode(None, 8, 32, None, None, None, None, 1, 4, None, None, None,
                               None) == _lib.ERR_UNSUPPORTED
    assert lib.moss_lfq_select(None, None, None, None, None, None, 1, 8, 1, 70000, 0, None, None,
                               None) == _lib.ERR_VALUE
    # empty inputs are a no-op success
    assert lib.moss_scale_add(None, 0, None, 0, None, None, 0, 4, None) == _lib.OK
    # k-major copy + tensor-core tile images (256 codes x (64 dims + an 8-wide
    # norm block) each), codes padded to a multiple of 256
    assert lib.moss_rvq_packed_floats(32, 1000, 64) == 32 * 1024 * 64 + 32 * 4 * 256 * 72
    assert lib.moss_rvq_encode_ffma(None, 8, 32, None, None, None, None, 1, 4, None, None, None,
                                    None) == _lib.ERR_UNSUPPORTED
    # the Linear covers k % 64 == 0 and n % 128 == 0; the K split of the
    # stack's shapes (148 SMs): 8 CTAs per 1280-wide output, 4 for qkv
    assert lib.moss_linear(None, 4, 96, None, 128, None, 0, 0, None, None) == _lib.ERR_UNSUPPORTED
    assert lib.moss_linear(None, 4, 128, None, 100, None, 0, 0, None, None) == _lib.ERR_UNSUPPORTED
    assert lib.moss_linear(None, 4, 128, None, 128, None, 5, 0, None, None) == _lib.ERR_VALUE
    assert lib.moss_linear(None, 0, 128, None, 128, None, 0, 0, None, None) == _lib.OK
    assert lib.moss_linear(None, 4, 128, None, 128, None, 0, 0, None, None) == _lib.ERR_VALUE
    assert lib.moss_linear_pack_weight(None, 100, 128, None, None) == _lib.ERR_UNSUPPORTED
    assert lib.moss_linear_pack_weight(None, 128, 128, None, None) == _lib.ERR_VALUE
    # the bounded-wait self-test takes limits of 1 us to 100 ms only
    assert lib.moss_test_bounded_wait(10, 0, None) == _lib.ERR_VALUE
    assert lib.moss_test_bounded_wait(10**9, 0, None) == _lib.ERR_VALUE
    # the history attention holds at most 512 slots per thread block: larger
    # rings are rejected before any launch (null pointers are never read)
    assert lib.moss_history_attention(None, None, None, None, None, 2, 20, 4, 513, 64, 250,
                                      0.125, None, None) == _lib.ERR_UNSUPPORTED
    assert b"512" in lib.moss_last_error()
    assert lib.moss_history_attention(None, None, None, None, None, 2, 20, 4, 512, 64, 250,
                                      0.125, None, None) == _lib.ERR_VALUE


def test_python_wrappers_raise_reference_exceptions():
    import torch

    import fast_moss_b200 as fm

    x = torch.zeros(2, 4, 8)
    with pytest.raises(ValueError, match="rotary"):
        fm.rotate(torch.zeros(2, 3), x, x, x)
    with pytest.raises(ValueError, match="channel scale"):
        fm.scale_add(x, x, torch.zeros(3))
    with pytest.raises(ValueError):
        fm.prepare(torch.zeros(1, 8, 4))  # CPU tensor
    with pytest.raises(ValueError, match="B,D,T"):
        fm.select(x, x, x, torch.zeros(3), x)


def test_static_quantizer_rejects_sizes_beyond_its_scratch(lib):
    """moss_rvq_encode_static checks sizes before any device work."""
    from fast_moss_b200 import _lib

    for stages, k, d in ((33, 1024, 64), (32, 1025, 64), (4, 16, 32)):
        st = lib.moss_rvq_encode_static(None, 10, d, None, stages, k, None, None, None, None)
        assert st == _lib.ERR_UNSUPPORTED
        assert b"static scratch" in lib.moss_last_error()
    for stages, k, d in ((0, 16, 64), (4, 0, 64), (4, 16, 0)):
        st = lib.moss_rvq_encode_static(None, 10, d, None, stages, k, None, None, None, None)
        assert st == _lib.ERR_VALUE
    st = lib.moss_rvq_encode_static(None, -1, 64, None, 4, 16, None, None, None, None)
    assert st == _lib.ERR_VALUE
