"""CPU: the oracle against the reference's own outputs (golden fixtures)."""

import ctypes
import os

import numpy as np
import pytest

from conftest import GOLDEN, golden, same_bits
from oracle import build_ref
from oracle import oracle as O


def test_scale_add_matches_reference_kernel():
    g = golden("scale_add.npz")
    for case in g["cases"]:
        y = O.scale_add(g[f"{case}_x"], g[f"{case}_u"], g[f"{case}_s"])
        assert same_bits(y, g[f"{case}_y"]), case


def test_rotate_matches_reference_kernel():
    g = golden("rotate.npz")
    for case in g["cases"]:
        bf16 = bool(g[f"{case}_bf16"])
        if case == "bf16_view":
            qkv = g[f"{case}_qbase"]  # [B, T, 3, H, D]
            q = qkv[:, :, 0].transpose(0, 2, 1, 3)
            k = qkv[:, :, 1].transpose(0, 2, 1, 3)
        else:
            q, k = g[f"{case}_q"], g[f"{case}_k"]
        oq, ok = O.rotate(q, k, g[f"{case}_cos"], g[f"{case}_sin"], bf16)
        assert same_bits(oq, g[f"{case}_oq"]), case
        assert same_bits(ok, g[f"{case}_ok"]), case


def test_select_matches_reference_kernel():
    g = golden("select.npz")
    for case in g["cases"]:
        ste = bool(g[f"{case}_ste"])
        out, idx = O.lfq_select(g[f"{case}_dots"], g[f"{case}_norm"].reshape(-1),
                                g[f"{case}_cnorm"].reshape(-1), g[f"{case}_book"],
                                g[f"{case}_lat"], straight_through=ste)
        assert np.array_equal(idx, g[f"{case}_idx"].reshape(-1)), case
        ref_out = g[f"{case}_out"]
        if not ste:
            ref_out = ref_out.reshape(out.shape)
        assert same_bits(out, ref_out), case


def test_select_tie_and_nan_rules():
    g = golden("select.npz")
    idx = g["plain_idx"].reshape(-1)
    assert idx[1] == 2  # first NaN wins over everything
    # row 2 has all dots = +inf -> distances -inf everywhere -> first index
    assert idx[2] == 0


def test_prepare_matches_reference_kernel():
    g = golden("prepare.npz")
    for case in g["cases"]:
        e, norm, tw, den = O.lfq_prepare(g[f"{case}_x"])
        assert same_bits(e, g[f"{case}_e"]), case
        assert same_bits(tw, g[f"{case}_twice"]), case
        assert same_bits(norm, g[f"{case}_norm"]), case
        assert same_bits(den, g[f"{case}_denom"]), case


@pytest.mark.skipif(not os.path.isdir(build_ref.DEFAULT_REFERENCE),
                    reason="reference checkout not present")
def test_prepare_matches_compiled_reference_random():
    lib = ctypes.CDLL(build_ref.build())
    rng = np.random.default_rng(7)
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    for b, t in [(1, 257), (4, 33), (1, 1), (7, 1)]:
        x = (rng.standard_normal((b, 8, t)) * rng.choice([1e-20, 1.0, 1e18], (b, 8, t))).astype(
            np.float32)
        transposed = b == 1 and t > 1
        e = np.zeros((8, t) if transposed else (b * t, 8), np.float32)
        tw, norm, den = np.zeros_like(e), np.zeros(b * t, np.float32), np.zeros(b * t, np.float32)
        lib.ref_prepare(p(x), p(e), p(norm), p(tw), p(den), ctypes.c_int(b), ctypes.c_int(t))
        oe, on, otw, od = O.lfq_prepare(x)
        assert same_bits(oe, e) and same_bits(otw, tw)
        assert same_bits(on, norm) and same_bits(od, den)


def test_rvq_loop_matches_reference_selection():
    g = golden("rvq_small.npz")
    codes, recon, res = O.rvq_encode(g["x"], g["books"], residual=True)
    assert np.array_equal(codes, g["codes"])
    assert same_bits(recon, g["recon"])
    assert same_bits(res, g["residual"])
    # the duplicated codeword 5 of stage 1 must never be chosen over code 2
    assert not np.any(codes[1] == 5)


def test_rvq_decode_inverts_encode():
    g = golden("rvq_small.npz")
    recon = O.rvq_decode(g["codes"], g["books"])
    assert same_bits(recon, g["recon"])


def test_lfq_decode_matches_reference_pipeline():
    g = golden("lfq_decode.npz")
    for case in g["cases"]:
        out, idx = O.lfq_decode(g[f"{case}_x"], g["book_normed"], g["cnorm"].reshape(-1),
                                g["weight"])
        assert np.array_equal(idx, g[f"{case}_idx"]), case
        assert same_bits(out, g[f"{case}_out"]), case


@pytest.mark.skipif(not os.path.exists(os.path.join(GOLDEN, "layer_norm_cuda.npz")),
                    reason="B200 layer-norm fixture not generated yet")
def test_layer_norm_matches_torch_cuda_fixture():
    g = golden("layer_norm_cuda.npz")
    for case in g["cases"]:
        x = g[f"{case}_x"]
        y, mean, ve, _ = O.layer_norm(x, g[f"{case}_w"], g[f"{case}_b"], float(g[f"{case}_eps"]),
                                      rstd=g[f"{case}_rstd"])
        assert same_bits(mean, g[f"{case}_mean"]), case
        assert same_bits(y, g[f"{case}_y"]), case
        # rstd is the device's rsqrtf of var+eps: within 2 ulp of the exact value
        exact = (1.0 / np.sqrt(ve.astype(np.float64))).astype(np.float32)
        ulps = np.abs(exact.view(np.int32).astype(np.int64) -
                      g[f"{case}_rstd"].astype(np.float32).view(np.int32).astype(np.int64))
        assert ulps.max() <= 2, case


def test_bf16_round_is_nearest_even():
    vals = np.array([1.0, 1.00390625, 1.005859375, 1.0078125 + 2**-9, -3.0e38, np.inf], np.float32)
    out = O.bf16_round(vals)
    assert out[0] == 1.0
    assert out[1] == 1.0  # tie -> even
    assert out[2] == np.float32(1.0078125)
    assert np.isinf(O.bf16_round(np.array([3.4e38], np.float32))[0])
