"""GPU: the tcgen05 Linear (`moss_linear`) against the path it replaces,
F.linear on cached bf16 weights (cuBLAS; fast_moss/v2_runtime.py:104), and
its activation epilogue against F.linear followed by the feed-forward's
eager bias + activation chain (`moss_gated_act`, ungated).

Bars: bit-exact where every partial sum is exact in any order
(integer-valued operands), so the kernel's tiling, K split across the
cluster, padding of the token tiles and epilogue are checked bit for bit;
on random operands every output within one bf16 ulp plus twice the FP32
summation bound gamma_{k+1} (sum|x w| + |bias|) of the two summation
orders; identical bits on repeated calls (fixed reduction order)."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

SHAPES = [  # (m, n, k): one stream, 64 streams, ragged and multi-tile token counts
    (4, 1280, 1280), (4, 3840, 1280), (4, 5120, 1280), (4, 1280, 5120),
    (256, 1280, 1280), (256, 5120, 1280), (256, 1280, 5120), (256, 3840, 1280),
    (1, 128, 64), (17, 256, 192), (300, 384, 640), (513, 128, 128),
]


def _integer_case(m, n, k, seed, device):
    g = torch.Generator().manual_seed(seed)
    x = torch.randint(-2, 3, (m, k), generator=g).to(device, torch.bfloat16)
    w = torch.randint(-1, 2, (n, k), generator=g).to(device, torch.bfloat16)
    b = torch.randint(-8, 9, (n,), generator=g).to(device, torch.bfloat16)
    return x, w, b


def _random_case(m, n, k, seed, device):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(device, torch.bfloat16)
    w = (0.02 * torch.randn(n, k, generator=g)).to(device, torch.bfloat16)
    b = (0.02 * torch.randn(n, generator=g)).to(device, torch.bfloat16)
    return x, w, b


def _cublas(x, w, b):
    prev = torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
    try:
        return F.linear(x, w, b)
    finally:
        torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = prev


def _device_errors():
    from fast_moss_b200 import _lib

    torch.cuda.synchronize()
    _lib.check(_lib.load().moss_check_device_error(None), "device error word")


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_linear_bit_exact_on_exact_sums(moss, cuda_device, m, n, k):
    from fast_moss_b200.linear import linear, pack_weight

    x, w, b = _integer_case(m, n, k, m + n + k, cuda_device)
    for bias in (b, None):
        got = linear(x, pack_weight(w), bias)
        want = _cublas(x, w, bias)
        _device_errors()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), (m, n, k, bias is None)


@pytest.mark.parametrize("act", ["gelu", "silu", "gelu_tanh"])
@pytest.mark.parametrize("m,n,k", [(4, 5120, 1280), (256, 5120, 1280), (37, 640, 256)])
def test_linear_activation_epilogue_bit_exact(moss, cuda_device, m, n, k, act):
    """Integer operands scaled by 1/16 (still exact sums): the fused
    epilogue must give the bits of F.linear (no bias) followed by the
    eager bias + activation chain."""
    from fast_moss_b200.linear import linear, pack_weight

    x, w, b = _integer_case(m, n, k, 3 * m + k, cuda_device)
    x = x * 0.0625
    b = b * 0.0625
    f = _cublas(x, w, None)
    for bias in (b, None):
        want = moss.gated_activation(f, bias, act, False)
        got = linear(x, pack_weight(w), bias, activation=act)
        _device_errors()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), (act, bias is None)


@pytest.mark.parametrize("m,n,k", SHAPES[:8])
def test_linear_random_within_one_ulp_of_the_sum_bound(moss, cuda_device, m, n, k):
    from fast_moss_b200.linear import linear, pack_weight

    x, w, b = _random_case(m, n, k, 7 * m + n, cuda_device)
    pw = pack_weight(w)
    got = linear(x, pw, b)
    again = linear(x, pw, b)
    want = _cublas(x, w, b)
    _device_errors()
    assert torch.equal(got.view(torch.int16), again.view(torch.int16))  # deterministic
    g, r = got.float(), want.float()
    sum_abs = x.float().abs() @ w.float().abs().T + b.float().abs()
    u = 2.0 ** -24
    gamma = (k + 1) * u / (1 - (k + 1) * u)
    top = torch.maximum(g.abs(), r.abs()).clamp_min(2.0 ** -126)
    ulp = torch.exp2(torch.floor(torch.log2(top)) - 7)
    assert torch.all((g - r).abs() <= ulp + 2 * gamma * sum_abs)
    assert (g == r).float().mean() > 0.97


def test_linear_leading_dims_and_out_buffer(moss, cuda_device):
    from fast_moss_b200.linear import linear, pack_weight

    x, w, b = _integer_case(12, 256, 128, 5, cuda_device)
    out = torch.full((3, 4, 256), 7.0, device=cuda_device, dtype=torch.bfloat16)
    got = linear(x.view(3, 4, 128), pack_weight(w), b, out=out)
    assert got is out
    assert torch.equal(out.view(12, 256), _cublas(x, w, b))


def test_linear_rejects_shapes_it_does_not_cover(moss, cuda_device):
    from fast_moss_b200 import _lib
    from fast_moss_b200.linear import linear, pack_weight

    with pytest.raises(_lib.UnsupportedError):
        pack_weight(torch.zeros(128, 96, device=cuda_device, dtype=torch.bfloat16))
    with pytest.raises(_lib.UnsupportedError):
        pack_weight(torch.zeros(100, 128, device=cuda_device, dtype=torch.bfloat16))
    x = torch.zeros(4, 128, device=cuda_device, dtype=torch.bfloat16)
    pw = pack_weight(torch.zeros(128, 128, device=cuda_device, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        linear(x.float(), pw)
    with pytest.raises(ValueError):
        linear(x, torch.zeros(128, 128, device=cuda_device, dtype=torch.bfloat16))  # not packed
    empty = linear(x[:0], pw)
    assert empty.shape == (0, 128)
