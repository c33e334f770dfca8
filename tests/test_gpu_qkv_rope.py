"""GPU: the fused qkv projection + rotary embedding + history writes
(`moss_qkv_rope`, tcgen05 bf16 GEMM with the rotation in its epilogue)
against the unfused path it replaces: F.linear (cuBLAS) followed by
`rope_kv` (fast_moss/v2_runtime.py:104 and :186-224).

Bars: bit-exact where the projection's sums are exact in any order
(integer-valued operands), and on random operands every element within
2 bf16 ulps with almost all bits equal (the dot products are summed in
another order than cuBLAS's)."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _unfused(x, w, bias, h, offset, slots, k_cache, v_cache, moss):
    b, t, _ = x.shape
    qkv = F.linear(x, w, bias).view(b, t, 3, h, 64)
    return moss.rope_kv(qkv[:, :, 0].transpose(1, 2), qkv[:, :, 1].transpose(1, 2),
                        qkv[:, :, 2].transpose(1, 2), offset, 10000.0, slots, k_cache, v_cache)


def _case(cuda_device, b, t, h, k, integer, seed):
    g = torch.Generator().manual_seed(seed)
    slots_total = t + 7  # a ring longer than the chunk: no two tokens share a slot
    n = 3 * h * 64
    if integer:
        x = torch.randint(-2, 3, (b, t, k), generator=g).float()
        w = torch.randint(-1, 2, (n, k), generator=g).float()
        bias = torch.randint(-4, 5, (n,), generator=g).float()
    else:
        x = torch.randn(b, t, k, generator=g)
        w = 0.02 * torch.randn(n, k, generator=g)
        bias = 0.02 * torch.randn(n, generator=g)
    offset = torch.randint(0, 5000, (b,), generator=g)
    slots = (offset[:, None] + torch.arange(t)) % slots_total
    to = lambda v, dt=torch.bfloat16: v.to(cuda_device, dt)
    return (to(x), to(w), to(bias), to(offset, torch.int64), to(slots, torch.int64),
            slots_total)


def _both(moss, cuda_device, case, h):
    x, w, bias, offset, slots, total = case
    b, t, _ = x.shape
    caches = [torch.zeros(b, h, total, 64, device=cuda_device, dtype=torch.bfloat16)
              for _ in range(4)]
    prev = torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
    try:
        q_ref = _unfused(x, w, bias, h, offset, slots, caches[0], caches[1], moss)
    finally:
        torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = prev
    image = moss.pack_qkv_weight(w)
    q = moss.qkv_rope(x, image, bias, h, offset, 10000.0, slots, caches[2], caches[3])
    torch.cuda.synchronize()
    from fast_moss_b200 import _lib
    _lib.check(_lib.load().moss_check_device_error(None), "device error word")
    return (q, caches[2], caches[3]), (q_ref, caches[0], caches[1])


@pytest.mark.parametrize("b,t,h,k", [(1, 4, 20, 1280), (64, 4, 20, 1280), (70, 4, 2, 256),
                                     (3, 1, 1, 64), (2, 129, 3, 128)])
def test_qkv_rope_bit_exact_on_exact_sums(moss, cuda_device, b, t, h, k):
    """Integer operands: every partial sum is an exact float32 integer, so
    any summation order gives the same projection, and the fused epilogue
    (bias, bf16 rounding, phase, rotation, ring writes) must reproduce the
    unfused bits."""
    got, want = _both(moss, cuda_device, _case(cuda_device, b, t, h, k, True, b + t + h), h)
    for g, w_ in zip(got, want):
        assert torch.equal(g.view(torch.int16), w_.view(torch.int16))


@pytest.mark.parametrize("b,t,h,k", [(1, 4, 20, 1280), (64, 4, 20, 1280), (33, 4, 4, 512)])
def test_qkv_rope_random_within_two_ulps(moss, cuda_device, b, t, h, k):
    got, want = _both(moss, cuda_device, _case(cuda_device, b, t, h, k, False, 7 * b + h), h)
    for g, w_ in zip(got, want):
        g, w_ = g.float(), w_.float()
        mag = torch.maximum(g.abs(), w_.abs()).clamp_min(2.0 ** -126)
        ulp = torch.exp2(torch.floor(torch.log2(mag)) - 7)
        assert torch.all((g - w_).abs() <= 2 * ulp)
        assert (g == w_).float().mean() > 0.98


def test_qkv_rope_reports_a_slot_out_of_range(moss, cuda_device):
    from fast_moss_b200 import _lib

    x, w, bias, offset, slots, total = _case(cuda_device, 2, 4, 2, 128, True, 3)
    slots[1, 2] = total  # one bad slot
    k_cache = torch.zeros(2, 2, total, 64, device=cuda_device, dtype=torch.bfloat16)
    v_cache = torch.zeros_like(k_cache)
    lib = _lib.load()
    lib.moss_check_device_error(None)  # clear
    moss.qkv_rope(x, moss.pack_qkv_weight(w), bias, 2, offset, 10000.0, slots, k_cache, v_cache)
    torch.cuda.synchronize()
    assert lib.moss_check_device_error(None) != 0
    # the other rows' keys landed
    good = slots[0, 0].item()
    assert torch.count_nonzero(k_cache[0, :, good]) > 0


def test_qkv_rope_validation(moss, cuda_device):
    x = torch.zeros(1, 4, 100, device=cuda_device, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        moss.pack_qkv_weight(torch.zeros(192, 100))
    with pytest.raises(ValueError):
        moss.qkv_rope(x, torch.zeros(192 * 100, device=cuda_device, dtype=torch.bfloat16), None, 1,
                      torch.zeros(1, device=cuda_device, dtype=torch.long), 1e4,
                      torch.zeros(1, 3, device=cuda_device, dtype=torch.long),
                      torch.zeros(1, 1, 5, 64, device=cuda_device, dtype=torch.bfloat16),
                      torch.zeros(1, 1, 5, 64, device=cuda_device, dtype=torch.bfloat16))


@pytest.mark.parametrize("b,t,h,k", [(1, 4, 20, 1280), (64, 4, 20, 1280), (33, 4, 4, 512)])
def test_qkv_rope_projection_within_one_ulp_of_its_sum_bound(moss, cuda_device, b, t, h, k):
    """The values (the projection's third part, stored unrotated) isolate
    the GEMM: each is one FP32 sum of k products plus the bias, rounded once
    to bf16 in both paths.  Two summation orders differ by at most
    2 gamma_{k+1} (sum|x w| + |bias|) (gamma_n = n u / (1 - n u),
    u = 2^-24), so the bf16 results differ by at most one bf16 ulp plus
    that bound.  (The rotated q
    and k can differ by 2 ulps: a one-ulp step in an input of the rotation
    moves an output of smaller magnitude by more than one of its own ulps.)"""
    case = _case(cuda_device, b, t, h, k, False, 11 * b + h)
    got, want = _both(moss, cuda_device, case, h)
    x, w, bias, offset, slots, total = case
    gv, wv = got[2].float(), want[2].float()
    # sum |x w| of every value feature, laid out like the value ring
    mag = (x.float().abs() @ w[2 * h * 64:].float().abs().T
           + bias[2 * h * 64:].float().abs()).view(b, t, h, 64)
    sum_abs = torch.zeros_like(gv)
    for bi in range(b):
        sum_abs[bi, :, slots[bi]] = mag[bi].transpose(0, 1)
    u = 2.0 ** -24
    gamma = (k + 1) * u / (1 - (k + 1) * u)  # k products and the bias
    top = torch.maximum(gv.abs(), wv.abs()).clamp_min(2.0 ** -126)
    ulp = torch.exp2(torch.floor(torch.log2(top)) - 7)
    assert torch.all((gv - wv).abs() <= ulp + 2 * gamma * sum_abs)
    assert (gv == wv).float().mean() > 0.98
