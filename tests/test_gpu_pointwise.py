"""GPU parity: residual scale-add, RoPE (tables and in-kernel phase), gated
activation.

Bars: scale_add / rotate bit-exact against the reference's kernels (golden
fixtures) and the oracle; the in-kernel RoPE phase bit-exact against the
reference's torch table construction on the same device; bf16 pointwise
within 1 bf16 ulp of the oracle (and bit-exact against torch's eager CUDA
chain, which uses the same math library).
"""

import math

import numpy as np
import pytest
import torch

from conftest import bf16_ulp_diff, golden, same_bits
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def dev(a, device, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device=device, dtype=dtype)


def test_scale_add_golden(moss, cuda_device):
    g = golden("scale_add.npz")
    for case in g["cases"]:
        xd = torch.bfloat16 if bool(g[f"{case}_xbf16"]) else torch.float32
        ud = torch.bfloat16 if bool(g[f"{case}_ubf16"]) else torch.float32
        y = moss.scale_add(dev(g[f"{case}_x"], cuda_device, xd), dev(g[f"{case}_u"], cuda_device, ud),
                           dev(g[f"{case}_s"], cuda_device))
        assert same_bits(y.cpu().numpy(), g[f"{case}_y"]), case


def test_scale_add_random_and_strided(moss, cuda_device):
    g = torch.Generator().manual_seed(11)
    for shape in [(1, 4096, 1024), (3, 7, 1280), (5, 33), (2, 3, 6)]:
        x = torch.randn(*shape, generator=g).to(cuda_device)
        u = torch.randn(*shape, generator=g).to(cuda_device, torch.bfloat16)
        s = torch.randn(shape[-1], generator=g).to(cuda_device)
        y = moss.scale_add(x, u, s)
        ref = O.scale_add(x.cpu().numpy(), u.float().cpu().numpy(), s.cpu().numpy())
        assert same_bits(y.cpu().numpy(), ref), shape
    # non-contiguous views give the same values as their contiguous copies
    x = torch.randn(8, 64, generator=g).to(cuda_device).t()
    u = torch.randn(8, 64, generator=g).to(cuda_device).t()
    s = torch.randn(8, generator=g).to(cuda_device)
    assert torch.equal(moss.scale_add(x, u, s), moss.scale_add(x.contiguous(), u.contiguous(), s))


def test_rotate_golden(moss, cuda_device):
    g = golden("rotate.npz")
    for case in g["cases"]:
        bf16 = bool(g[f"{case}_bf16"])
        dt = torch.bfloat16 if bf16 else torch.float32
        if case == "bf16_view":
            qkv = dev(g[f"{case}_qbase"], cuda_device, dt)
            q, k = qkv[:, :, 0].transpose(1, 2), qkv[:, :, 1].transpose(1, 2)
        else:
            q, k = dev(g[f"{case}_q"], cuda_device, dt), dev(g[f"{case}_k"], cuda_device, dt)
        oq, ok = moss.rotate(q, k, dev(g[f"{case}_cos"], cuda_device), dev(g[f"{case}_sin"], cuda_device))
        assert oq.is_contiguous() and oq.dtype == dt
        assert same_bits(oq.float().cpu().numpy(), g[f"{case}_oq"]), case
        assert same_bits(ok.float().cpu().numpy(), g[f"{case}_ok"]), case


def reference_tables(offset, t, d, period, device):
    """The reference's rotary table construction (fast_moss/v2_runtime.py:214-222)."""
    b = offset.numel()
    ds = torch.arange(d // 2, device=device, dtype=torch.float32)
    freq = torch.exp(ds * (-math.log(period) * 2 / d))
    ts = offset.float().view(-1, 1) + torch.arange(t, device=device, dtype=torch.float32)
    phase = freq * ts.view(b, t, 1)
    return torch.cos(phase), torch.sin(phase)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rope_config3_matches_reference_tables(moss, cuda_device, dtype):
    b, h, t, d = 4, 16, 2048, 64
    g = torch.Generator().manual_seed(3)
    qkv = torch.randn(b, t, 3, h, d, generator=g).to(cuda_device, dtype)
    q, k = qkv[:, :, 0].transpose(1, 2), qkv[:, :, 1].transpose(1, 2)
    offset = torch.zeros(b, dtype=torch.long, device=cuda_device)
    cos, sin = reference_tables(offset, t, d, 10000.0, cuda_device)
    rq, rk = moss.rotate(q, k, cos, sin)
    fq, fk = moss.rope(q, k, offset, 10000.0)
    assert torch.equal(fq.view(torch.int16 if dtype == torch.bfloat16 else torch.int32),
                       rq.view(torch.int16 if dtype == torch.bfloat16 else torch.int32))
    assert torch.equal(fk.view(torch.int16 if dtype == torch.bfloat16 else torch.int32),
                       rk.view(torch.int16 if dtype == torch.bfloat16 else torch.int32))
    # rotation itself against the oracle, on a slice
    sl = slice(0, 64)
    oq, ok = O.rotate(q[:, :, sl].float().cpu().numpy(), k[:, :, sl].float().cpu().numpy(),
                      cos[:, sl].cpu().numpy(), sin[:, sl].cpu().numpy(), dtype == torch.bfloat16)
    assert same_bits(rq[:, :, sl].float().cpu().numpy(), oq)
    assert same_bits(rk[:, :, sl].float().cpu().numpy(), ok)


def test_rope_phase_tables_bit_exact(moss, cuda_device):
    """With q = (1, 0) pairs the f32 rotation returns (cos, sin) exactly, which
    exposes the in-kernel tables for a direct comparison."""
    b, h, t, d = 3, 1, 700, 128
    q = torch.zeros(b, h, t, d, device=cuda_device)
    q[..., 0::2] = 1.0
    for offset in (torch.tensor([0, 5, 123456], device=cuda_device),
                   torch.tensor([7, 0, 3], device=cuda_device, dtype=torch.int32),
                   torch.tensor([0.0, 2.0, 1e5], device=cuda_device)):
        oq, _ = moss.rope(q, q, offset, 10000.0)
        cos, sin = reference_tables(offset, t, d, 10000.0, cuda_device)
        assert torch.equal(oq[:, 0, :, 0::2], cos)
        assert torch.equal(oq[:, 0, :, 1::2], sin)
        ocs, osn = O.rope_tables(offset.float().cpu().numpy(), t, d,
                                 np.float32(-math.log(10000.0) * 2 / d))
        # CUDA's expf may differ from double libm by an ulp of freq, which
        # moves the phase by up to ~2 ulps of the phase itself.
        ts = offset.float().cpu().numpy()[:, None] + np.arange(t, dtype=np.float32)
        tol = 4 * np.spacing(np.abs(ts[..., None]).astype(np.float32)) + 2e-6
        assert np.all(np.abs(ocs - cos.cpu().numpy()) <= tol)
        assert np.all(np.abs(osn - sin.cpu().numpy()) <= tol)


def test_rope_generic_strides(moss, cuda_device):
    g = torch.Generator().manual_seed(5)
    base = torch.randn(2, 6, 5, 4, 10, generator=g).to(cuda_device, torch.bfloat16)
    q = base[..., 0, :].permute(0, 2, 1, 3)  # [2,5,6,10], innermost stride 1
    k = base[..., 1, :].permute(0, 2, 1, 3).flip(-1)  # innermost stride -1
    offset = torch.tensor([3, 0], device=cuda_device)
    cos, sin = reference_tables(offset, 6, 10, 500.0, cuda_device)
    oq, ok = moss.rotate(q, k, cos, sin)
    rq, rk = O.rotate(q.float().cpu().numpy(), k.float().cpu().numpy(), cos.cpu().numpy(),
                      sin.cpu().numpy(), True)
    assert same_bits(oq.float().cpu().numpy(), rq)
    assert same_bits(ok.float().cpu().numpy(), rk)
    fq, fk = moss.rope(q, k, offset, 500.0)
    assert torch.equal(fq, oq) and torch.equal(fk, ok)


def torch_gated(x, bias, act, gated):
    h = x + bias
    if gated:
        w = x.shape[-1] // 2
        gate, up = h[..., :w], h[..., w:]
    else:
        gate = h
    if act == "silu":
        a = torch.nn.functional.silu(gate)
    elif act == "gelu":
        a = torch.nn.functional.gelu(gate)
    else:
        a = torch.nn.functional.gelu(gate, approximate="tanh")
    return a * up if gated else a


def test_silu_gate_config3(moss, cuda_device):
    g = torch.Generator().manual_seed(4)
    x = torch.randn(4, 2048, 4096, generator=g).to(cuda_device, torch.bfloat16)
    bias = (0.02 * torch.randn(4096, generator=g)).to(cuda_device, torch.bfloat16)
    y = moss.gated_activation(x, bias, "silu", gated=True)
    ref = torch_gated(x, bias, "silu", True)
    assert y.shape == (4, 2048, 2048) and y.dtype == torch.bfloat16
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16))
    sub = slice(0, 64)
    oy = O.gated_act(x[:, sub].float().cpu().numpy(), bias.float().cpu().numpy(), "silu", True, True)
    assert bf16_ulp_diff(y[:, sub].float().cpu().numpy(), oy) <= 1


@pytest.mark.parametrize("copies", [1, 64])
@pytest.mark.parametrize("act", ["silu", "gelu", "gelu_tanh"])
def test_activation_exhaustive_bf16(moss, cuda_device, act, copies):
    """Every one of the 65,536 bf16 bit patterns as the gate input (up = a
    random bf16), with and without a bias: bit-exact against torch.  One
    copy (65,536 outputs) takes the register kernel; 64 copies (2^22
    outputs) the shared-memory table kernel."""
    bits = torch.arange(65536, dtype=torch.int32).to(torch.int16)
    gate = bits.view(torch.bfloat16).reshape(-1, 128).repeat(copies, 1).to(cuda_device)
    g = torch.Generator().manual_seed(31)
    up = torch.randn(gate.shape, generator=g).to(cuda_device, torch.bfloat16)
    x = torch.cat([gate, up], dim=1)
    for bias in (None, (0.5 * torch.randn(256, generator=g)).to(cuda_device, torch.bfloat16)):
        y = moss.gated_activation(x, bias, act, gated=True)
        h = x if bias is None else x + bias
        gh, uh = h[:, :128], h[:, 128:]
        if act == "silu":
            a = torch.nn.functional.silu(gh)
        elif act == "gelu":
            a = torch.nn.functional.gelu(gh)
        else:
            a = torch.nn.functional.gelu(gh, approximate="tanh")
        ref = a * uh
        nan = torch.isnan(ref)
        assert torch.equal(torch.isnan(y), nan)
        assert torch.equal(y.view(torch.int16)[~nan], ref.view(torch.int16)[~nan]), bias is None


@pytest.mark.parametrize("act", ["silu", "gelu", "gelu_tanh"])
@pytest.mark.parametrize("gated", [True, False])
def test_activations_match_torch(moss, cuda_device, act, gated):
    g = torch.Generator().manual_seed(9)
    x = (3 * torch.randn(37, 96, generator=g)).to(cuda_device, torch.bfloat16)
    bias = torch.randn(96, generator=g).to(cuda_device, torch.bfloat16)
    y = moss.gated_activation(x, bias, act, gated=gated)
    ref = torch_gated(x, bias, act, gated)
    # torch's eager CUDA chain calls the same math library: bit-exact
    assert bf16_ulp_diff(y.float().cpu().numpy(), ref.float().cpu().numpy()) == 0
    oy = O.gated_act(x.float().cpu().numpy(), bias.float().cpu().numpy(), act, gated, True)
    yn = y.float().cpu().numpy()
    if act != "silu":
        # For gate inputs below about -3, 1 + erf / 1 + tanh cancels and the
        # float erff/tanhf error dominates; compare with the oracle elsewhere.
        w = x.shape[-1] // 2 if gated else x.shape[-1]
        h = (x[:, :w].float() + bias[:w].float()).to(torch.bfloat16).float().cpu().numpy()
        keep = np.abs(h) <= 3.0
        yn, oy = yn[keep], oy[keep]
    assert bf16_ulp_diff(yn, oy) <= 1
    # odd width -> scalar path; float32 path
    x2 = torch.randn(5, 22, generator=g).to(cuda_device)
    b2 = torch.randn(22, generator=g).to(cuda_device)
    y2 = moss.gated_activation(x2, b2, act, gated=gated)
    r2 = torch_gated(x2, b2, act, gated)
    assert torch.allclose(y2, r2, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(3, 5, 203, 64), (2, 1, 1000, 128), (1, 40, 37, 32)])
def test_rope_streaming_and_register_paths_agree(moss, cuda_device, dtype, shape):
    """Contiguous q/k take the shared-memory streaming kernel; the same values
    behind a padded time stride take the register kernel.  Ragged last tiles
    in every shape; both must give the same bits, with and without tables."""
    b, h, t, d = shape
    g = torch.Generator().manual_seed(11)
    qc = torch.randn(b, h, t, d, generator=g).to(cuda_device, dtype)
    kc = torch.randn(b, h, t, d, generator=g).to(cuda_device, dtype)
    qp = torch.zeros(b, h, t, d + 16, device=cuda_device, dtype=dtype)[..., :d]
    kp = torch.zeros(b, h, t, d + 16, device=cuda_device, dtype=dtype)[..., :d]
    qp.copy_(qc)
    kp.copy_(kc)
    offset = torch.arange(b, device=cuda_device) * 1000 + 3
    bits = torch.int16 if dtype == torch.bfloat16 else torch.int32
    fq, fk = moss.rope(qc, kc, offset, 10000.0)
    pq, pk = moss.rope(qp, kp, offset, 10000.0)
    assert torch.equal(fq.view(bits), pq.view(bits)) and torch.equal(fk.view(bits), pk.view(bits))
    cos, sin = reference_tables(offset, t, d, 10000.0, cuda_device)
    rq, rk = moss.rotate(qc, kc, cos, sin)
    sq, sk = moss.rotate(qp, kp, cos, sin)
    assert torch.equal(rq.view(bits), sq.view(bits)) and torch.equal(rk.view(bits), sk.view(bits))
    assert torch.equal(rq.view(bits), fq.view(bits)) and torch.equal(rk.view(bits), fk.view(bits))
    sl = slice(0, 8)
    oq, ok = O.rotate(qc[:, sl].float().cpu().numpy(), kc[:, sl].float().cpu().numpy(),
                      cos.cpu().numpy(), sin.cpu().numpy(), dtype == torch.bfloat16)
    assert same_bits(rq[:, sl].float().cpu().numpy(), oq)
    assert same_bits(rk[:, sl].float().cpu().numpy(), ok)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(4, 16, 2048, 64), (1, 1, 4000, 1024), (3, 1, 1500, 1024),
                                   (5, 2, 33, 256)])
def test_rope_streaming_row_shares(moss, cuda_device, dtype, shape):
    """The streaming kernel gives each CTA an even share of the b * t rows:
    shares that cross batch boundaries (a different offset on each side),
    shares longer than one phase-table window (head dim 1024: 16 rows per
    window), and the benchmark shape.  In-kernel phase and given
    tables must both give the bits of the reference's tables."""
    b, h, t, d = shape
    g = torch.Generator().manual_seed(17)
    q = torch.randn(b, h, t, d, generator=g).to(cuda_device, dtype)
    k = torch.randn(b, h, t, d, generator=g).to(cuda_device, dtype)
    offset = torch.arange(b, device=cuda_device) * 977 + 11
    bits = torch.int16 if dtype == torch.bfloat16 else torch.int32
    cos, sin = reference_tables(offset, t, d, 10000.0, cuda_device)
    fq, fk = moss.rope(q, k, offset, 10000.0)
    rq, rk = moss.rotate(q, k, cos, sin)
    assert torch.equal(fq.view(bits), rq.view(bits)) and torch.equal(fk.view(bits), rk.view(bits))
    # the same rotation in torch, with the reference's op order
    qf, kf = q.float(), k.float()
    c, s = cos[:, None], sin[:, None]
    for src, got in ((qf, rq), (kf, rk)):
        want = torch.empty_like(src)
        want[..., 0::2] = src[..., 0::2] * c - src[..., 1::2] * s
        want[..., 1::2] = src[..., 0::2] * s + src[..., 1::2] * c
        assert torch.equal(got.view(bits), want.to(dtype).view(bits))


@pytest.mark.parametrize("act", ["silu", "gelu"])
def test_gate_rows_wider_than_a_stage(moss, cuda_device, act):
    """Rows of 40,000 bytes exceed one shared-memory stage and take the
    register kernel; ragged row counts take partial stages."""
    g = torch.Generator().manual_seed(12)
    for rows, width in ((3, 20000), (171, 192), (1, 16)):
        x = torch.randn(rows, width, generator=g).to(cuda_device, torch.bfloat16)
        bias = torch.randn(width, generator=g).to(cuda_device, torch.bfloat16)
        for b in (bias, None):
            y = moss.gated_activation(x, b, act, gated=True)
            ref = torch_gated(x, b, act, True) if b is not None else torch_gated_nobias(x, act)
            assert torch.equal(y.view(torch.int16), ref.view(torch.int16)), (rows, width, b is None)


def torch_gated_nobias(x, act):
    w = x.shape[-1] // 2
    gate, up = x[..., :w], x[..., w:]
    if act == "silu":
        a = torch.nn.functional.silu(gate)
    else:
        a = torch.nn.functional.gelu(gate)
    return a * up


def _rope_kv_case(cuda_device, dtype, b=3, h=4, t=5, d=64, slots_n=9, seed=31):
    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn(b, t, 3, h, d, generator=g).to(cuda_device, dtype)
    q, k, v = (qkv[:, :, i].transpose(1, 2) for i in range(3))  # strided [b,h,t,d] views
    offset = torch.tensor(([0, 7, 123456] + [97 * i for i in range(3, b)])[:b], device=cuda_device,
                          dtype=torch.int64)
    pos = offset[:, None] + torch.arange(t, device=cuda_device)
    slots = torch.remainder(pos, slots_n)
    k_cache = torch.randn(b, h, slots_n, d, generator=g).to(cuda_device, dtype)
    v_cache = torch.randn(b, h, slots_n, d, generator=g).to(cuda_device, dtype)
    return q, k, v, offset, slots, k_cache, v_cache


@pytest.mark.parametrize("shape", [
    (3, 4, 5, 64, 9),      # 16-byte rows: the vector kernel
    (64, 20, 4, 64, 253),  # the stack's 64 batched streams
    (3, 4, 5, 6, 9),       # rows that are not 16-byte vectors: the tile kernel
])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rope_kv_matches_rope_and_scatter(moss, cuda_device, dtype, shape):
    b, h, t, d, slots_n = shape
    q, k, v, offset, slots, kc, vc = _rope_kv_case(cuda_device, dtype, b, h, t, d, slots_n)
    b, h, t, d = q.shape
    kc_ref, vc_ref = kc.clone(), vc.clone()
    oq_ref, ok_ref = moss.rope(q, k, offset, 10000.0)
    index = slots[:, None, :, None].expand(b, h, t, d)
    kc_ref.scatter_(2, index, ok_ref)
    vc_ref.scatter_(2, index, v)
    oq = moss.rope_kv(q, k, v, offset, 10000.0, slots, kc, vc)
    assert torch.equal(oq, oq_ref)
    assert torch.equal(kc, kc_ref)
    assert torch.equal(vc, vc_ref)


def test_rope_kv_reports_a_slot_out_of_range(moss, cuda_device):
    from fast_moss_b200 import _lib

    q, k, v, offset, slots, kc, vc = _rope_kv_case(cuda_device, torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(_lib.load().moss_check_device_error(stream), "clear")
    slots[1, 2] = kc.shape[2]  # one past the ring
    before_k, before_v = kc.clone(), vc.clone()
    moss.rope_kv(q, k, v, offset, 10000.0, slots, kc, vc)
    with pytest.raises(RuntimeError):
        _lib.check(_lib.load().moss_check_device_error(stream), "device error word")
    # the bad token wrote nothing; every other token landed in its slot
    b, h, t, d = q.shape
    _, ok_ref = moss.rope(q, k, offset, 10000.0)
    for bi in range(b):
        for ti in range(t):
            sl = int(slots[bi, ti])
            if sl >= kc.shape[2]:
                continue
            assert torch.equal(kc[bi, :, sl], ok_ref[bi, :, ti])
            assert torch.equal(vc[bi, :, sl], v[bi, :, ti])
    untouched = [s for s in range(kc.shape[2]) if s not in set(slots[1].tolist())]
    assert torch.equal(kc[1, :, untouched], before_k[1, :, untouched])
    assert torch.equal(vc[1, :, untouched], before_v[1, :, untouched])


@pytest.mark.parametrize("rows,n", [(4, 1280), (300, 1024), (4096, 1024), (7, 100)])
def test_layer_norm_bf16_output_is_the_cast(moss, cuda_device, rows, n):
    g = torch.Generator().manual_seed(rows + n)
    x = (torch.randn(rows, n, generator=g) * 2 + 1).to(cuda_device)
    u = torch.randn(rows, n, generator=g).to(cuda_device, torch.bfloat16)
    ls = (0.02 * torch.randn(n, generator=g)).to(cuda_device)
    w = torch.randn(n, generator=g).to(cuda_device)
    bias = torch.randn(n, generator=g).to(cuda_device)
    r, y = moss.residual_layer_norm(x, u, ls, w, bias, 1e-5, out_dtype=torch.bfloat16)
    r_ref = x + u.float() * ls
    y_ref = torch.nn.functional.layer_norm(r_ref, (n,), w, bias, 1e-5).to(torch.bfloat16)
    assert y.dtype == torch.bfloat16
    assert torch.equal(r, r_ref)
    assert torch.equal(y, y_ref)
    y2 = moss.layer_norm(x, w, bias, 1e-5, out_dtype=torch.bfloat16)
    assert torch.equal(y2, torch.nn.functional.layer_norm(x, (n,), w, bias, 1e-5).to(torch.bfloat16))
