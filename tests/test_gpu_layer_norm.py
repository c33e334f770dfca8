"""GPU parity: residual + layer scale + LayerNorm.

Reference path on the same device: the reference's residual (`x + u*s`,
unfused -- eager torch on CUDA runs the multiply and the add as separate
kernels, like `_scale_add`) followed by torch's CUDA LayerNorm, the op the
reference calls (fast_moss/v2_runtime.py:259).  Bar: bit-exact FP32
(residual, normalised output, mean and rstd).  The CPU oracle must agree bit
for bit on mean and output given the device rstd (rsqrtf is a hardware
approximation, checked to be within 2 ulp of 1/sqrt(var+eps)).
"""

import numpy as np
import pytest
import torch

from conftest import same_bits
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def config1_inputs(device, rows=4096, n=1024, seed=0, bf16_update=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(1, rows, n, generator=g)
    y = torch.randn(1, rows, n, generator=g)
    gamma = 1 + 0.1 * torch.randn(n, generator=g)
    beta = 0.1 * torch.randn(n, generator=g)
    ls = 0.01 * torch.randn(n, generator=g)
    if bf16_update:
        y = y.to(torch.bfloat16)
    return [t.to(device) for t in (x, y, gamma, beta, ls)]


def torch_reference(x, u, ls, gamma, beta, eps):
    r = x.float() + ls * u.float()
    out, mean, rstd = torch.native_layer_norm(r, (r.shape[-1],), gamma, beta, eps)
    return r, out, mean.reshape(-1), rstd.reshape(-1)


def oracle_check(r, normed, mean, rstd, gamma, beta, eps):
    rn = r.cpu().numpy().reshape(-1, r.shape[-1])
    y, m, ve, _ = O.layer_norm(rn, gamma.cpu().numpy(), beta.cpu().numpy(), eps,
                               rstd=rstd.cpu().numpy())
    if not same_bits(m, mean.cpu().numpy()):
        variants = {v: same_bits(O.layer_norm(rn, gamma.cpu().numpy(), beta.cpu().numpy(), eps,
                                              mean_variant=v)[1], mean.cpu().numpy())
                    for v in (1, 2)}
        raise AssertionError(f"oracle mean differs from the device; other merge forms: {variants}")
    assert same_bits(y, normed.cpu().numpy().reshape(y.shape))
    exact = (1.0 / np.sqrt(ve.astype(np.float64))).astype(np.float32)
    ulps = np.abs(exact.view(np.int32).astype(np.int64) -
                  rstd.cpu().numpy().view(np.int32).astype(np.int64))
    assert ulps.max() <= 2


def test_config1_matches_torch_cuda_bit_exact(moss, cuda_device):
    x, u, gamma, beta, ls = config1_inputs(cuda_device)
    r, normed, mean, rstd = moss.residual_layer_norm(x, u, ls, gamma, beta, 1e-5,
                                                     return_stats=True)
    rr, rn, rm, rs = torch_reference(x, u, ls, gamma, beta, 1e-5)
    torch.cuda.synchronize()
    assert torch.equal(r, rr)
    assert same_bits(normed.cpu().numpy(), rn.cpu().numpy())
    assert same_bits(mean.cpu().numpy(), rm.cpu().numpy())
    assert same_bits(rstd.cpu().numpy(), rs.cpu().numpy())


def test_config1_matches_oracle(moss, cuda_device):
    x, u, gamma, beta, ls = config1_inputs(cuda_device, rows=512)
    r, normed, mean, rstd = moss.residual_layer_norm(x, u, ls, gamma, beta, 1e-5,
                                                     return_stats=True)
    assert same_bits(r.cpu().numpy(),
                     O.scale_add(x.cpu().numpy(), u.cpu().numpy(), ls.cpu().numpy()))
    oracle_check(r, normed, mean, rstd, gamma, beta, 1e-5)


@pytest.mark.parametrize("n", [4, 8, 64, 100, 512, 1000, 1024, 1280, 1536, 2048])
@pytest.mark.parametrize("rows", [1, 3, 37])
def test_widths_match_torch_cuda(moss, cuda_device, n, rows):
    g = torch.Generator().manual_seed(n * 1000 + rows)
    # a large common offset stresses the Welford merge arithmetic
    x = (torch.randn(rows, n, generator=g) * 3 + 100).to(cuda_device)
    u = torch.randn(rows, n, generator=g).to(cuda_device)
    gamma = torch.randn(n, generator=g).to(cuda_device)
    beta = torch.randn(n, generator=g).to(cuda_device)
    ls = torch.randn(n, generator=g).to(cuda_device)
    r, normed, mean, rstd = moss.residual_layer_norm(x, u, ls, gamma, beta, 1e-5,
                                                     return_stats=True)
    rr, rn, rm, rs = torch_reference(x, u, ls, gamma, beta, 1e-5)
    assert torch.equal(r, rr)
    assert same_bits(normed.cpu().numpy(), rn.cpu().numpy())
    assert same_bits(mean.cpu().numpy(), rm.cpu().numpy())
    assert same_bits(rstd.cpu().numpy(), rs.cpu().numpy())
    oracle_check(r, normed, mean, rstd, gamma, beta, 1e-5)


def test_bf16_update_and_plain_layer_norm(moss, cuda_device):
    x, u, gamma, beta, ls = config1_inputs(cuda_device, rows=300, n=1280, bf16_update=True)
    r, normed = moss.residual_layer_norm(x, u, ls, gamma, beta, 1e-5)
    rr, rn, _, _ = torch_reference(x, u, ls, gamma, beta, 1e-5)
    assert torch.equal(r, rr) and same_bits(normed.cpu().numpy(), rn.cpu().numpy())
    y = moss.layer_norm(rr, gamma, beta, 1e-5)
    assert same_bits(y.cpu().numpy(), rn.cpu().numpy())
    # without an affine transform, and with only one of gamma / beta
    for w, b in ((None, None), (gamma, None), (None, beta)):
        y = moss.layer_norm(rr, w, b, 1e-5)
        ref = torch.nn.functional.layer_norm(rr, (1280,), w, b, 1e-5)
        assert same_bits(y.cpu().numpy(), ref.cpu().numpy())
    # residual_out may be skipped
    none, normed2 = moss.residual_layer_norm(x, u, ls, gamma, beta, 1e-5, write_residual=False)
    assert none is None and torch.equal(normed2, normed)


def test_special_values_and_empty(moss, cuda_device):
    x, u, gamma, beta, ls = config1_inputs(cuda_device, rows=8, n=256)
    x[0, 1, 5] = float("nan")
    x[0, 2, 7] = float("inf")
    x[0, 3, :] = 0.0
    u[0, 3, :] = 0.0
    x[0, 4, :] = 1e30
    r, normed, mean, rstd = moss.residual_layer_norm(x, u, ls, gamma, beta, 1e-5,
                                                     return_stats=True)
    rr, rn, rm, rs = torch_reference(x, u, ls, gamma, beta, 1e-5)
    assert same_bits(r.cpu().numpy(), rr.cpu().numpy())
    assert same_bits(normed.cpu().numpy(), rn.cpu().numpy())
    assert same_bits(mean.cpu().numpy(), rm.cpu().numpy())
    assert same_bits(rstd.cpu().numpy(), rs.cpu().numpy())
    e = torch.empty(0, 256, device=cuda_device)
    r0, n0 = moss.residual_layer_norm(e, e, ls, gamma, beta)
    assert r0.shape == (0, 256) and n0.shape == (0, 256)


def test_unsupported_widths_raise(moss, cuda_device):
    from fast_moss_b200._lib import UnsupportedError

    x = torch.randn(4, 1026, device=cuda_device)
    with pytest.raises(UnsupportedError):
        moss.layer_norm(x, None, None)
    x = torch.randn(4, 4096, device=cuda_device)
    with pytest.raises(UnsupportedError):
        moss.layer_norm(x, None, None)


# Thousands of rows (several rows per resident block slot on every SM),
# every dtype pair, widths with and without 16-byte rows, NaN and inf.
@pytest.mark.parametrize("rows", [1187, 2072, 3001])
@pytest.mark.parametrize("n", [8, 100, 1024, 1280, 2048])
@pytest.mark.parametrize("dtypes", [(torch.float32, torch.float32), (torch.float32, torch.bfloat16),
                                    (torch.bfloat16, torch.float32),
                                    (torch.bfloat16, torch.bfloat16)])
def test_many_rows_match_torch_cuda(moss, cuda_device, rows, n, dtypes):
    g = torch.Generator().manual_seed(rows * 7 + n)
    x = (torch.randn(rows, n, generator=g) * 3 + 10).to(cuda_device, dtypes[0])
    u = torch.randn(rows, n, generator=g).to(cuda_device, dtypes[1])
    x[5, 3] = float("nan")
    x[rows - 1, 0] = float("inf")
    gamma = torch.randn(n, generator=g).to(cuda_device)
    beta = torch.randn(n, generator=g).to(cuda_device)
    ls = torch.randn(n, generator=g).to(cuda_device)
    r, normed, mean, rstd = moss.residual_layer_norm(x, u, ls, gamma, beta, 1e-5,
                                                     return_stats=True)
    rr, rn, rm, rs = torch_reference(x, u, ls, gamma, beta, 1e-5)
    assert same_bits(r.cpu().numpy(), rr.cpu().numpy())
    assert same_bits(normed.cpu().numpy(), rn.cpu().numpy())
    assert same_bits(mean.cpu().numpy(), rm.cpu().numpy())
    assert same_bits(rstd.cpu().numpy(), rs.cpu().numpy())


@pytest.mark.parametrize("rows", [1200, 4097])
def test_many_rows_plain_layer_norm_and_affine_variants(moss, cuda_device, rows):
    n = 1024
    g = torch.Generator().manual_seed(rows)
    x = (torch.randn(rows, n, generator=g) * 2 - 5).to(cuda_device)
    gamma = torch.randn(n, generator=g).to(cuda_device)
    beta = torch.randn(n, generator=g).to(cuda_device)
    for w, b in ((gamma, beta), (None, None), (gamma, None), (None, beta)):
        y, mean, rstd = moss.layer_norm(x, w, b, 1e-5, return_stats=True)
        ref, rm, rs = torch.native_layer_norm(x, (n,), w, b, 1e-5)
        assert same_bits(y.cpu().numpy(), ref.cpu().numpy())
        assert same_bits(mean.cpu().numpy(), rm.reshape(-1).cpu().numpy())
        assert same_bits(rstd.cpu().numpy(), rs.reshape(-1).cpu().numpy())
    # an input that starts 4 bytes past a 16-byte boundary takes scalar loads
    buf = torch.empty(rows * n + 1, device=cuda_device)
    xs = buf[1:].view(rows, n)
    xs.copy_(x)
    ls = torch.randn(n, generator=g).to(cuda_device)
    u = torch.randn(rows, n, generator=g).to(cuda_device)
    r, normed = moss.residual_layer_norm(xs, u, ls, gamma, beta, 1e-5)
    rr, rn, _, _ = torch_reference(x, u, ls, gamma, beta, 1e-5)
    assert same_bits(r.cpu().numpy(), rr.cpu().numpy())
    assert same_bits(normed.cpu().numpy(), rn.cpu().numpy())
