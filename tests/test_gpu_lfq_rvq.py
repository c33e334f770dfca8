"""GPU: the real codec's multi-stage LFQ quantizer in one kernel
(moss_lfq_rvq_encode) against the oracle loop, bit for bit: codes and the
final residual, over the three frame groupings of the kernel (1, 4 and 16
frames per CTA), the transposed prepare order (one clip of many frames),
ragged sizes, and non-finite frames."""

import numpy as np
import pytest
import torch

from conftest import same_bits
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _params(d, stages, k, seed):
    rng = np.random.default_rng(seed)
    w_in = (rng.standard_normal((stages, 8, d)) / np.sqrt(d)).astype(np.float32)
    b_in = (0.1 * rng.standard_normal((stages, 8))).astype(np.float32)
    weight = rng.standard_normal((stages, k, 8)).astype(np.float32)
    w_out = (0.3 * rng.standard_normal((stages, d, 8)) / np.sqrt(8)).astype(np.float32)
    b_out = (0.01 * rng.standard_normal((stages, d))).astype(np.float32)
    return w_in, b_in, weight, w_out, b_out


def _run(moss, cuda_device, x, params):
    from fast_moss_b200 import _lib
    from fast_moss_b200.lfq_rvq import LFQResidualQuantizer

    q = LFQResidualQuantizer(*(torch.from_numpy(p).to(cuda_device) for p in params))
    xd = torch.from_numpy(x).to(cuda_device)
    res = torch.empty_like(xd)
    codes = q.encode(xd, residual=res)
    torch.cuda.synchronize()
    _lib.check(_lib.load().moss_check_device_error(None), "device error word")
    w_in, b_in, weight, w_out, b_out = params
    oc, ores = O.lfq_rvq_encode(x, w_in, b_in, q.book_normed.cpu().numpy(),
                                q.code_norm.cpu().numpy(), weight, w_out, b_out)
    return codes.cpu().numpy(), res.cpu().numpy(), oc, ores


@pytest.mark.parametrize("b,d,t,stages,k", [
    (2, 1280, 23, 32, 1024),   # the stack's width, all 32 stages; 1 frame per CTA
    (1, 256, 50, 8, 300),      # one clip: the transposed prepare order
    (5, 96, 1, 3, 64),         # streaming: one frame per clip
    (2, 256, 300, 4, 512),     # 4 frames per CTA
    (2, 256, 301, 4, 512),     # 4 frames per CTA, the last CTA holds 2
    (3, 128, 800, 3, 256),     # 16 frames per CTA, every CTA full
    (3, 128, 801, 3, 256),     # 16 frames per CTA, the last CTA holds 3
    (2, 200, 5, 2, 1000),      # a width that is not a multiple of 32
])
def test_lfq_rvq_matches_the_oracle_loop(moss, cuda_device, b, d, t, stages, k):
    rng = np.random.default_rng(b * 1000 + d + t)
    x = rng.standard_normal((b, d, t)).astype(np.float32)
    codes, res, oc, ores = _run(moss, cuda_device, x, _params(d, stages, k, d + k))
    assert np.array_equal(codes.reshape(stages, -1), oc)
    assert same_bits(res, ores)


def test_lfq_rvq_non_finite_frames(moss, cuda_device):
    """A NaN or infinite frame makes every distance NaN at the first stage
    (first NaN index wins, as in the reference's select); the loop carries
    the non-finite residual on exactly as the oracle does."""
    b, d, t, stages, k = 2, 64, 6, 3, 40
    rng = np.random.default_rng(9)
    x = rng.standard_normal((b, d, t)).astype(np.float32)
    x[0, 5, 2] = np.nan
    x[1, 0, 4] = np.inf
    codes, res, oc, ores = _run(moss, cuda_device, x, _params(d, stages, k, 3))
    assert np.array_equal(codes.reshape(stages, -1), oc)
    assert same_bits(res, ores)


@pytest.mark.parametrize("t", [6, 2400])  # 1 and 16 frames per CTA
def test_lfq_rvq_non_finite_code(moss, cuda_device, t):
    """A NaN in one code of one stage makes that code's distance NaN for
    every frame, so every frame takes it at that stage (first NaN wins);
    the stages before it run on finite data.  Same codes and residual as
    the oracle."""
    b, d, stages, k = 1, 64, 3, 300
    rng = np.random.default_rng(10)
    x = rng.standard_normal((b, d, t)).astype(np.float32)
    params = list(_params(d, stages, k, 4))
    params[2] = params[2].copy()
    params[2][1, 7, 3] = np.nan
    codes, res, oc, ores = _run(moss, cuda_device, x, tuple(params))
    assert np.array_equal(codes.reshape(stages, -1), oc)
    assert (oc[1] == 7).all()
    assert same_bits(res, ores)
