"""GPU: the failure path of the bounded waits, without a GPU fault.

Every spin in the kernels (mbarrier phases of the bulk-copy pipelines and
of the tensor-core quantizer) gives up after a time limit, records
MOSS_ERR_TIMEOUT in the device error word and returns.  moss_test_bounded_wait
runs that same wait with a short caller-given limit on a phase that nothing
completes, so the timeout really happens; the test then reads the status on
the host and checks that the context is still usable: the next kernels on
the same stream give the oracle's results.
"""

import time

import numpy as np
import pytest
import torch

from conftest import same_bits
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_wait_that_completes_records_nothing(moss, cuda_device):
    from fast_moss_b200 import _lib

    lib = _lib.load()
    sh = torch.cuda.current_stream(cuda_device).cuda_stream
    assert lib.moss_check_device_error(sh) in (_lib.OK, _lib.ERR_TIMEOUT)  # clear the word
    _lib.check(lib.moss_test_bounded_wait(1_000_000, 1, sh), "moss_test_bounded_wait")
    assert lib.moss_check_device_error(sh) == _lib.OK


def test_wait_that_never_completes_times_out_and_the_context_survives(moss, cuda_device):
    from fast_moss_b200 import _lib

    lib = _lib.load()
    sh = torch.cuda.current_stream(cuda_device).cuda_stream
    assert lib.moss_check_device_error(sh) in (_lib.OK, _lib.ERR_TIMEOUT)
    limit_ns = 2_000_000  # 2 ms instead of the kernels' ~2 s
    t = time.perf_counter()
    _lib.check(lib.moss_test_bounded_wait(limit_ns, 0, sh), "moss_test_bounded_wait")
    torch.cuda.synchronize()
    waited = time.perf_counter() - t
    assert waited < 5.0  # gave up on its own, long before any watchdog
    assert lib.moss_check_device_error(sh) == _lib.ERR_TIMEOUT
    assert b"bounded wait" in lib.moss_last_error()
    assert lib.moss_check_device_error(sh) == _lib.OK  # read and cleared

    # the same stream still runs kernels correctly: a pipelined kernel
    # (bulk copies + mbarriers) and the tensor-core quantizer
    g = torch.Generator().manual_seed(3)
    q = torch.randn(2, 4, 64, 64, generator=g).to(cuda_device, torch.bfloat16)
    k = torch.randn(2, 4, 64, 64, generator=g).to(cuda_device, torch.bfloat16)
    ones = torch.zeros(2, 1, 64, 64, device=cuda_device)
    ones[..., 0::2] = 1.0
    offset = torch.tensor([0, 5], device=cuda_device)
    tab, _ = moss.rope(ones, ones, offset, 10000.0)
    cos, sin = tab[:, 0, :, 0::2].contiguous(), tab[:, 0, :, 1::2].contiguous()
    oq, ok = moss.rope(q, k, offset, 10000.0)
    rq, rk = O.rotate(q.float().cpu().numpy(), k.float().cpu().numpy(), cos.cpu().numpy(),
                      sin.cpu().numpy(), True)
    assert same_bits(oq.float().cpu().numpy(), rq) and same_bits(ok.float().cpu().numpy(), rk)

    rng = np.random.default_rng(4)
    x = rng.standard_normal((500, 64)).astype(np.float32)
    books = (rng.standard_normal((3, 512, 64)) / 8).astype(np.float32)
    rvq = moss.ResidualVectorQuantizer(torch.from_numpy(books).to(cuda_device))
    codes, recon = rvq.encode(torch.from_numpy(x).to(cuda_device))
    oc, orc = O.rvq_encode(x, books)
    assert np.array_equal(codes.cpu().numpy(), oc)
    assert same_bits(recon.cpu().numpy(), orc)
    assert lib.moss_check_device_error(sh) == _lib.OK

