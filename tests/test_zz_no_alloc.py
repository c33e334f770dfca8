"""GPU: moss_rvq_encode_static (prepared codebooks in the library's static
device array) against moss_rvq_encode with caller-allocated prepared
buffers, on consecutive calls with different codebooks and sizes.  Named to
be collected last, so it also runs after every other GPU test."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _workspace_encode(lib, _lib, x, books):
    stages, k, d = books.shape
    floats = lib.moss_rvq_packed_floats(stages, k, d)
    kpad = -(-k // 256) * 256
    dev = x.device
    packed = torch.empty(floats, device=dev)
    code_norm = torch.empty((stages, kpad), device=dev)
    stats = torch.empty((stages, 4), device=dev)
    codes = torch.empty((stages, x.shape[0]), dtype=torch.int32, device=dev)
    recon = torch.empty_like(x)
    residual = torch.empty_like(x)
    sh = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(lib.moss_rvq_prepare_codebooks(books.data_ptr(), stages, k, d, code_norm.data_ptr(),
                                              packed.data_ptr(), stats.data_ptr(), sh),
               "moss_rvq_prepare_codebooks")
    _lib.check(lib.moss_rvq_encode(x.data_ptr(), x.shape[0], d, books.data_ptr(), packed.data_ptr(),
                                   code_norm.data_ptr(), stats.data_ptr(), stages, k,
                                   codes.data_ptr(), recon.data_ptr(), residual.data_ptr(), sh),
               "moss_rvq_encode")
    return codes, recon, residual


def _static_encode(lib, _lib, x, books):
    stages, k, d = books.shape
    codes = torch.full((stages, x.shape[0]), -7, dtype=torch.int32, device=x.device)
    recon = torch.full_like(x, float("nan"))
    residual = torch.full_like(x, float("nan"))
    sh = torch.cuda.current_stream(x.device).cuda_stream
    _lib.check(lib.moss_rvq_encode_static(x.data_ptr(), x.shape[0], d, books.data_ptr(), stages, k,
                                          codes.data_ptr(), recon.data_ptr(), residual.data_ptr(),
                                          sh), "moss_rvq_encode_static")
    return codes, recon, residual


def test_static_scratch_matches_workspace_entry_point(moss, cuda_device):
    from fast_moss_b200 import _lib

    lib = _lib.load()
    rng = np.random.default_rng(77)
    # two consecutive calls: full capacity, then a smaller ragged case whose
    # preparation must fully replace the first one's
    for rows, stages, k in ((1000, 32, 1024), (301, 7, 300)):
        x = torch.from_numpy(rng.standard_normal((rows, 64)).astype(np.float32)).to(cuda_device)
        books = torch.from_numpy(
            (rng.standard_normal((stages, k, 64)) / 8).astype(np.float32)).to(cuda_device)
        got = _static_encode(lib, _lib, x, books)
        want = _workspace_encode(lib, _lib, x, books)
        torch.cuda.synchronize()
        for g, w in zip(got, want):
            assert torch.equal(g, w), (rows, stages, k)
        assert lib.moss_check_device_error(None) == 0
