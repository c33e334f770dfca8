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


def test_static_scratch_without_residual_and_with_no_rows(moss, cuda_device):
    """residual_out may be NULL (the header allows it); rows == 0 is a no-op
    that returns MOSS_OK and leaves the outputs untouched."""
    from fast_moss_b200 import _lib

    lib = _lib.load()
    rng = np.random.default_rng(78)
    x = torch.from_numpy(rng.standard_normal((513, 64)).astype(np.float32)).to(cuda_device)
    books = torch.from_numpy(
        (rng.standard_normal((9, 700, 64)) / 8).astype(np.float32)).to(cuda_device)
    sh = torch.cuda.current_stream(cuda_device).cuda_stream
    codes = torch.full((9, 513), -7, dtype=torch.int32, device=cuda_device)
    recon = torch.full_like(x, float("nan"))
    _lib.check(lib.moss_rvq_encode_static(x.data_ptr(), 513, 64, books.data_ptr(), 9, 700,
                                          codes.data_ptr(), recon.data_ptr(), None, sh),
               "moss_rvq_encode_static")
    want = _workspace_encode(lib, _lib, x, books)
    torch.cuda.synchronize()
    assert torch.equal(codes, want[0]) and torch.equal(recon, want[1])

    codes0 = codes.clone()
    recon0 = recon.clone()
    st = lib.moss_rvq_encode_static(x.data_ptr(), 0, 64, books.data_ptr(), 9, 700,
                                    codes.data_ptr(), recon.data_ptr(), None, sh)
    torch.cuda.synchronize()
    assert st == _lib.OK
    assert torch.equal(codes, codes0) and torch.equal(recon, recon0)
    assert lib.moss_check_device_error(None) == 0
