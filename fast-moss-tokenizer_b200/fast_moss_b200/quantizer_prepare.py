"""Eight-channel LFQ latent preparation (reference fast_moss/quantizer_prepare.py).

`prepare` keeps the reference's signature, validation, output layouts and
summation orders; it is an ahead-of-time sm_100a kernel of
libfast_moss_b200 instead of a runtime-compiled sm_120 one.
"""

import torch

from . import _lib


def prepare(x):
    """Returns (normalized, norm, twice, denom) for x [B,8,T] FP32 contiguous.

    normalized/twice are [B*T,8], or the [T,8] transpose view of an [8,T]
    buffer when B == 1 < T; norm and denom are [B*T,1]
    (reference fast_moss/quantizer_prepare.py:111-157).
    """
    if (
        x.ndim != 3
        or x.shape[1] != 8
        or not x.is_cuda
        or x.dtype != torch.float32
        or not x.is_contiguous()
        or x.shape[0] < 1
        or x.shape[2] < 1
        or x.numel() > 2147483647
    ):
        raise ValueError("Expected nonempty contiguous CUDA FP32 B,8,T latents")
    b, _, t = x.shape
    with torch.cuda.device(x.device):
        normalized = torch.empty(
            (8, t) if b == 1 and t > 1 else (b * t, 8), device=x.device, dtype=x.dtype
        )
        if b == 1 and t > 1:
            normalized = normalized.T
        twice = torch.empty_strided(
            normalized.shape, normalized.stride(), device=x.device, dtype=x.dtype
        )
        norm = torch.empty((b * t, 1), device=x.device, dtype=x.dtype)
        denom = torch.empty_like(norm)
        _lib.call(
            "moss_lfq_prepare", x.data_ptr(), b, t, normalized.data_ptr(), norm.data_ptr(),
            twice.data_ptr(), denom.data_ptr(), torch.cuda.current_stream(x.device).cuda_stream)
    return normalized, norm, twice, denom
