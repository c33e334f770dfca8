"""Exact nearest-codeword selection on B200 (reference fast_moss/quantizer.py).

`select` keeps the reference's signature, validation, exceptions and output
layout (values as the transposed B,D,T view of a [B,T,D] buffer, or a
contiguous B,D,T straight-through output; int64 indices [B,T]).
`decode_latents` is the fused LFQ stage used by the optimized runtime: it
computes the preparation, the dot products and the selection in one kernel,
without the [B*T, K] dot-product matrix.
"""

import torch

from . import _lib


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


def select(dots, row_norm, codebook_norm, codebook, latents, *, straight_through=False):
    """distance = (row_norm - dots) + codebook_norm; first NaN, else first minimum.

    Reference fast_moss/quantizer.py:52-108.
    """
    if latents.ndim != 3 or codebook.ndim != 2:
        raise ValueError("Expected B,D,T latents and K,D codebook")
    b, d, t = latents.shape
    k, book_d = codebook.shape
    if (
        d != book_d
        or not k
        or k > 65536
        or dots.shape != (b * t, k)
        or row_norm.shape != (b * t, 1)
        or codebook_norm.shape != (1, k)
    ):
        raise ValueError("Incompatible quantizer shapes or unsupported codebook size")
    tensors = (dots, row_norm, codebook_norm, codebook, latents)
    if any(
        x.dtype != torch.float32 or not x.is_cuda or x.device != dots.device
        for x in tensors
    ):
        raise ValueError("Quantizer fusion requires same-device CUDA FP32 inputs")
    if not all(x.is_contiguous() for x in tensors[:-1]):
        raise ValueError("Distance inputs and codebook must be contiguous")
    indices = torch.empty((b, t), device=dots.device, dtype=torch.long)
    output = (
        torch.empty((b, d, t), device=dots.device, dtype=torch.float32)
        if straight_through
        else torch.empty((b, t, d), device=dots.device, dtype=torch.float32)
    )
    if b * t:
        with torch.cuda.device(dots.device):
            _lib.call(
                "moss_lfq_select", dots.data_ptr(), row_norm.data_ptr(), codebook_norm.data_ptr(),
                codebook.data_ptr(), latents.data_ptr(), _lib.strides(latents.stride()), b, d, t,
                k, 1 if straight_through else 0, output.data_ptr(), indices.data_ptr(),
                _stream(dots.device))
    return (output if straight_through else output.transpose(1, 2)), indices


def decode_latents(x, book_normed, code_norm, weight):
    """Fused LFQ decode of x [B,8,T] (reference fast_moss/v2_runtime.py:143-181).

    book_normed [K,8] = F.normalize(weight), code_norm [1,K] or [K] = its row
    sums of squares, weight [K,8] = raw codebook.  Returns (values as the
    B,8,T transposed view of a [B,T,8] buffer, int64 indices [B,T]).
    Dots are a sequential FMA over the 8 channels.
    """
    if x.ndim != 3 or x.shape[1] != 8 or x.shape[0] < 1 or x.shape[2] < 1:
        raise ValueError("Expected nonempty B,8,T latents")
    k = weight.shape[0]
    if (
        book_normed.shape != (k, 8) or weight.shape != (k, 8) or code_norm.numel() != k
        or not k or k > 65536
    ):
        raise ValueError("Incompatible quantizer shapes or unsupported codebook size")
    tensors = (x, book_normed, code_norm, weight)
    if any(v.dtype != torch.float32 or not v.is_cuda or v.device != x.device for v in tensors):
        raise ValueError("Quantizer fusion requires same-device CUDA FP32 inputs")
    x = x.contiguous()
    book_normed, code_norm, weight = (v.contiguous() for v in (book_normed, code_norm, weight))
    b, _, t = x.shape
    out = torch.empty((b, t, 8), device=x.device, dtype=torch.float32)
    indices = torch.empty((b, t), device=x.device, dtype=torch.long)
    with torch.cuda.device(x.device):
        _lib.call(
            "moss_lfq_decode", x.data_ptr(), book_normed.data_ptr(), code_norm.data_ptr(),
            weight.data_ptr(), b, t, k, out.data_ptr(), indices.data_ptr(), _stream(x.device))
    return out.transpose(1, 2), indices
