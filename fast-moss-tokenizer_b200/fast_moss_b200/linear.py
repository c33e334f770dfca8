"""Linear layers on cached bf16 weights with the B200 tensor-core kernel.

`pack_weight(w)` packs a cached bf16 weight once (the reference caches the
bf16 copy of each FP32 Linear weight when its context is entered:
fast_moss/v2_runtime.py:77-106); `linear(x, packed, bias)` is then that
cached Linear (F.linear at :104) as one tcgen05 kernel (moss_linear), and
`linear(x, packed, bias, activation=...)` also applies the feed-forward's
bias + activation in the same kernel (the Linear without bias followed by
act(h + b), one rounding per torch op).  Results are deterministic; the
FP32 sums run in the kernel's order, not cuBLAS's.
"""

import torch

from . import _lib

_ACTS = {"silu": _lib.ACT_SILU, "gelu": _lib.ACT_GELU_ERF, "gelu_tanh": _lib.ACT_GELU_TANH}


class PackedWeight:
    """A bf16 weight [N, K] in the kernel's tile layout (same bytes, another
    order): per 128-row tile and 64-column chunk one 16 KB block in the
    tensor cores' 128-byte-swizzled K-major layout."""

    def __init__(self, image, n, k):
        self.image, self.n, self.k = image, n, k
        self.device = image.device


def pack_weight(weight):
    """Packs a bf16 CUDA weight [N, K] (N a multiple of 128, K of 64; other
    shapes raise UnsupportedError)."""
    if weight.ndim != 2 or weight.dtype != torch.bfloat16 or not weight.is_cuda:
        raise ValueError("pack_weight expects a bf16 CUDA weight [N, K]")
    n, k = weight.shape
    w = weight.contiguous()
    image = torch.empty(n * k, device=w.device, dtype=torch.bfloat16)
    with torch.cuda.device(w.device):
        _lib.call("moss_linear_pack_weight", w.data_ptr(), n, k, image.data_ptr(),
                  torch.cuda.current_stream(w.device).cuda_stream)
    return PackedWeight(image, n, k)


def linear(x, weight, bias=None, activation=None, *, out=None):
    """y = x @ W.T + bias, or act(bf16(x @ W.T) + bias) with `activation`
    in ("silu", "gelu", "gelu_tanh"), W given as a PackedWeight.

    x [..., K], bias [N] (optional): bf16 CUDA tensors on W's device."""
    if not isinstance(weight, PackedWeight):
        raise ValueError("linear expects a weight packed by pack_weight")
    if x.dtype != torch.bfloat16 or not x.is_cuda or x.device != weight.device:
        raise ValueError("linear expects bf16 CUDA input on the weight's device")
    n, k = weight.n, weight.k
    if x.shape[-1] != k:
        raise ValueError(f"input width {x.shape[-1]} does not match the weight's {k}")
    if bias is not None and (bias.shape != (n,) or bias.dtype != torch.bfloat16
                             or bias.device != x.device):
        raise ValueError("bias must be bf16 [N] on the input's device")
    if activation is not None and activation not in _ACTS:
        raise ValueError(f"unknown activation {activation!r}")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, k)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    b = None if bias is None else bias.contiguous()
    if out is None:
        out = torch.empty(lead + (n,), device=x.device, dtype=torch.bfloat16)
    elif out.shape != lead + (n,) or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError("out must be a contiguous bf16 tensor of the output shape")
    epilogue = _lib.LINEAR_BIAS if activation is None else _lib.LINEAR_BIAS_ACT
    act = 0 if activation is None else _ACTS[activation]
    with torch.cuda.device(x.device):
        _lib.call("moss_linear", x2.data_ptr(), x2.shape[0], k, weight.image.data_ptr(), n,
                  None if b is None else b.data_ptr(), epilogue, act, out.data_ptr(),
                  torch.cuda.current_stream(x.device).cuda_stream)
    return out
