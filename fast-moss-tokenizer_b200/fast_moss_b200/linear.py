"""Linear layers on cached bf16 weights with the B200 tensor-core kernel.

`linear(x, weight, bias)` is the cached bf16 Linear of the reference's
optimised model (fast_moss/v2_runtime.py:77-106: F.linear on bf16 copies of
the FP32 weight and bias) as one tcgen05 kernel (moss_linear);
`linear(x, weight, bias, activation=...)` also applies the feed-forward's
bias + activation in the same kernel (the Linear without bias followed by
act(h + b), one rounding per torch op).  Results are deterministic; the FP32
sums run in the kernel's order, not cuBLAS's.
"""

import torch

from . import _lib

_ACTS = {"silu": _lib.ACT_SILU, "gelu": _lib.ACT_GELU_ERF, "gelu_tanh": _lib.ACT_GELU_TANH}


def linear(x, weight, bias=None, activation=None, *, out=None):
    """y = x @ weight.T + bias, or act(bf16(x @ weight.T) + bias) with
    `activation` in ("silu", "gelu", "gelu_tanh").

    x [..., K], weight [N, K], bias [N] (optional): bf16 CUDA tensors on one
    device.  K must be a multiple of 64 and N of 128; other shapes raise
    UnsupportedError (callers fall back to F.linear)."""
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16 or not x.is_cuda:
        raise ValueError("linear expects bf16 CUDA tensors")
    if weight.ndim != 2 or x.shape[-1] != weight.shape[1] or weight.device != x.device:
        raise ValueError("weight must be [N, K] on the input's device")
    if bias is not None and (bias.shape != (weight.shape[0],) or bias.dtype != torch.bfloat16
                             or bias.device != x.device):
        raise ValueError("bias must be bf16 [N] on the input's device")
    if activation is not None and activation not in _ACTS:
        raise ValueError(f"unknown activation {activation!r}")
    n, k = weight.shape
    lead = x.shape[:-1]
    x2 = x.reshape(-1, k)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    w = weight if weight.is_contiguous() else weight.contiguous()
    b = None if bias is None else bias.contiguous()
    m = x2.shape[0]
    if out is None:
        out = torch.empty(lead + (n,), device=x.device, dtype=torch.bfloat16)
    elif out.shape != lead + (n,) or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError("out must be a contiguous bf16 tensor of the output shape")
    epilogue = _lib.LINEAR_BIAS if activation is None else _lib.LINEAR_BIAS_ACT
    act = 0 if activation is None else _ACTS[activation]
    with torch.cuda.device(x.device):
        _lib.call("moss_linear", x2.data_ptr(), m, k, w.data_ptr(), n,
                  None if b is None else b.data_ptr(), epilogue, act, out.data_ptr(),
                  torch.cuda.current_stream(x.device).cuda_stream)
    return out
