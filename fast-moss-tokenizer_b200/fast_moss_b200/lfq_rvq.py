"""The real codec's multi-stage LFQ quantizer as one B200 kernel.

Per stage the upstream quantizer (called by the reference at
fast_moss/v2_codec.py:45) projects the residual to 8 channels, runs the
LFQ decode the reference patches (fast_moss/v2_runtime.py:143-181: prepare,
FP32 dot products, select), projects the chosen raw codeword back and
subtracts it.  `LFQResidualQuantizer.encode` runs every stage of that loop
in moss_lfq_rvq_encode with the residual on chip; the loop's projection
order is the one the header defines (the upstream module is not
available), and each stage's LFQ arithmetic is the reference's.
"""

import torch
import torch.nn.functional as F

from . import _lib


class LFQResidualQuantizer:
    """Stage parameters, FP32 on one CUDA device:
    in_weight [S, 8, D], in_bias [S, 8], codebooks [S, K, 8] (raw),
    out_weight [S, D, 8], out_bias [S, D].

    The codebooks are normalised once here, as the reference does when its
    optimisation context is entered (fast_moss/v2_runtime.py:401-403:
    F.normalize of each LFQ module's weight and the sum of its squares)."""

    def __init__(self, in_weight, in_bias, codebooks, out_weight, out_bias):
        tensors = (in_weight, in_bias, codebooks, out_weight, out_bias)
        if not all(isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float32
                   for t in tensors):
            raise ValueError("stage parameters must be FP32 CUDA tensors")
        if any(t.device != codebooks.device for t in tensors):
            raise ValueError("stage parameters must share one device")
        s, k, c = codebooks.shape
        d = in_weight.shape[-1]
        if (c != 8 or in_weight.shape != (s, 8, d) or in_bias.shape != (s, 8)
                or out_weight.shape != (s, d, 8) or out_bias.shape != (s, d)):
            raise ValueError("expected in_weight [S, 8, D], in_bias [S, 8], codebooks [S, K, 8], "
                             "out_weight [S, D, 8], out_bias [S, D]")
        self.stages, self.codes, self.dim = s, k, d
        self.device = codebooks.device
        self.in_weight = in_weight.contiguous()
        self.in_bias = in_bias.contiguous()
        self.weight = codebooks.contiguous()
        self.out_weight = out_weight.contiguous()
        self.out_bias = out_bias.contiguous()
        with torch.inference_mode():
            book = torch.stack([F.normalize(w.float()) for w in self.weight])
            self.book_normed = book.contiguous()
            self.code_norm = torch.stack([b.pow(2).sum(1) for b in book]).contiguous()

    @classmethod
    def from_modules(cls, in_projs, lfqs, out_projs):
        """From the upstream stage modules: Linear(D, 8) input projections,
        LFQ modules with a `codebook` embedding [K, 8], Linear(8, D) output
        projections (Linear weights are [out, in])."""
        stack = lambda ts: torch.stack([t.detach().float() for t in ts])  # noqa: E731
        return cls(stack(p.weight for p in in_projs), stack(p.bias for p in in_projs),
                   stack(m.codebook.weight for m in lfqs), stack(p.weight for p in out_projs),
                   stack(p.bias for p in out_projs))

    def encode(self, x, *, codes=None, residual=None):
        """Quantizes x [B, D, T] FP32 through every stage; returns codes
        int64 [S, B, T].  `residual` (optional, [B, D, T]) receives the
        residual left after the last stage."""
        if (x.ndim != 3 or x.shape[1] != self.dim or x.dtype != torch.float32
                or x.device != self.device):
            raise ValueError(f"expected FP32 [B, {self.dim}, T] on {self.device}")
        x = x.contiguous()
        b, d, t = x.shape
        if codes is None:
            codes = torch.empty((self.stages, b, t), device=self.device, dtype=torch.int64)
        if codes.shape != (self.stages, b, t) or codes.dtype != torch.int64 \
                or not codes.is_contiguous():
            raise ValueError("codes must be contiguous int64 [stages, B, T]")
        if residual is not None and (residual.shape != x.shape or residual.dtype != torch.float32
                                     or not residual.is_contiguous()):
            raise ValueError("residual must be contiguous FP32 [B, D, T]")
        with torch.cuda.device(self.device):
            _lib.call("moss_lfq_rvq_encode", x.data_ptr(), b, d, t, self.stages, self.codes,
                      self.in_weight.data_ptr(), self.in_bias.data_ptr(),
                      self.book_normed.data_ptr(), self.code_norm.data_ptr(),
                      self.weight.data_ptr(), self.out_weight.data_ptr(),
                      self.out_bias.data_ptr(), codes.data_ptr(),
                      None if residual is None else residual.data_ptr(),
                      torch.cuda.current_stream(self.device).cuda_stream)
        return codes
