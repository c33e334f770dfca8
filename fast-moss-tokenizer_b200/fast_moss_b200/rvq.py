"""Multi-stage residual vector quantizer on B200 (encode + decode, FP32).

The stage loop of the upstream quantizer that the reference calls at
fast_moss/v2_codec.py:45, every stage selecting with the rule of
fast_moss/quantizer.py:33-39 (distance = (norm - dot) + code_norm, first
NaN, else first minimum).  The whole loop runs in ONE kernel with the
residual kept on chip across stages.  Two kernels implement it with
identical results: "tensor_core" screens the codes with TF32 tcgen05 dot
products under a proven error margin and resolves the survivors exactly
(the default), "ffma" evaluates every distance with FP32 FMAs.  Numerics
(the documented order the CPU oracle also follows): norm and code norms
are sequential FMAs over the
dimensions in ascending order starting from +0, dot_j = the same over
(2 r[d]) * c_j[d]; r -= c and recon += c in float32.
"""

import torch

from . import _lib


class ResidualVectorQuantizer:
    """Holds the codebooks [S, K, 64] and their prepared device copies.

    Preparation (code norms and a k-major packed copy of the books) runs once
    at construction, like the reference's one-off codebook normalisation when
    its optimisation context is entered (fast_moss/v2_runtime.py:401-403).
    """

    def __init__(self, books):
        if books.ndim != 3 or books.dtype != torch.float32 or not books.is_cuda:
            raise ValueError("Expected CUDA FP32 codebooks [stages, codes, dim]")
        self.books = books.contiguous()
        self.stages, self.codes, self.dim = self.books.shape
        lib = _lib.load()
        floats = lib.moss_rvq_packed_floats(self.stages, self.codes, self.dim)
        kpad = -(-self.codes // 256) * 256  # codes rounded up to whole 256-code chunks
        dev = self.books.device
        self.code_norm = torch.empty((self.stages, kpad), device=dev, dtype=torch.float32)
        self.packed = torch.empty(floats, device=dev, dtype=torch.float32)
        self.stats = torch.empty((self.stages, 4), device=dev, dtype=torch.float32)
        with torch.cuda.device(dev):
            _lib.call(
                "moss_rvq_prepare_codebooks", self.books.data_ptr(), self.stages, self.codes,
                self.dim, self.code_norm.data_ptr(), self.packed.data_ptr(),
                self.stats.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)

    def _check_rows(self, x):
        if (
            x.ndim != 2 or x.shape[1] != self.dim or x.dtype != torch.float32
            or x.device != self.books.device
        ):
            raise ValueError(f"Expected FP32 rows [N, {self.dim}] on {self.books.device}")

    def encode(self, x, *, codes=None, recon=None, residual=None, algorithm="tensor_core"):
        """Quantizes rows x [N, D]; returns (codes int32 [S, N], recon [N, D]).

        Output buffers may be passed in (e.g. static buffers of a CUDA graph);
        `residual` (optional) receives the final residual.  `algorithm` picks
        the kernel ("tensor_core" or "ffma"; both give the same bits); books
        with more than 4096 codes always use "ffma".
        """
        if algorithm not in ("tensor_core", "ffma"):
            raise ValueError(f"Unknown algorithm {algorithm!r}")
        entry = "moss_rvq_encode" if algorithm == "tensor_core" and self.codes <= 4096 \
            else "moss_rvq_encode_ffma"
        self._check_rows(x)
        x = x.contiguous()
        n = x.shape[0]
        dev = x.device
        if codes is None:
            codes = torch.empty((self.stages, n), device=dev, dtype=torch.int32)
        if recon is None:
            recon = torch.empty((n, self.dim), device=dev, dtype=torch.float32)
        if codes.shape != (self.stages, n) or codes.dtype != torch.int32:
            raise ValueError("codes buffer must be int32 [stages, rows]")
        if recon.shape != (n, self.dim) or recon.dtype != torch.float32:
            raise ValueError("recon buffer must be float32 [rows, dim]")
        with torch.cuda.device(dev):
            _lib.call(
                entry, x.data_ptr(), n, self.dim, self.books.data_ptr(),
                self.packed.data_ptr(), self.code_norm.data_ptr(), self.stats.data_ptr(),
                self.stages, self.codes, codes.data_ptr(), recon.data_ptr(),
                residual.data_ptr() if residual is not None else None,
                torch.cuda.current_stream(dev).cuda_stream)
        return codes, recon

    def decode(self, codes):
        """Dequantizes int32 codes [S, N] to recon [N, D] (stage order sum)."""
        if codes.ndim != 2 or codes.shape[0] != self.stages or codes.dtype != torch.int32:
            raise ValueError("Expected int32 codes [stages, rows]")
        codes = codes.contiguous()
        n = codes.shape[1]
        recon = torch.empty((n, self.dim), device=codes.device, dtype=torch.float32)
        with torch.cuda.device(codes.device):
            _lib.call(
                "moss_rvq_decode", codes.data_ptr(), n, self.books.data_ptr(), self.stages,
                self.codes, self.dim, recon.data_ptr(),
                torch.cuda.current_stream(codes.device).cuda_stream)
        return recon
