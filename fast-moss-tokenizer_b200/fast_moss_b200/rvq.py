"""Multi-stage residual vector quantizer on B200 (encode + decode, FP32).

The stage loop of the upstream quantizer that the reference calls at
fast_moss/v2_codec.py:45, every stage selecting with the rule of
fast_moss/quantizer.py:33-39 (distance = (norm - dot) + code_norm, first
NaN, else first minimum).  The whole loop runs in ONE kernel with the
residual kept on chip across stages.  Two algorithms implement it with
identical results: "tensor_core" screens the codes with TF32 tcgen05 dot
products under a proven error margin and resolves the survivors exactly
(the default), "ffma" evaluates every distance with FP32 FMAs.  The
tensor-core algorithm has two kernels: one CTA per row block over the whole
codebook ("tensor_core_single", what "tensor_core" runs), and a CTA pair per
row block, each CTA screening half of every codebook and the two exchanging
one key per row and stage ("tensor_core_pair", for codebooks of more than
256 codes and rows within one wave of pairs).  Numerics
(the documented order the CPU oracle also follows): norm and code norms
are sequential FMAs over the
dimensions in ascending order starting from +0, dot_j = the same over
(2 r[d]) * c_j[d]; r -= c and recon += c in float32.
"""

import torch

from . import _lib


# algorithm -> tensor-core kernel selector of moss_rvq_encode_kernel (None: FFMA)
_KERNELS = {"tensor_core": 0, "tensor_core_single": 1, "tensor_core_pair": 2, "ffma": None}


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
        the kernel ("tensor_core", "tensor_core_pair", "tensor_core_single" or
        "ffma"; all give the same bits); books with more than 4096 codes use
        "ffma" under "tensor_core".  "tensor_core_pair" raises UnsupportedError
        where the pair kernel does not apply.
        """
        if algorithm not in _KERNELS:
            raise ValueError(f"Unknown algorithm {algorithm!r}")
        kernel = _KERNELS[algorithm]
        if kernel is None or (algorithm == "tensor_core" and self.codes > 4096):
            entry, extra = "moss_rvq_encode_ffma", ()
        else:
            entry, extra = "moss_rvq_encode_kernel", (kernel,)
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
                residual.data_ptr() if residual is not None else None, *extra,
                torch.cuda.current_stream(dev).cuda_stream)
        return codes, recon

    def encode_host_batches(self, xs, codes_out, recon_out, *, depth=2,
                            algorithm="tensor_core"):
        """Quantizes a sequence of batches that live in (pinned) host memory.

        xs[i]: FP32 rows [N_i, D] on the host; codes_out[i] (int32 [S, N_i])
        and recon_out[i] ([N_i, D]) are host tensors that receive the
        results.  Batch i+1 is copied in on one copy stream and batch i-1's
        results are copied out on another while batch i is quantized, with
        `depth` device buffer sets in rotation (events order every reuse).
        Work is queued on the current stream's device; on return the current
        stream waits for the last copy out (synchronize before reading the
        host outputs).  The copies overlap the quantizer only when every
        host tensor is pinned and contiguous: torch stages any other copy
        through pageable memory, which serialises it with the host.
        """
        if not len(xs) == len(codes_out) == len(recon_out):
            raise ValueError("xs, codes_out and recon_out must have the same length")
        if depth < 1:
            raise ValueError("depth must be >= 1")
        dev = self.books.device
        main = torch.cuda.current_stream(dev)
        h2d = torch.cuda.Stream(device=dev)
        d2h = torch.cuda.Stream(device=dev)
        bufs = {}
        freed = [None] * depth  # event: buffer set b may be overwritten
        for i, (xh, ch, rh) in enumerate(zip(xs, codes_out, recon_out)):
            n = xh.shape[0]
            if xh.ndim != 2 or xh.shape[1] != self.dim or xh.dtype != torch.float32 or xh.is_cuda:
                raise ValueError(f"xs[{i}] must be FP32 host rows [N, {self.dim}]")
            if ch.shape != (self.stages, n) or ch.dtype != torch.int32 or ch.is_cuda:
                raise ValueError(f"codes_out[{i}] must be an int32 host tensor [stages, N]")
            if rh.shape != (n, self.dim) or rh.dtype != torch.float32 or rh.is_cuda:
                raise ValueError(f"recon_out[{i}] must be an FP32 host tensor [N, dim]")
            b = i % depth
            x_d, c_d, r_d = bufs.get((b, n)) or bufs.setdefault((b, n), (
                torch.empty((n, self.dim), device=dev, dtype=torch.float32),
                torch.empty((self.stages, n), device=dev, dtype=torch.int32),
                torch.empty((n, self.dim), device=dev, dtype=torch.float32)))
            if freed[b] is not None:
                h2d.wait_event(freed[b])
            with torch.cuda.stream(h2d):
                x_d.copy_(xh, non_blocking=True)
                loaded = torch.cuda.Event()
                loaded.record(h2d)
            main.wait_event(loaded)
            self.encode(x_d, codes=c_d, recon=r_d, algorithm=algorithm)
            done = torch.cuda.Event()
            done.record(main)
            d2h.wait_event(done)
            with torch.cuda.stream(d2h):
                ch.copy_(c_d, non_blocking=True)
                rh.copy_(r_d, non_blocking=True)
                freed[b] = torch.cuda.Event()
                freed[b].record(d2h)
        main.wait_stream(d2h)
        main.wait_stream(h2d)

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
