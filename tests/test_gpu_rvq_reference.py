"""GPU parity of the 32-stage RVQ against the reference's own per-stage
arithmetic, run on the same B200.

The reference selects a code per stage with an FP32 cuBLAS GEMM for the dot
products (`dots = twice @ book.T`, TF32 off: fast_moss/v2_runtime.py:179,
fast_moss/v2_loading.py:11-15) followed by its selection kernel
(fast_moss/quantizer.py:8-49: distance = (norm - dots) + code_norm, first
NaN, else first minimum; here `moss_lfq_select`, which is bit-exact against
that kernel's golden vectors).  cuBLAS sums each dot product in its own
internal order, which is not published and cannot be reproduced, so the
tensor-core kernel (and the oracle) pin a sequential-FMA order instead.  The
two orders can then only disagree on near ties, and this test proves that
every disagreement is one.

Error bound.  With u = 2^-24, any FP32 evaluation of an inner product of
n = 64 terms -- in any summation order, with or without fused multiply-adds
-- is within gamma_64 = 64u / (1 - 64u) of sum |x_d y_d| (Higham, Accuracy
and Stability of Numerical Algorithms, 2nd ed., section 3.1).  That covers
the row norm N = sum r_d^2, the code norm C_j = sum c_jd^2 and the dot
A_j = sum (2 r_d) c_jd (2 r_d is exact) of either implementation, and the
two roundings of (N - dot) + C_j add at most 2.01u (N + |A|_j + C_j).  So
each implementation's distance d_j lies within
    E_j = 70 u (N + sum_d |2 r_d c_jd| + C_j)
of the exact distance D_j = sum_d (r_d - c_jd)^2 of the same FP32 residual.
If one picks i and the other j != i, then |D_i - D_j| <= E_i + E_j: the two
candidates are a near tie.  D and E are evaluated in float64 (error ~1e-13,
covered by an absolute slack of 1e-9).

Two checks at the benchmark's RVQ configuration (8192 x 64 frames, 32 x
1024 x 64 codebooks, seed 1):
  * teacher-forced: every stage's selection by the reference arithmetic on
    the tensor-core kernel's own residual of that stage (all 262,144
    decisions), each disagreement a near tie, and at most 1e-3 of them;
  * free-running: the reference loop run on its own, codes equal to the
    kernel's for at least 0.999 of (stage, frame) pairs, and in every frame
    the first stage where the loops part is a near tie (up to that stage the
    two residuals are bit-identical: r -= c is one FP32 subtraction in both).
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

U = 2.0 ** -24
BOUND_UNITS = 70.0
FLIP_RATE_MAX = 1e-3


def config2(device):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((8192, 64)).astype(np.float32)
    books = (rng.standard_normal((32, 1024, 64)) / 8).astype(np.float32)
    return torch.from_numpy(x).to(device), torch.from_numpy(books).to(device)


def reference_stage(moss, r, book, book_t, cnorm):
    """One stage of the reference: twice = 2r, norm = sum r^2 (torch), the
    FP32 GEMM with TF32 off (cuBLAS), the selection kernel.  Returns int64
    indices [rows] and the picked codewords [rows, 64]."""
    twice = r * 2.0
    norm = (r * r).sum(dim=1, keepdim=True)
    dots = twice @ book_t
    values, idx = moss.select(dots, norm, cnorm, book, r.t().unsqueeze(0))
    return idx[0], values.transpose(1, 2)[0]


def near_tie(r, book, i, j):
    """(|D_i - D_j|, E_i + E_j) in float64 for residual r and codes i, j."""
    r64 = r.astype(np.float64)
    ci = book[i].astype(np.float64)
    cj = book[j].astype(np.float64)
    n = float(np.sum(r64 * r64))

    def dist_and_err(c):
        d = float(np.sum((r64 - c) ** 2))
        e = BOUND_UNITS * U * (n + float(np.sum(np.abs(2.0 * r64 * c))) + float(np.sum(c * c)))
        return d, e

    di, ei = dist_and_err(ci)
    dj, ej = dist_and_err(cj)
    return abs(di - dj), ei + ej + 1e-9


@pytest.fixture(scope="module")
def run(moss, cuda_device):
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        x, books = config2(cuda_device)
        q = moss.ResidualVectorQuantizer(books)
        residual = torch.empty_like(x)
        codes, recon = q.encode(x, residual=residual)
        books_t = books.transpose(1, 2).contiguous()
        cnorm = books.pow(2).sum(-1).unsqueeze(1).contiguous()
        yield x, books, books_t, cnorm, codes.long(), recon, residual
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def test_teacher_forced_stages_differ_only_on_near_ties(moss, run):
    x, books, books_t, cnorm, codes, _, residual = run
    r = x.clone()
    ref_codes = torch.empty_like(codes)
    flips = []  # (stage, frame, kernel code, reference code, residual)
    for s in range(books.shape[0]):
        idx, _ = reference_stage(moss, r, books[s], books_t[s], cnorm[s])
        ref_codes[s] = idx
        diff = torch.nonzero(idx != codes[s]).flatten()
        for f in diff.tolist():
            flips.append((s, f, int(codes[s, f]), int(idx[f]), r[f].cpu().numpy()))
        r = r - books[s][codes[s]]  # the kernel's own residual update
    # teacher forcing followed the kernel exactly
    assert torch.equal(r, residual)
    rate = len(flips) / codes.numel()
    assert rate <= FLIP_RATE_MAX, f"{len(flips)} of {codes.numel()} decisions differ"
    books_np = books.cpu().numpy()
    worst = 0.0
    for s, f, i, j, rr in flips:
        gap, bound = near_tie(rr, books_np[s], i, j)
        assert gap <= bound, (s, f, i, j, gap, bound)
        worst = max(worst, gap / bound)
    print(f"teacher-forced: {len(flips)} of {codes.numel()} decisions differ "
          f"(rate {rate:.2e}); largest gap / bound {worst:.3f}")


def test_free_running_loops_part_only_on_near_ties(moss, run):
    x, books, books_t, cnorm, codes, _, _ = run
    r = x.clone()
    ref_codes = torch.empty_like(codes)
    first = {}  # frame -> (stage, residual before that stage)
    for s in range(books.shape[0]):
        idx, picked = reference_stage(moss, r, books[s], books_t[s], cnorm[s])
        ref_codes[s] = idx
        diff = torch.nonzero(idx != codes[s]).flatten().tolist()
        new = [f for f in diff if f not in first]
        if new:
            rows = r[new].cpu().numpy()
            for f, rr in zip(new, rows):
                first[f] = (s, rr)
        r = r - picked
    agree = float((ref_codes == codes).float().mean())
    assert agree >= 1.0 - FLIP_RATE_MAX, agree
    books_np = books.cpu().numpy()
    codes_np = codes.cpu().numpy()
    ref_np = ref_codes.cpu().numpy()
    for f, (s, rr) in first.items():
        gap, bound = near_tie(rr, books_np[s], codes_np[s, f], ref_np[s, f])
        assert gap <= bound, (s, f, gap, bound)
    print(f"free-running: codes equal for {agree:.6f} of (stage, frame) pairs; "
          f"{len(first)} frames part, each first at a near tie")
