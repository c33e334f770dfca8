"""Generates tests/golden/*.npz from the REFERENCE implementation.

Run with the reference checkout at --reference PATH (default:
$FAST_MOSS_REFERENCE, else a directory `reference` beside the repository
root).  The reference's Triton kernels (`_scale_add`,
`_rotate`, `_select`) run on the CPU under TRITON_INTERPRET=1 and its LFQ
preparation kernel runs as host code compiled by oracle/build_ref.py.  The
fixtures record inputs and the reference's outputs; the tests compare the
CPU oracle (and, on a GPU, the B200 kernels) against them.  Nothing here is
needed at test time.

Usage: python tests/golden/make_golden.py [--reference PATH]
"""

import argparse
import ctypes
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import build_ref  # noqa: E402
from oracle import oracle as O  # noqa: E402


def bf16_values(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16)


def specials(rng, shape, frac=0.05):
    """N(0,1) with a sprinkle of NaN, +-inf, -0 and subnormal values."""
    a = rng.standard_normal(shape).astype(np.float32)
    flat = a.reshape(-1)
    n = flat.size
    picks = rng.choice(n, size=max(5, int(n * frac)), replace=False)
    vals = np.array([np.nan, np.inf, -np.inf, -0.0, 1e-40, 3e38, -3e38], np.float32)
    flat[picks] = vals[np.arange(picks.size) % vals.size]
    return a


def gen_scale_add(pw, rng):
    out = {}
    cases = [
        ("f32_f32", (3, 5, 64), torch.float32, torch.float32),
        ("f32_bf16", (2, 7, 48), torch.float32, torch.bfloat16),
        ("bf16_bf16", (4, 32), torch.bfloat16, torch.bfloat16),
        ("bf16_f32", (1, 3, 20), torch.bfloat16, torch.float32),
    ]
    for name, shape, xd, ud in cases:
        x = torch.from_numpy(specials(rng, shape)).to(xd)
        u = torch.from_numpy(specials(rng, shape)).to(ud)
        s = torch.from_numpy((0.01 * rng.standard_normal(shape[-1])).astype(np.float32))
        y = torch.empty(shape, dtype=torch.float32)
        pw._scale_add[(triton_cdiv(x.numel(), 256),)](
            x, u, s, y, x.numel(), shape[-1], 256, enable_fp_fusion=False)
        out[f"{name}_x"] = x.float().numpy()
        out[f"{name}_u"] = u.float().numpy()
        out[f"{name}_xbf16"] = np.array(xd == torch.bfloat16)
        out[f"{name}_ubf16"] = np.array(ud == torch.bfloat16)
        out[f"{name}_s"] = s.numpy()
        out[f"{name}_y"] = y.numpy()
    out["cases"] = np.array([c[0] for c in cases])
    return out


def triton_cdiv(a, b):
    return (a + b - 1) // b


def gen_rotate(pw, rng):
    out = {}
    # bf16 q/k as views of a [B, T, 3, H, D] qkv projection output.
    b, t, h, d = 2, 5, 3, 16
    qkv = torch.from_numpy(specials(rng, (b, t, 3, h, d), 0.02)).to(torch.bfloat16)
    q = qkv[:, :, 0].transpose(1, 2)
    k = qkv[:, :, 1].transpose(1, 2)
    cases = {"bf16_view": (q, k)}
    qf = torch.from_numpy(rng.standard_normal((1, 2, 7, 8)).astype(np.float32))
    kf = torch.from_numpy(rng.standard_normal((1, 2, 7, 8)).astype(np.float32))
    cases["f32_contig"] = (qf, kf)
    for name, (q, k) in cases.items():
        bb, hh, tt, dd = q.shape
        phase = torch.from_numpy(rng.uniform(-50, 50, (bb, tt, dd // 2)).astype(np.float32))
        cos, sin = torch.cos(phase), torch.sin(phase)
        # The interpreter truncates on a float32 -> bf16 store while the
        # compiled kernel rounds to nearest even (cvt.rn), so the kernel runs
        # with float32 output buffers and the GPU's RNE cast is applied after.
        oq = torch.empty((bb, hh, tt, dd), dtype=torch.float32)
        ok = torch.empty_like(oq)
        n = q.numel() // 2
        pw._rotate[(triton_cdiv(n, 256),)](
            q, k, cos, sin, oq, ok, n, hh, tt, dd, *q.stride(), *k.stride(), 256,
            enable_fp_fusion=False)
        oq, ok = oq.to(q.dtype), ok.to(q.dtype)
        out[f"{name}_q"] = q.float().contiguous().numpy()
        out[f"{name}_k"] = k.float().contiguous().numpy()
        out[f"{name}_qbase"] = (qkv.float().numpy() if name == "bf16_view" else q.numpy())
        out[f"{name}_bf16"] = np.array(q.dtype == torch.bfloat16)
        out[f"{name}_cos"] = cos.numpy()
        out[f"{name}_sin"] = sin.numpy()
        out[f"{name}_oq"] = oq.float().numpy()
        out[f"{name}_ok"] = ok.float().numpy()
    out["cases"] = np.array(list(cases))
    return out


def ref_select(qz, dots, norm, cnorm, book, lat, ste):
    b, d, t = lat.shape
    k = book.shape[0]
    idx = torch.empty((b, t), dtype=torch.long)
    outp = torch.empty((b, d, t) if ste else (b, t, d), dtype=torch.float32)
    qz._select[(b * t,)](
        dots, norm, cnorm, book, lat, outp, idx, k, d, t, *lat.stride(), ste,
        next_pow2(k), next_pow2(d), num_warps=4, enable_fp_fusion=False)
    return outp, idx


def next_pow2(v):
    p = 1
    while p < v:
        p *= 2
    return p


def gen_select(qz, rng):
    out = {}
    cases = []
    for name, (b, d, t, k, ste) in {
        "plain": (2, 8, 3, 37, False),
        "ste": (2, 8, 3, 37, True),
        "single_code": (1, 8, 4, 1, False),
        "wide": (3, 5, 2, 300, False),
    }.items():
        lat = torch.from_numpy(rng.standard_normal((b, d, t)).astype(np.float32))
        book = torch.from_numpy(rng.standard_normal((k, d)).astype(np.float32))
        dots = torch.from_numpy(rng.standard_normal((b * t, k)).astype(np.float32))
        norm = torch.from_numpy(rng.standard_normal((b * t, 1)).astype(np.float32))
        cnorm = torch.from_numpy(rng.standard_normal((1, k)).astype(np.float32))
        if k > 4:
            dots[0, 3] = dots[0, 1]  # exact ties: the first one must win
            cnorm[0, 3] = cnorm[0, 1]
            dots[1, 2] = float("nan")  # a NaN row: the first NaN wins
            dots[1, 4] = float("nan")
            dots[min(2, b * t - 1), :] = float("inf")  # all distances -inf
        outp, idx = ref_select(qz, dots, norm, cnorm, book, lat, ste)
        for key, val in (("lat", lat), ("book", book), ("dots", dots), ("norm", norm),
                         ("cnorm", cnorm), ("out", outp), ("idx", idx)):
            out[f"{name}_{key}"] = val.numpy()
        out[f"{name}_ste"] = np.array(ste)
        cases.append(name)
    out["cases"] = np.array(cases)
    return out


def gen_prepare(rng):
    lib = ctypes.CDLL(build_ref.build(force=True))
    out = {}
    cases = {"transposed": (1, 9), "contiguous": (3, 4), "single": (1, 1), "batch_t1": (5, 1)}
    for name, (b, t) in cases.items():
        x = rng.standard_normal((b, 8, t)).astype(np.float32)
        if b * t > 2:
            x[0, :, 0] = 0.0  # denominator clamp
            x[0, 3, 1 % t] = np.nan
            x[-1, 5, -1] = 1e-30
        transposed = b == 1 and t > 1
        e = np.zeros((8, t) if transposed else (b * t, 8), np.float32)
        tw = np.zeros_like(e)
        norm = np.zeros(b * t, np.float32)
        den = np.zeros(b * t, np.float32)
        p = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
        lib.ref_prepare(p(x), p(e), p(norm), p(tw), p(den), ctypes.c_int(b), ctypes.c_int(t))
        for key, val in (("x", x), ("e", e), ("twice", tw), ("norm", norm), ("denom", den)):
            out[f"{name}_{key}"] = val
    out["cases"] = np.array(list(cases))
    return out


def gen_rvq(qz, rng):
    """Small residual VQ whose per-stage selection is the reference's `_select`
    kernel applied to the pinned-order norms and dot products."""
    rows, d, k, stages = 12, 64, 37, 3
    x = rng.standard_normal((rows, d)).astype(np.float32)
    books = (rng.standard_normal((stages, k, d)) / 8).astype(np.float32)
    books[1, 5] = books[1, 2]  # duplicate codeword: ties resolved to the first
    cn = O.rvq_code_norms(books)
    r = x.copy()
    recon = np.zeros_like(x)
    codes = np.zeros((stages, rows), np.int32)
    for s in range(stages):
        norms = np.zeros((rows, 1), np.float32)
        dots = np.zeros((rows, k), np.float32)
        for i in range(rows):
            norms[i, 0], dots[i] = O.rvq_stage_terms(r[i], books[s])
        lat = torch.zeros((rows, d, 1))
        _, idx = ref_select(qz, torch.from_numpy(dots), torch.from_numpy(norms),
                            torch.from_numpy(cn[s][None]), torch.from_numpy(books[s]), lat, False)
        idx = idx.numpy()[:, 0]
        codes[s] = idx
        c = books[s][idx]
        r = (r - c).astype(np.float32)
        recon = (recon + c).astype(np.float32)
    return {"x": x, "books": books, "codes": codes, "recon": recon, "residual": r}


def gen_lfq_decode(qz, rng):
    """LFQ decode = reference prepare + sequential-FMA dots + reference select."""
    lib = ctypes.CDLL(build_ref.build())
    out = {}
    k = 64
    weight = rng.standard_normal((k, 8)).astype(np.float32)
    wn = weight / np.maximum(np.linalg.norm(weight.astype(np.float64), axis=1, keepdims=True), 1e-12)
    book_normed = wn.astype(np.float32)
    cnorm = np.zeros((1, k), np.float32)
    for j in range(k):  # any fixed rounding: it is an input of the decode
        acc = np.float32(0)
        for q in range(8):
            acc = np.float32(acc + np.float32(book_normed[j, q] * book_normed[j, q]))
        cnorm[0, j] = acc
    for name, (b, t) in {"transposed": (1, 6), "contiguous": (2, 3)}.items():
        x = rng.standard_normal((b, 8, t)).astype(np.float32)
        transposed = b == 1 and t > 1
        e = np.zeros((8, t) if transposed else (b * t, 8), np.float32)
        tw = np.zeros_like(e)
        norm = np.zeros(b * t, np.float32)
        den = np.zeros(b * t, np.float32)
        p = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
        lib.ref_prepare(p(x), p(e), p(norm), p(tw), p(den), ctypes.c_int(b), ctypes.c_int(t))
        twr = np.ascontiguousarray(tw.T if transposed else tw)  # [b*t, 8]
        dots = lfq_dots(twr, book_normed)
        outp, idx = ref_select(qz, torch.from_numpy(dots), torch.from_numpy(norm[:, None]),
                               torch.from_numpy(cnorm), torch.from_numpy(weight),
                               torch.from_numpy(x), False)
        out[f"{name}_x"] = x
        out[f"{name}_out"] = outp.numpy().reshape(b * t, 8)
        out[f"{name}_idx"] = idx.numpy().reshape(-1)
    out["weight"] = weight
    out["book_normed"] = book_normed
    out["cnorm"] = cnorm
    out["cases"] = np.array(["transposed", "contiguous"])
    return out


def lfq_dots(tw, book):
    """dot = tw0*c0 then seven FMAs, evaluated exactly through float64."""
    n, k = tw.shape[0], book.shape[0]
    dots = np.zeros((n, k), np.float32)
    for i in range(n):
        for j in range(k):
            acc = np.float32(np.float64(tw[i, 0]) * np.float64(book[j, 0]))
            for q in range(1, 8):
                acc = fma32(tw[i, q], book[j, q], acc)
            dots[i, j] = acc
    return dots


def fma32(a, b, c):
    """Correctly rounded float32 fma via exact rational arithmetic."""
    from fractions import Fraction
    v = Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c))
    return np.float32(round_fraction_to_f32(v))


def round_fraction_to_f32(v):
    from fractions import Fraction
    if v == 0:
        return 0.0
    f64 = float(v)  # nearest double
    f32 = np.float32(f64)
    # Correct a possible double rounding by checking the two f32 neighbours.
    cands = [f32, np.nextafter(f32, np.float32(np.inf)), np.nextafter(f32, np.float32(-np.inf))]
    best = min(cands, key=lambda c: (abs(Fraction(float(c)) - v),
                                     int(np.frombuffer(np.float32(c).tobytes(), np.uint32)[0]) & 1))
    return float(best)


def main():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", default=build_ref.DEFAULT_REFERENCE)
    args = parser.parse_args()
    sys.path.insert(0, args.reference)
    from fast_moss import quantizer as qz  # the reference package
    from fast_moss import v2_pointwise as pw

    rng = np.random.default_rng(20261201)
    np.savez_compressed(os.path.join(HERE, "scale_add.npz"), **gen_scale_add(pw, rng))
    np.savez_compressed(os.path.join(HERE, "rotate.npz"), **gen_rotate(pw, rng))
    np.savez_compressed(os.path.join(HERE, "select.npz"), **gen_select(qz, rng))
    np.savez_compressed(os.path.join(HERE, "prepare.npz"), **gen_prepare(rng))
    np.savez_compressed(os.path.join(HERE, "rvq_small.npz"), **gen_rvq(qz, rng))
    np.savez_compressed(os.path.join(HERE, "lfq_decode.npz"), **gen_lfq_decode(qz, rng))
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
