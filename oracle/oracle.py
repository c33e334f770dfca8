"""CPU oracle for the MOSS Audio Tokenizer v2 hot path -- TEST INFRASTRUCTURE.

numpy front end of moss_oracle.c (built on first use with gcc into
oracle/_build/).  Only the tests, the smoke check and the benchmark's CPU
baseline use this module, and only as the checker; the product package
never imports it.  Every function cites the reference code it restates.
"""

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "moss_oracle.c")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(BUILD, "libmoss_oracle.so")
CFLAGS = ["-O3", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-shared", "-fPIC",
          "-fvisibility=hidden"]

_lib = None


def build(force=False):
    """Compiles the oracle; returns the shared-library path."""
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        os.makedirs(BUILD, exist_ok=True)
        tmp = LIB + f".{os.getpid()}.tmp"
        subprocess.run(["gcc", *CFLAGS, SRC, "-o", tmp, "-lm"], check=True)
        os.replace(tmp, LIB)
    return LIB


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        _lib.oracle_max_threads.restype = ctypes.c_int
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _i64(v):
    return ctypes.c_int64(int(v))


def max_threads():
    """Host threads the oracle may use: every CPU this process may run on
    (launchers such as torchrun set OMP_NUM_THREADS=1, which would otherwise
    cap the OpenMP default)."""
    import os

    try:
        n = len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        n = os.cpu_count() or 1
    return max(1, n)


def bf16_round(x):
    """Round-to-nearest-even to bfloat16 (values returned as float32)."""
    x = _f32(x)
    y = np.empty_like(x)
    lib().oracle_bf16_round(_p(x), _p(y), _i64(x.size))
    return y


def scale_add(x, u, s):
    """fast_moss/v2_pointwise.py:92-98: x + u*s[i % C], unfused, float32."""
    x, u, s = _f32(x), _f32(u), _f32(s)
    y = np.empty(x.shape, np.float32)
    lib().oracle_scale_add(_p(x), _p(u), _p(s), _p(y), _i64(x.size), _i64(s.size))
    return y


def layer_norm(x, gamma, beta, eps=1e-5, mean_variant=0, rstd=None):
    """torch CUDA vectorised layer norm (called at fast_moss/v2_runtime.py:259).

    Returns (y, mean, var_plus_eps, rstd).  With `rstd` given (per row), the
    output uses those values, e.g. the device's rsqrtf results.
    """
    x = _f32(x)
    n = x.shape[-1]
    rows = x.size // n
    g = None if gamma is None else _f32(gamma)
    b = None if beta is None else _f32(beta)
    r_in = None if rstd is None else _f32(rstd).reshape(rows)
    y = np.empty(x.shape, np.float32)
    mean = np.empty(rows, np.float32)
    ve = np.empty(rows, np.float32)
    r_out = np.empty(rows, np.float32)
    lib().oracle_layer_norm(_p(x), None if g is None else _p(g), None if b is None else _p(b),
                            ctypes.c_float(eps), _i64(rows), _i64(n), ctypes.c_int(mean_variant),
                            None if r_in is None else _p(r_in), _p(y), _p(mean), _p(ve),
                            _p(r_out))
    return y, mean, ve, r_out


def rotate(q, k, cos, sin, bf16):
    """fast_moss/v2_pointwise.py:8-47: interleaved-pair rotation, unfused.

    q, k: float32 arrays holding the input values (any strides); returns
    contiguous (oq, ok) as float32 values, rounded to bf16 if `bf16`.
    """
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    b, h, t, d = q.shape
    qs = (ctypes.c_int64 * 4)(*[s // 4 for s in q.strides])
    ks = (ctypes.c_int64 * 4)(*[s // 4 for s in k.strides])
    cs, sn = _f32(cos), _f32(sin)
    oq = np.empty((b, h, t, d), np.float32)
    ok = np.empty((b, h, t, d), np.float32)
    lib().oracle_rotate(_p(q), _p(k), qs, ks, _p(cs), _p(sn), _i64(b), _i64(h), _i64(t), _i64(d),
                        ctypes.c_int(1 if bf16 else 0), _p(oq), _p(ok))
    return oq, ok


def rope_tables(offset, t, d, coef):
    """fast_moss/v2_runtime.py:209-222 in double-precision libm (approximate)."""
    off = _f32(offset)
    b = off.size
    cs = np.empty((b, t, d // 2), np.float32)
    sn = np.empty_like(cs)
    lib().oracle_rope_tables(_p(off), _i64(b), _i64(t), _i64(d), ctypes.c_float(coef), _p(cs),
                             _p(sn))
    return cs, sn


ACTS = {"silu": 0, "gelu": 1, "gelu_tanh": 2}


def gated_act(x, bias, act="silu", gated=True, bf16=True):
    """Eager torch chain: round(x+b) -> round(act(gate)) -> round(a * up)."""
    x = _f32(x)
    width = x.shape[-1]
    rows = x.size // width
    b = None if bias is None else _f32(bias)
    out_w = width // 2 if gated else width
    y = np.empty(x.shape[:-1] + (out_w,), np.float32)
    lib().oracle_gated_act(_p(x), None if b is None else _p(b), _p(y), _i64(rows), _i64(width),
                           ctypes.c_int(ACTS[act]), ctypes.c_int(1 if gated else 0),
                           ctypes.c_int(1 if bf16 else 0))
    return y


def lfq_prepare(x):
    """fast_moss/quantizer_prepare.py:17-57 for x [b,8,t]; returns
    (e, norm, twice, denom) with e/twice shaped [8,t] when b == 1 < t
    (the reference returns its transpose view) else [b*t, 8]."""
    x = _f32(x)
    b, _, t = x.shape
    transposed = b == 1 and t > 1
    shape = (8, t) if transposed else (b * t, 8)
    e = np.empty(shape, np.float32)
    tw = np.empty(shape, np.float32)
    norm = np.empty(b * t, np.float32)
    den = np.empty(b * t, np.float32)
    lib().oracle_lfq_prepare(_p(x), _i64(b), _i64(t), _p(e), _p(norm), _p(tw), _p(den))
    return e, norm, tw, den


def lfq_select(dots, row_norm, code_norm, book, latents, straight_through=False):
    """fast_moss/quantizer.py:29-49: returns (out, indices); out is [b*t, d]
    without STE and [b, d, t] with STE."""
    dots, row_norm, code_norm, book = _f32(dots), _f32(row_norm), _f32(code_norm), _f32(book)
    lat = np.asarray(latents, np.float32)
    b, d, t = lat.shape
    k = book.shape[0]
    ls = (ctypes.c_int64 * 3)(*[s // 4 for s in lat.strides])
    out = np.empty((b, d, t) if straight_through else (b * t, d), np.float32)
    idx = np.empty(b * t, np.int64)
    lib().oracle_lfq_select(_p(dots), _p(row_norm), _p(code_norm), _p(book), _p(lat), ls, _i64(b),
                            _i64(d), _i64(t), _i64(k), ctypes.c_int(1 if straight_through else 0),
                            _p(out), _p(idx))
    return out, idx


def lfq_decode(x, book_normed, code_norm, weight):
    """fast_moss/v2_runtime.py:143-181 with sequential-FMA dots; returns
    (values [b*t, 8], indices [b*t])."""
    x, bn, cn, w = _f32(x), _f32(book_normed), _f32(code_norm), _f32(weight)
    b, _, t = x.shape
    k = bn.shape[0]
    out = np.empty((b * t, 8), np.float32)
    idx = np.empty(b * t, np.int64)
    lib().oracle_lfq_decode(_p(x), _p(bn), _p(cn), _p(w), _i64(b), _i64(t), _i64(k), _p(out),
                            _p(idx))
    return out, idx


def lfq_rvq_encode(x, w_in, b_in, book_normed, code_norm, weight, w_out, b_out):
    """The multi-stage LFQ quantizer of the real codec in the loop order
    moss_oracle.c defines (projections) around the reference's LFQ decode of
    every stage; x [b, d, t].  Returns (codes int64 [stages, b*t], final
    residual [b, d, t])."""
    x = _f32(x)
    w_in, b_in, bn, cn = _f32(w_in), _f32(b_in), _f32(book_normed), _f32(code_norm)
    weight, w_out, b_out = _f32(weight), _f32(w_out), _f32(b_out)
    b, d, t = x.shape
    stages, k, _ = bn.shape
    codes = np.empty((stages, b * t), np.int64)
    res = np.empty_like(x)
    lib().oracle_lfq_rvq_encode(_p(x), _i64(b), _i64(d), _i64(t), _i64(stages), _i64(k),
                                _p(w_in), _p(b_in), _p(bn), _p(cn), _p(weight), _p(w_out),
                                _p(b_out), _p(codes), _p(res))
    return codes, res


def rvq_code_norms(books):
    """sum_d c^2 per code, sequential FMA (books [stages, k, d])."""
    books = _f32(books)
    s, k, d = books.shape
    cn = np.empty((s, k), np.float32)
    lib().oracle_rvq_code_norms(_p(books), _i64(s), _i64(k), _i64(d), _p(cn))
    return cn


def rvq_encode(x, books, nthreads=0, residual=False):
    """Multi-stage residual VQ (selection rule of fast_moss/quantizer.py:33-39,
    loop of the upstream quantizer called at fast_moss/v2_codec.py:45).
    Returns (codes int32 [stages, rows], recon [rows, d]) and the final
    residual when `residual`."""
    x, books = _f32(x), _f32(books)
    rows, d = x.shape
    s, k, _ = books.shape
    cn = rvq_code_norms(books)
    codes = np.empty((s, rows), np.int32)
    recon = np.empty((rows, d), np.float32)
    res = np.empty((rows, d), np.float32) if residual else None
    lib().oracle_rvq_encode(_p(x), _i64(rows), _i64(d), _p(books), _p(cn), _i64(s), _i64(k),
                            _p(codes), _p(recon), None if res is None else _p(res),
                            ctypes.c_int(int(nthreads)))
    return (codes, recon, res) if residual else (codes, recon)


def rvq_stage_terms(r, book):
    """(norm, dots) of one residual row against one book, pinned order."""
    r, book = _f32(r), _f32(book)
    k, d = book.shape
    dots = np.empty(k, np.float32)
    norm = np.empty(1, np.float32)
    lib().oracle_rvq_stage_terms(_p(r), _i64(d), _p(book), _i64(k), _p(norm), _p(dots))
    return norm[0], dots


def rvq_decode(codes, books):
    """recon = sum_s books[s][codes[s]] in stage order from +0."""
    codes = np.ascontiguousarray(codes, np.int32)
    books = _f32(books)
    s, k, d = books.shape
    rows = codes.shape[1]
    recon = np.empty((rows, d), np.float32)
    lib().oracle_rvq_decode(_p(codes), _i64(rows), _p(books), _i64(s), _i64(k), _i64(d),
                            _p(recon))
    return recon
