"""CPU: the oracle of the real codec's multi-stage LFQ quantizer is pinned
stage by stage to the reference-pinned LFQ decode.

With integer-valued projections, residuals and codebooks scaled by powers
of two, every projection sum is exact in any order, so each stage's latent
z is known exactly; the oracle loop must then pick, at every stage, the
code that oracle.lfq_decode (checked against the reference's own prepare
and select kernels by the golden vectors) picks for that z, and update the
residual exactly.  This pins everything but the projections' summation
order, which the loop defines for itself."""

import numpy as np
import pytest

from oracle import oracle as O


def _case(b, d, t, stages, k, seed):
    rng = np.random.default_rng(seed)
    x = rng.integers(-4, 5, (b, d, t)).astype(np.float32)
    w_in = rng.integers(-2, 3, (stages, 8, d)).astype(np.float32)
    b_in = rng.integers(-2, 3, (stages, 8)).astype(np.float32)
    weight = (rng.integers(-8, 9, (stages, k, 8)) / 8).astype(np.float32)
    w_out = rng.integers(-2, 3, (stages, d, 8)).astype(np.float32)
    b_out = rng.integers(-2, 3, (stages, d)).astype(np.float32)
    return x, w_in, b_in, weight, w_out, b_out


def _normalise(weight):
    n = np.sqrt((weight.astype(np.float64) ** 2).sum(-1, keepdims=True))
    book = (weight / np.maximum(n, 1e-12)).astype(np.float32)
    return book, (book * book).sum(-1).astype(np.float32)


@pytest.mark.parametrize("b,t", [(2, 7), (1, 9), (3, 1)])  # (1, 9): transposed prepare order
def test_loop_stages_match_the_pinned_decode(b, t):
    d, stages, k = 40, 4, 50
    x, w_in, b_in, weight, w_out, b_out = _case(b, d, t, stages, k, 10 * b + t)
    book, cnorm = _normalise(weight)
    codes, res = O.lfq_rvq_encode(x, w_in, b_in, book, cnorm, weight, w_out, b_out)
    r = x.astype(np.float64).copy()  # exact: every value below is a small dyadic rational
    for s in range(stages):
        z = np.einsum("jd,bdt->bjt", w_in[s].astype(np.float64), r) + b_in[s][None, :, None]
        _, idx = O.lfq_decode(z.astype(np.float32), book[s], cnorm[s], weight[s])
        assert np.array_equal(codes[s], idx), s
        c = weight[s][idx].reshape(b, t, 8).astype(np.float64)
        o = np.einsum("dj,btj->bdt", w_out[s].astype(np.float64), c) + b_out[s][None, :, None]
        r = r - o
    assert np.array_equal(res, r.astype(np.float32))
