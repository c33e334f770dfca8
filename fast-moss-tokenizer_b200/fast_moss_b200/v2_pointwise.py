"""Pointwise hot-path ops on B200: residual, LayerNorm, RoPE, gated activation.

`rotate` and `scale_add` keep the names, argument meaning, validation and
exception types of fast_moss/v2_pointwise.py (rotate :50-89, scale_add
:101-122); the remaining functions are the fused forms the optimized
transformer layer uses.  Every op launches a kernel of libfast_moss_b200 on
the current CUDA stream; there is no other implementation behind them.
"""

import math

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16}


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


def rotate(q, k, cos, sin):
    """Interleaved-pair rotation of q and k by FP32 tables [B,T,D/2].

    Returns contiguous B,H,T,D tensors of q's dtype (reference
    fast_moss/v2_pointwise.py:50-89).
    """
    if q.ndim != 4 or q.shape != k.shape or q.shape[-1] < 2 or q.shape[-1] % 2:
        raise ValueError("Expected equal B,H,T,even-D rotary inputs")
    b, h, t, d = q.shape
    if (
        q.dtype not in _DTYPES
        or k.dtype != q.dtype
        or cos.dtype != torch.float32
        or sin.dtype != torch.float32
        or not q.is_cuda
        or any(x.device != q.device for x in (k, cos, sin))
        or cos.shape != (b, t, d // 2)
        or sin.shape != cos.shape
        or not cos.is_contiguous()
        or not sin.is_contiguous()
    ):
        raise ValueError(
            "Expected same-device BF16/FP32 Q/K and contiguous FP32 rotary tables"
        )
    oq = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    ok = torch.empty_like(oq)
    if q.numel():
        with torch.cuda.device(q.device):
            _lib.call(
                "moss_rotate", q.data_ptr(), k.data_ptr(), _DTYPES[q.dtype], cos.data_ptr(),
                sin.data_ptr(), oq.data_ptr(), ok.data_ptr(), b, h, t, d,
                _lib.strides(q.stride()), _lib.strides(k.stride()), _stream(q.device))
    return oq, ok


def rope(q, k, offset, max_period):
    """Rotary embedding with the phase computed inside the kernel.

    Same result as the reference's patched rotary forward
    (fast_moss/v2_runtime.py:209-224): freq = exp(arange(d/2) * c) with
    c = float32(-ln(max_period) * 2 / d), phase = freq * (offset + t),
    cos/sin of the phase, then `rotate` -- without materialising the tables.
    offset: [B] integer or float tensor on q's device.
    """
    if q.ndim != 4 or q.shape != k.shape or q.shape[-1] < 2 or q.shape[-1] % 2:
        raise ValueError("Expected equal B,H,T,even-D rotary inputs")
    b, h, t, d = q.shape
    if (
        q.dtype not in _DTYPES
        or k.dtype != q.dtype
        or not q.is_cuda
        or k.device != q.device
        or offset.device != q.device
        or offset.numel() != b
    ):
        raise ValueError("Expected same-device BF16/FP32 Q/K and a per-batch offset")
    if offset.dtype == torch.int64:
        odt = 0
    elif offset.dtype == torch.int32:
        odt = 1
    else:
        odt = 2
        offset = offset.float()
    offset = offset.contiguous()
    coef = -math.log(max_period) * 2 / d
    oq = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    ok = torch.empty_like(oq)
    if q.numel():
        with torch.cuda.device(q.device):
            _lib.call(
                "moss_rope", q.data_ptr(), k.data_ptr(), _DTYPES[q.dtype], offset.data_ptr(), odt,
                coef, oq.data_ptr(), ok.data_ptr(), b, h, t, d, _lib.strides(q.stride()),
                _lib.strides(k.stride()), _stream(q.device))
    return oq, ok


def rope_kv(q, k, v, offset, max_period, slots, k_cache, v_cache):
    """`rope` with the rotated keys and the values written into a history ring.

    q, k, v: [B, H, T, D] (any strides, same dtype); offset: [B] on q's
    device; slots: int64 [B, T] on q's device, the ring slot of every token;
    k_cache, v_cache: contiguous [B, H, S, D] of q's dtype.  Returns the
    rotated q (contiguous); k_cache[b, h, slots[b, t]] receives the rotated
    key and v_cache the value.  Same bits as `rope` followed by
    `k_cache.scatter_(2, ...)` / `v_cache.scatter_(2, ...)`.
    """
    if q.ndim != 4 or q.shape != k.shape or q.shape != v.shape or q.shape[-1] % 2:
        raise ValueError("Expected equal B,H,T,even-D q, k and v")
    b, h, t, d = q.shape
    if (
        q.dtype not in _DTYPES
        or k.dtype != q.dtype
        or v.dtype != q.dtype
        or not q.is_cuda
        or any(x.device != q.device for x in (k, v, offset, slots, k_cache, v_cache))
        or offset.numel() != b
        or slots.shape != (b, t)
        or slots.dtype != torch.int64
        or k_cache.ndim != 4
        or k_cache.shape[:2] != (b, h)
        or k_cache.shape[3] != d
        or v_cache.shape != k_cache.shape
        or k_cache.dtype != q.dtype
        or v_cache.dtype != q.dtype
        or not k_cache.is_contiguous()
        or not v_cache.is_contiguous()
    ):
        raise ValueError("Expected same-device q/k/v, [B] offset, int64 [B,T] slots and "
                         "contiguous [B,H,S,D] caches of q's dtype")
    if offset.dtype == torch.int64:
        odt = 0
    elif offset.dtype == torch.int32:
        odt = 1
    else:
        odt = 2
        offset = offset.float()
    offset = offset.contiguous()
    slots = slots.contiguous()
    coef = -math.log(max_period) * 2 / d
    oq = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    if q.numel():
        with torch.cuda.device(q.device):
            _lib.call(
                "moss_rope_kv", q.data_ptr(), k.data_ptr(), v.data_ptr(), _DTYPES[q.dtype],
                offset.data_ptr(), odt, coef, slots.data_ptr(), oq.data_ptr(),
                k_cache.data_ptr(), v_cache.data_ptr(), b, h, t, d, k_cache.shape[2],
                _lib.strides(q.stride()), _lib.strides(k.stride()), _lib.strides(v.stride()),
                _stream(q.device))
    return oq


def history_attention(q, k_cache, v_cache, slot_pos, pos, context, scale=None, out=None):
    """Attention of a chunk's queries over a streaming history ring.

    q: bf16 [S, H, T, 64] (T <= 8); k_cache, v_cache: contiguous bf16
    [S, H, N, 64] rings (N <= 512); slot_pos: int64 [S, N], the position held
    by each slot (-1 = empty); pos: int64 [S], the position of the chunk's
    first token.  Query t attends to the slots holding positions in
    (pos + t - context, pos + t] -- the mask of the streaming history -- with
    scale 1/sqrt(64) by default.  Returns bf16 [S, T, H, 64] (or fills
    `out`), the layout the output projection reads.  Replaces the SDPA call
    over the bounded history (fast_moss/v2_runtime.py:40-41, :254-262;
    fast_moss/streaming.py:68-79); FP32 arithmetic with one bf16 rounding.
    """
    if q.ndim != 4 or k_cache.ndim != 4:
        raise ValueError("Expected q [S, H, T, D] and caches [S, H, N, D]")
    s, h, t, d = q.shape
    n = k_cache.shape[2]
    if (
        q.dtype != torch.bfloat16
        or k_cache.dtype != torch.bfloat16
        or v_cache.dtype != torch.bfloat16
        or not q.is_cuda
        or any(x.device != q.device for x in (k_cache, v_cache, slot_pos, pos))
        or k_cache.shape[:2] != (s, h)
        or k_cache.shape[3] != d
        or v_cache.shape != k_cache.shape
        or not k_cache.is_contiguous()
        or not v_cache.is_contiguous()
        or slot_pos.shape != (s, n)
        or slot_pos.dtype != torch.int64
        or pos.shape != (s,)
        or pos.dtype != torch.int64
    ):
        raise ValueError("Expected same-device bf16 q and contiguous [S,H,N,D] bf16 caches, "
                         "int64 [S,N] slot positions and int64 [S] chunk positions")
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    if out is None:
        out = torch.empty((s, t, h, d), device=q.device, dtype=torch.bfloat16)
    elif out.shape != (s, t, h, d) or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError("out must be a contiguous bf16 [S, T, H, D] tensor")
    q = q.contiguous()
    slot_pos = slot_pos.contiguous()
    pos = pos.contiguous()
    with torch.cuda.device(q.device):
        _lib.call("moss_history_attention", q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                  slot_pos.data_ptr(), pos.data_ptr(), s, h, t, n, d, int(context), float(scale),
                  out.data_ptr(), _stream(q.device))
    return out


def history_attention_qkv(qkv, heads, pos, max_period, slots, k_cache, v_cache, slot_pos,
                          context, scale=None, out=None):
    """`rope_kv` followed by `history_attention` in one kernel.

    qkv: bf16 [S, T, 3 * heads * 64] (the qkv projection's output: q, k, v of
    every head); pos: int64 [S], the chunk's first position (the rotary
    offset and the queries' position); slots: int64 [S, T]; k_cache,
    v_cache, slot_pos, context, scale as for `history_attention`.  Rotates q
    and k as `rope_kv` does, writes the rotated keys and the values into the
    rings and returns the attention [S, T, heads, 64]: the same bits as the
    two calls.  Covers many (stream, head) items (at least twice the SM
    count), rings of at most 256 slots and at most 8 queries; other inputs
    raise UnsupportedError (call `rope_kv` and `history_attention` then)."""
    if qkv.ndim != 3 or k_cache.ndim != 4:
        raise ValueError("Expected qkv [S, T, 3*H*D] and caches [S, H, N, D]")
    s, t, width = qkv.shape
    h, n, d = k_cache.shape[1], k_cache.shape[2], k_cache.shape[3]
    if (
        qkv.dtype != torch.bfloat16
        or k_cache.dtype != torch.bfloat16
        or v_cache.dtype != torch.bfloat16
        or not qkv.is_cuda
        or any(x.device != qkv.device for x in (k_cache, v_cache, slot_pos, pos, slots))
        or h != heads
        or width != 3 * h * d
        or k_cache.shape[0] != s
        or v_cache.shape != k_cache.shape
        or not k_cache.is_contiguous()
        or not v_cache.is_contiguous()
        or slot_pos.shape != (s, n)
        or slot_pos.dtype != torch.int64
        or pos.shape != (s,)
        or pos.dtype != torch.int64
        or slots.shape != (s, t)
        or slots.dtype != torch.int64
    ):
        raise ValueError("Expected same-device bf16 qkv [S,T,3*H*D] and contiguous [S,H,N,D] bf16 "
                         "caches, int64 [S,N] slot positions, [S] positions and [S,T] slots")
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    if out is None:
        out = torch.empty((s, t, h, d), device=qkv.device, dtype=torch.bfloat16)
    elif out.shape != (s, t, h, d) or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError("out must be a contiguous bf16 [S, T, H, D] tensor")
    qkv = qkv.contiguous()
    slots = slots.contiguous()
    slot_pos = slot_pos.contiguous()
    pos = pos.contiguous()
    coef = -math.log(max_period) * 2 / d
    with torch.cuda.device(qkv.device):
        _lib.call("moss_history_attention_qkv", qkv.data_ptr(), slots.data_ptr(), coef,
                  k_cache.data_ptr(), v_cache.data_ptr(), slot_pos.data_ptr(), pos.data_ptr(),
                  s, h, t, n, d, int(context), float(scale), out.data_ptr(), _stream(qkv.device))
    return out


def pack_qkv_weight(weight):
    """Packs a bf16 qkv Linear weight [3*H*64, K] (K a multiple of 64) for
    `qkv_rope`: blocks of 32 rows x 64 columns in the tensor cores'
    no-swizzle K-major core-matrix order, block (row tile, column chunk) at
    [n // 32][k // 64], inside a block [row group][k core][row][element] of
    8 each (4 row groups).  Done once per weight, like the reference's
    cached bf16 Linear weight (fast_moss/v2_runtime.py:77-106)."""
    if weight.ndim != 2 or weight.shape[0] % 192 or weight.shape[1] % 64 or not weight.shape[1]:
        raise ValueError("Expected a [3*H*64, K] weight with K a multiple of 64")
    n, k = weight.shape
    w = weight.to(torch.bfloat16).contiguous()
    return w.view(n // 32, 4, 8, k // 64, 8, 8).permute(0, 3, 1, 4, 2, 5).contiguous()


def qkv_rope(x, w_image, bias, heads, offset, max_period, slots, k_cache, v_cache):
    """The qkv Linear with the rotary embedding and the history-ring writes
    in its epilogue (one tcgen05 kernel).

    x: bf16 [B, T, K] (the LayerNorm output); w_image: `pack_qkv_weight` of
    the [3*heads*64, K] weight; bias: bf16 [3*heads*64] or None; offset [B]
    and int64 slots [B, T] as in `rope_kv`; k_cache, v_cache: contiguous
    bf16 [B, heads, S, 64].  Returns the rotated q [B, heads, T, 64].  The
    same bits as F.linear followed by `rope_kv` whenever the projection's
    FP32 sums round to the same bf16 value (the summation order differs
    from cuBLAS's).
    """
    if x.ndim != 3 or x.dtype != torch.bfloat16 or not x.is_cuda:
        raise ValueError("Expected bf16 CUDA x [B, T, K]")
    b, t, k = x.shape
    n = 3 * heads * 64
    if (
        w_image.dtype != torch.bfloat16
        or w_image.numel() != n * k
        or not w_image.is_contiguous()
        or (bias is not None and (bias.dtype != torch.bfloat16 or bias.shape != (n,)))
        or offset.numel() != b
        or slots.shape != (b, t)
        or slots.dtype != torch.int64
        or k_cache.dtype != torch.bfloat16
        or k_cache.ndim != 4
        or k_cache.shape[:2] != (b, heads)
        or k_cache.shape[3] != 64
        or v_cache.shape != k_cache.shape
        or v_cache.dtype != torch.bfloat16
        or not k_cache.is_contiguous()
        or not v_cache.is_contiguous()
        or any(v.device != x.device for v in (w_image, offset, slots, k_cache, v_cache))
        or (bias is not None and bias.device != x.device)
    ):
        raise ValueError("Incompatible qkv_rope inputs")
    if offset.dtype == torch.int64:
        odt = 0
    elif offset.dtype == torch.int32:
        odt = 1
    else:
        odt = 2
        offset = offset.float()
    x = x.contiguous()
    offset = offset.contiguous()
    slots = slots.contiguous()
    bias = bias.contiguous() if bias is not None else None
    q = torch.empty((b, heads, t, 64), device=x.device, dtype=torch.bfloat16)
    if x.numel():
        with torch.cuda.device(x.device):
            _lib.call(
                "moss_qkv_rope", x.data_ptr(), w_image.data_ptr(),
                bias.data_ptr() if bias is not None else None, b, t, heads, k,
                offset.data_ptr(), odt, -math.log(max_period) * 2 / 64, slots.data_ptr(),
                q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[2],
                _stream(x.device))
    return q


def scale_add(x, update, scale):
    """Residual update x + update * scale (FP32 out, no FMA).

    Reference fast_moss/v2_pointwise.py:101-122.  Non-contiguous inputs are
    made contiguous first (the arithmetic is elementwise, so the result is
    the same as the reference's eager path for them).
    """
    if (
        x.shape != update.shape
        or scale.shape != (x.shape[-1],)
        or x.dtype not in _DTYPES
        or update.dtype not in _DTYPES
        or scale.dtype != torch.float32
        or not x.is_cuda
        or update.device != x.device
        or scale.device != x.device
    ):
        raise ValueError(
            "Expected equal BF16/FP32 residuals and same-device FP32 channel scale"
        )
    x, update, scale = x.contiguous(), update.contiguous(), scale.contiguous()
    out = torch.empty(x.shape, device=x.device, dtype=torch.float32)
    if x.numel():
        with torch.cuda.device(x.device):
            _lib.call(
                "moss_scale_add", x.data_ptr(), _DTYPES[x.dtype], update.data_ptr(),
                _DTYPES[update.dtype], scale.data_ptr(), out.data_ptr(), x.numel(),
                x.shape[-1], _stream(x.device))
    return out


def _check_norm_params(x, weight, bias):
    n = x.shape[-1]
    for p in (weight, bias):
        if p is not None and (
            p.shape != (n,) or p.dtype != torch.float32 or p.device != x.device
            or not p.is_contiguous()
        ):
            raise ValueError("Expected contiguous same-device FP32 LayerNorm parameters")


def _out_dtype(out_dtype):
    if out_dtype not in _DTYPES:
        raise ValueError("out_dtype must be torch.float32 or torch.bfloat16")
    return _DTYPES[out_dtype]


def layer_norm(x, weight, bias, eps=1e-5, *, return_stats=False, out_dtype=torch.float32):
    """FP32 LayerNorm over the last dim, bit-identical to torch's CUDA op.

    out_dtype=torch.bfloat16 stores the result rounded to bf16 (the bits of
    `layer_norm(...).to(torch.bfloat16)`, without a separate cast kernel).
    Raises _lib.UnsupportedError for widths PyTorch would not vectorise
    (n % 4 != 0) or misaligned buffers.
    """
    if x.dtype != torch.float32 or not x.is_cuda or x.ndim < 1:
        raise ValueError("Expected a CUDA FP32 tensor")
    _check_norm_params(x, weight, bias)
    x = x.contiguous()
    n = x.shape[-1]
    rows = x.numel() // n if n else 0
    odt = _out_dtype(out_dtype)
    y = torch.empty(x.shape, device=x.device, dtype=out_dtype)
    mean = torch.empty(rows, device=x.device, dtype=torch.float32) if return_stats else None
    rstd = torch.empty(rows, device=x.device, dtype=torch.float32) if return_stats else None
    if x.numel():
        with torch.cuda.device(x.device):
            _lib.call(
                "moss_residual_layer_norm_out", x.data_ptr(), _lib.F32, None, _lib.F32, None,
                weight.data_ptr() if weight is not None else None,
                bias.data_ptr() if bias is not None else None, float(eps), rows, n, None,
                y.data_ptr(), odt, mean.data_ptr() if mean is not None else None,
                rstd.data_ptr() if rstd is not None else None, _stream(x.device))
    return (y, mean, rstd) if return_stats else y


def residual_layer_norm(x, update, scale, weight, bias, eps=1e-5, *, write_residual=True,
                        return_stats=False, out_dtype=torch.float32):
    """Fused `r = scale_add(x, update, scale)` and `LayerNorm(r)` in one pass.

    Returns (r, normed) -- r is None when write_residual is False -- plus
    (mean, rstd) when return_stats.  Same bits as the reference's
    scale_add followed by torch's CUDA layer norm; out_dtype=torch.bfloat16
    stores normed rounded to bf16 (the next Linear's input cast).
    """
    if (
        x.shape != update.shape
        or scale.shape != (x.shape[-1],)
        or x.dtype not in _DTYPES
        or update.dtype not in _DTYPES
        or scale.dtype != torch.float32
        or not x.is_cuda
        or update.device != x.device
        or scale.device != x.device
    ):
        raise ValueError(
            "Expected equal BF16/FP32 residuals and same-device FP32 channel scale"
        )
    _check_norm_params(x, weight, bias)
    x, update, scale = x.contiguous(), update.contiguous(), scale.contiguous()
    n = x.shape[-1]
    rows = x.numel() // n if n else 0
    odt = _out_dtype(out_dtype)
    res = torch.empty(x.shape, device=x.device, dtype=torch.float32) if write_residual else None
    y = torch.empty(x.shape, device=x.device, dtype=out_dtype)
    mean = torch.empty(rows, device=x.device, dtype=torch.float32) if return_stats else None
    rstd = torch.empty(rows, device=x.device, dtype=torch.float32) if return_stats else None
    if x.numel():
        with torch.cuda.device(x.device):
            _lib.call(
                "moss_residual_layer_norm_out", x.data_ptr(), _DTYPES[x.dtype], update.data_ptr(),
                _DTYPES[update.dtype], scale.data_ptr(),
                weight.data_ptr() if weight is not None else None,
                bias.data_ptr() if bias is not None else None, float(eps), rows, n,
                res.data_ptr() if res is not None else None, y.data_ptr(), odt,
                mean.data_ptr() if mean is not None else None,
                rstd.data_ptr() if rstd is not None else None, _stream(x.device))
    if return_stats:
        return res, y, mean, rstd
    return res, y


_ACTS = {"silu": _lib.ACT_SILU, "gelu": _lib.ACT_GELU_ERF, "gelu_tanh": _lib.ACT_GELU_TANH}


def gated_activation(x, bias=None, activation="silu", gated=True):
    """Bias + activation (+ gate) with torch's per-op rounding.

    gated: act(x[..., :w] + b[:w]) * (x[..., w:] + b[w:]) with w = width/2;
    otherwise act(x + b).  x: BF16 or FP32 CUDA tensor, bias of x's dtype.
    """
    if activation not in _ACTS:
        raise ValueError(f"Unknown activation {activation!r}")
    if x.dtype not in _DTYPES or not x.is_cuda or x.ndim < 1:
        raise ValueError("Expected a CUDA BF16/FP32 tensor")
    width = x.shape[-1]
    if gated and width % 2:
        raise ValueError("Gated activation needs an even last dimension")
    if bias is not None and (
        bias.shape != (width,) or bias.dtype != x.dtype or bias.device != x.device
    ):
        raise ValueError("Expected a same-device bias of x's dtype and width")
    x = x.contiguous()
    bias = bias.contiguous() if bias is not None else None
    out_w = width // 2 if gated else width
    y = torch.empty(x.shape[:-1] + (out_w,), device=x.device, dtype=x.dtype)
    rows = x.numel() // width if width else 0
    if x.numel():
        with torch.cuda.device(x.device):
            _lib.call(
                "moss_gated_act", x.data_ptr(), bias.data_ptr() if bias is not None else None,
                y.data_ptr(), _DTYPES[x.dtype], rows, width, _ACTS[activation], 1 if gated else 0,
                _stream(x.device))
    return y
