"""Eager-PyTorch oracle of the streaming transformer stack -- TEST INFRASTRUCTURE.

Restates, with stock torch ops only, the layer the reference patches
(fast_moss/v2_runtime.py:231-276) in the form the reference computes it:

  * LayerNorm: torch.nn.functional.layer_norm (the stock nn.LayerNorm the
    reference keeps, v2_runtime.py:259);
  * residual: float(x) + float(u) * s, product and sum rounded separately
    (the reference's eager formula beside _scale_add, v2_pointwise.py:116);
  * rotary: freq = exp(arange(d/2) * (-ln(period) * 2 / d)),
    phase = freq * (offset + t), torch cos/sin tables (v2_runtime.py:209-222)
    and the interleaved-pair rotation in FP32 with the result cast to q's
    dtype (v2_pointwise.py:8-47);
  * feed-forward bias + activation: the eager bf16 chain act(h + b);
  * GEMMs (F.linear on the cached bf16 weights, v2_runtime.py:104) and SDPA
    attention (memory-efficient backend) are the same library calls as the
    product path.

It keeps its own history tensors, so the product stack and this oracle can
be stepped side by side on the same chunks.  Only tests, the smoke check and
the benchmark's CPU baseline use it; the product package never imports it.
"""

import math

import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel


def rotary_tables(offset, t, d, period):
    """cos, sin [B, T, d/2] FP32 (fast_moss/v2_runtime.py:209-222)."""
    ds = torch.arange(d // 2, device=offset.device, dtype=torch.float32)
    freq = torch.exp(ds * (-math.log(period) * 2 / d))
    ts = offset.float().view(-1, 1) + torch.arange(t, device=offset.device, dtype=torch.float32)
    phase = freq * ts.view(-1, t, 1)
    return torch.cos(phase), torch.sin(phase)


def rotate(x, cos, sin):
    """Interleaved-pair rotation in FP32, cast to x's dtype, contiguous
    [B, H, T, D] (fast_moss/v2_pointwise.py:8-47)."""
    b, h, t, d = x.shape
    c, s = cos.view(b, 1, t, d // 2), sin.view(b, 1, t, d // 2)
    xr, xi = x.float()[..., 0::2], x.float()[..., 1::2]
    out = torch.stack([xr * c - xi * s, xr * s + xi * c], dim=-1)
    return out.reshape(b, h, t, d).to(x.dtype)


_ACTS = {
    "silu": F.silu,
    "gelu": F.gelu,
    "gelu_tanh": lambda v: F.gelu(v, approximate="tanh"),
}


class EagerStack:
    """The stack of `cfg` (fast_moss_b200.transformer.StackConfig) with stock
    torch ops on `device`, for `streams` streams."""

    def __init__(self, cfg, weights, device, streams):
        self.cfg = cfg
        self.device = torch.device(device)
        self.layers = []
        for w in weights:
            p = {k: v.to(self.device, torch.float32) for k, v in w.items()}
            for k in ("qkv_w", "qkv_b", "out_w", "out_b", "ffn1_w", "ffn1_b", "ffn2_w", "ffn2_b"):
                p[k + "16"] = p[k].to(torch.bfloat16)
            self.layers.append(p)
        shape = (streams, cfg.heads, cfg.history_slots, cfg.head_dim)
        self.keys = [torch.zeros(shape, device=self.device, dtype=torch.bfloat16)
                     for _ in range(cfg.layers)]
        self.values = [torch.zeros(shape, device=self.device, dtype=torch.bfloat16)
                       for _ in range(cfg.layers)]
        self.slot_pos = torch.full((streams, cfg.history_slots), -1, device=self.device,
                                   dtype=torch.int64)
        self.pos = torch.zeros(streams, device=self.device, dtype=torch.int64)

    def reset(self, streams=None):
        if streams is None:
            self.slot_pos.fill_(-1)
            self.pos.zero_()
        else:
            for s in streams:
                self.slot_pos[s] = -1
                self.pos[s] = 0

    def _mask(self, t):
        """Ring-buffer bookkeeping written out as loops over the tokens: the
        slot of position p is p mod (context + chunk_tokens - 1); a query at
        p sees the written positions p' with p - context < p' <= p."""
        c = self.cfg.context
        n = self.cfg.history_slots
        streams = self.pos.shape[0]
        slots = torch.empty(streams, t, dtype=torch.int64)
        mask = torch.zeros(streams, 1, t, n, dtype=torch.bool)
        slot_pos = self.slot_pos.cpu().clone()
        pos = self.pos.cpu()
        for s in range(streams):
            for i in range(t):
                p = int(pos[s]) + i
                slots[s, i] = p % n
                slot_pos[s, p % n] = p
        for s in range(streams):
            for i in range(t):
                p = int(pos[s]) + i
                for j in range(n):
                    q = int(slot_pos[s, j])
                    mask[s, 0, i, j] = q >= 0 and p - c < q <= p
        self.slot_pos.copy_(slot_pos)
        return slots.to(self.device), mask.to(self.device)

    @torch.inference_mode()
    def step(self, x):
        cfg = self.cfg
        s, t, d = x.shape
        h, dh = cfg.heads, cfg.head_dim
        act = _ACTS[cfg.activation]
        slots, mask = self._mask(t)
        cos, sin = rotary_tables(self.pos, t, dh, cfg.max_period)
        index = slots[:, None, :, None].expand(s, h, t, dh)
        x = x.float()
        for i, p in enumerate(self.layers):
            normed = F.layer_norm(x, (d,), p["norm1_w"], p["norm1_b"], cfg.eps)
            qkv = F.linear(normed.to(torch.bfloat16), p["qkv_w16"], p["qkv_b16"])
            qkv = qkv.view(s, t, 3, h, dh)
            q = rotate(qkv[:, :, 0].transpose(1, 2), cos, sin)
            k = rotate(qkv[:, :, 1].transpose(1, 2), cos, sin)
            self.keys[i].scatter_(2, index, k)
            self.values[i].scatter_(2, index, qkv[:, :, 2].transpose(1, 2))
            with sdpa_kernel([SDPBackend.EFFICIENT_ATTENTION, SDPBackend.MATH]):
                a = F.scaled_dot_product_attention(q, self.keys[i], self.values[i],
                                                   attn_mask=mask)
            u = F.linear(a.transpose(1, 2).reshape(s, t, d), p["out_w16"], p["out_b16"])
            x = x + u.float() * p["ls1"]
            normed = F.layer_norm(x, (d,), p["norm2_w"], p["norm2_b"], cfg.eps)
            f = F.linear(normed.to(torch.bfloat16), p["ffn1_w16"]) + p["ffn1_b16"]
            if cfg.gated:
                w = f.shape[-1] // 2
                f = act(f[..., :w]) * f[..., w:]
            else:
                f = act(f)
            u = F.linear(f, p["ffn2_w16"], p["ffn2_b16"])
            x = x + u.float() * p["ls2"]
        self.pos += t
        return x


def windowed_attention_reference(q, k, v, positions_q, positions_k, context):
    """Plain attention over an explicit key list (FP32 math): query at
    position p sees keys at p - context < p' <= p.  Used to check the ring
    buffer bookkeeping on the CPU."""
    scores = (q.float() @ k.float().transpose(-1, -2)) / math.sqrt(q.shape[-1])
    pq = positions_q.view(-1, 1)
    pk = positions_k.view(1, -1)
    allowed = (pk <= pq) & (pk > pq - context)
    scores = scores.masked_fill(~allowed, float("-inf"))
    return torch.softmax(scores, dim=-1) @ v.float()
