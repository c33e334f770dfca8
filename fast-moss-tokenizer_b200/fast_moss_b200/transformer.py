"""Streaming codec transformer stack on the B200 kernels, and the batched
streaming scheduler that replays it under CUDA graphs.

The layer is the one the reference patches (fast_moss/v2_runtime.py:231-276):
pre-LayerNorm attention with RoPE (:186-224) over a bounded causal history,
residual + layer scale, pre-LayerNorm feed-forward, residual + layer scale;
FP32 residual stream and parameters, bf16 GEMMs on cached bf16 weights
(:77-106, F.linear as in :104).  Per layer the hot-path ops run as the
native kernels of libfast_moss_b200:

  LayerNorm of the stack input              moss_residual_layer_norm_out
  rotary phase + rotation of q and k, the    moss_rope_kv
    rotated keys and the values written
    straight into the attention history
  residual + layer scale 1 + LayerNorm 2     moss_residual_layer_norm_out (one pass,
                                             normed output stored as the next
                                             GEMM's bf16 input)
  feed-forward bias + activation             moss_gated_act
  residual + layer scale 2 + next LN 1       moss_residual_layer_norm_out
                                             (moss_scale_add after the last layer)

With `owned_linear=True` the four Linears of a layer run as moss_linear
(tcgen05 bf16 GEMM with TMA-fed operands, K split across a thread-block
cluster and reduced in a fixed order) and the feed-forward's bias +
activation move into the first feed-forward Linear's epilogue; the sums run
in that kernel's order, not cuBLAS's.

With `fused_qkv=True` the qkv Linear, the rotary embedding and the history
writes are one tcgen05 kernel (moss_qkv_rope: bf16 tensor-core GEMM whose
epilogue rounds, rotates and stores into the ring; its dot products are
summed in its own order, not cuBLAS's) for chunks of at most
FUSED_QKV_MAX_ROWS token rows (all streams together), where it is faster;
larger chunks keep the cuBLAS GEMM + moss_rope_kv.  The other GEMMs (cuBLAS) and
attention (SDPA) stay library calls, as in the reference;
attention is pinned to SDPA's memory-efficient backend, which runs these
few-query, masked shapes about twice as fast as the backend chosen by
default on B200 (66 us against 121 us per layer at 64 streams).

The attention history of every layer is a ring of `context + chunk_tokens - 1`
token slots per stream ([streams, heads, slots, head_dim] bf16 keys and
values, plus the position held by each slot; position p lives in slot
p mod slots).  A query at position p attends to the keys at positions
p - context < p' <= p that have been written, which includes causal
attention inside the chunk; the extra chunk_tokens - 1 slots keep the keys
that the chunk's first queries still see while the chunk's own keys go in.  All state lives at fixed addresses and
is updated in place, so a chunk step can be captured once and replayed.
"""

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel

from .graphs import CapturedStep
from .linear import linear as owned_linear
from .linear import pack_weight
from .v2_pointwise import (
    gated_activation,
    history_attention,
    history_attention_qkv,
    layer_norm,
    pack_qkv_weight,
    qkv_rope,
    residual_layer_norm,
    rope_kv,
    scale_add,
)


_LINEAR_ACTS = ("silu", "gelu", "gelu_tanh")

# Token rows (streams x chunk tokens) up to which the fused qkv projection
# runs: one 32-row tile of moss_qkv_rope.  Measured per layer on B200 at
# the configured shape: 9.2 us fused against 16.5 us for the cuBLAS GEMM +
# moss_rope_kv at 4 rows; 70 us against 21 us at 256 rows.
FUSED_QKV_MAX_ROWS = 32


@dataclass(frozen=True)
class StackConfig:
    """Shape of a streaming transformer stack.

    The defaults are the codec's streaming stack: 24 layers, hidden 1280,
    20 heads, feed-forward 5120, 4 tokens per 80 ms chunk.  `context` is the
    attention history in tokens (250 tokens = 5 s of audio at 50 tokens/s).
    The feed-forward is Linear (no bias) -> act(h + bias) -> Linear (bias);
    `gated` makes the first Linear twice as wide and gates act(h[:, :ffn])
    with h[:, ffn:].
    """

    layers: int = 24
    dim: int = 1280
    heads: int = 20
    ffn: int = 5120
    context: int = 250
    chunk_tokens: int = 4
    max_period: float = 10000.0
    activation: str = "gelu"
    gated: bool = False
    eps: float = 1e-5

    def __post_init__(self):
        if self.dim % self.heads or (self.dim // self.heads) % 2:
            raise ValueError("dim must split into heads of even width")
        if self.context < self.chunk_tokens:
            raise ValueError("context must hold at least one chunk of tokens")
        if min(self.layers, self.ffn, self.chunk_tokens) < 1:
            raise ValueError("layers, ffn and chunk_tokens must be positive")

    @property
    def head_dim(self):
        return self.dim // self.heads

    @property
    def history_slots(self):
        return self.context + self.chunk_tokens - 1


WEIGHT_NAMES = ("norm1_w", "norm1_b", "qkv_w", "qkv_b", "out_w", "out_b", "ls1", "norm2_w",
                "norm2_b", "ffn1_w", "ffn1_b", "ffn2_w", "ffn2_b", "ls2")


def init_weights(cfg, seed=2, device="cpu"):
    """Seeded random FP32 weights: every matrix, bias and layer scale
    ~ 0.02 N(0, 1); LayerNorm weights 1 + 0.02 N(0, 1), biases 0.02 N(0, 1).
    Drawn in a fixed order by a generator on `device` (the CPU by default:
    those values do not depend on where they are later moved; a CUDA
    generator draws other values, much faster)."""
    device = torch.device(device)
    g = torch.Generator(device=device).manual_seed(seed)
    d, f = cfg.dim, cfg.ffn
    f1 = 2 * f if cfg.gated else f

    def n(*shape):
        return 0.02 * torch.randn(*shape, generator=g, device=device)

    layers = []
    for _ in range(cfg.layers):
        layers.append({
            "norm1_w": 1 + n(d), "norm1_b": n(d),
            "qkv_w": n(3 * d, d), "qkv_b": n(3 * d),
            "out_w": n(d, d), "out_b": n(d),
            "ls1": n(d),
            "norm2_w": 1 + n(d), "norm2_b": n(d),
            "ffn1_w": n(f1, d), "ffn1_b": n(f1),
            "ffn2_w": n(d, f), "ffn2_b": n(d),
            "ls2": n(d),
        })
    return layers


class StreamHistory:
    """Attention history of `streams` independent streams, updated in place.

    keys[i], values[i]: [streams, heads, slots, head_dim] bf16 of layer i;
    slot_pos: [streams, slots] int64, the position held by each slot
    (-1: empty); pos: [streams] int64, the position of the next token.
    """

    def __init__(self, cfg, streams, device):
        if streams < 1:
            raise ValueError("streams must be >= 1")
        shape = (streams, cfg.heads, cfg.history_slots, cfg.head_dim)
        self.streams = streams
        self.context = cfg.context
        self.max_tokens = cfg.chunk_tokens
        self.keys = [torch.zeros(shape, device=device, dtype=torch.bfloat16)
                     for _ in range(cfg.layers)]
        self.values = [torch.zeros(shape, device=device, dtype=torch.bfloat16)
                       for _ in range(cfg.layers)]
        self.slot_pos = torch.full((streams, cfg.history_slots), -1, device=device,
                                   dtype=torch.int64)
        self.pos = torch.zeros(streams, device=device, dtype=torch.int64)

    def reset(self, streams=None):
        """Starts the given streams (all by default) afresh, in place.  The
        old keys stay in memory but are masked out (their slots are empty)."""
        with torch.inference_mode():
            if streams is None:
                self.slot_pos.fill_(-1)
                self.pos.zero_()
            else:
                idx = torch.as_tensor(streams, device=self.pos.device, dtype=torch.int64)
                self.slot_pos.index_fill_(0, idx, -1)
                self.pos.index_fill_(0, idx, 0)

    def advance(self, tokens, *, mask=True):
        """Writes the slot positions of the next `tokens` tokens and returns
        (positions [S, T], slots [S, T], attention mask [S, 1, T, slots] or
        None when `mask` is false: the history attention kernel derives the
        mask from the slot positions itself)."""
        if not 1 <= tokens <= self.max_tokens:
            raise ValueError(f"a chunk holds 1 to {self.max_tokens} tokens")
        positions = self.pos[:, None] + torch.arange(tokens, device=self.pos.device)
        slots = torch.remainder(positions, self.slot_pos.shape[1])
        self.slot_pos.scatter_(1, slots, positions)
        if not mask:
            return positions, slots, None
        held = self.slot_pos[:, None, :]
        query = positions[:, :, None]
        mask = (held >= 0) & (held <= query) & (held > query - self.context)
        return positions, slots, mask[:, None]


def additive_mask(mask, dtype):
    """The boolean attention mask as the additive mask (0 where attended,
    -inf elsewhere) that SDPA builds from a boolean one, in a buffer whose
    key dimension is padded to a multiple of 16 (the memory-efficient
    kernel's alignment; the returned tensor is a view of the real keys).
    Built once per chunk, so the 24 layers' attention calls skip SDPA's
    own conversion and padding (four small kernels per layer)."""
    n = mask.shape[-1]
    padded = torch.zeros(mask.shape[:-1] + ((n + 15) // 16 * 16,), device=mask.device,
                         dtype=dtype)
    out = padded[..., :n]
    out.masked_fill_(~mask, float("-inf"))
    return out


class StreamingTransformer:
    """The stack: FP32 parameters on one CUDA device, bf16 GEMM weights cached
    once (the reference's cached Linear, fast_moss/v2_runtime.py:77-106)."""

    def __init__(self, cfg, weights, device, *, fused_qkv=False, history_attention=False,
                 owned_linear=False):
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("StreamingTransformer runs on a CUDA device")
        if len(weights) != cfg.layers:
            raise ValueError("one weight dict per layer expected")
        self.cfg = cfg
        self.device = device
        self.layers = []
        for w in weights:
            p = {k: w[k].to(device=device, dtype=torch.float32).contiguous() for k in WEIGHT_NAMES}
            for k in ("qkv_w", "qkv_b", "out_w", "out_b", "ffn1_w", "ffn1_b", "ffn2_w", "ffn2_b"):
                p[k + "16"] = p[k].to(torch.bfloat16)
            if fused_qkv:
                p["qkv_image"] = pack_qkv_weight(p["qkv_w16"])
            if owned_linear:
                for k in ("qkv_w", "out_w", "ffn1_w", "ffn2_w"):
                    p[k + "_packed"] = pack_weight(p[k + "16"])
            self.layers.append(p)
        self.fused_qkv = bool(fused_qkv)
        if self.fused_qkv and cfg.head_dim != 64:
            raise ValueError("the fused qkv projection needs heads of 64")
        # the four Linears as moss_linear (tcgen05, K split over a cluster)
        # with the feed-forward's bias + activation in the first one's
        # epilogue, instead of cuBLAS + moss_gated_act
        self.owned_linear = bool(owned_linear)
        if self.owned_linear and (cfg.gated or cfg.dim % 128 or cfg.ffn % 128
                                  or cfg.activation not in _LINEAR_ACTS):
            raise ValueError("the owned Linear needs widths that are multiples of 128 and an "
                             "ungated silu / gelu / gelu_tanh feed-forward")
        # the attention as moss_history_attention (FP32 softmax and P.V over
        # the ring, mask from the slot positions) instead of SDPA
        self.history_attention = bool(history_attention)
        if self.history_attention and (cfg.head_dim != 64 or cfg.chunk_tokens > 8
                                       or cfg.history_slots > 512):
            raise ValueError("the history attention kernel needs heads of 64, at most 8 "
                             "tokens per chunk and at most 512 history slots")
        # with many (stream, head) items the rotary and the ring update run
        # inside the attention kernel (moss_history_attention_qkv)
        self._fused_attention_items = 2 * torch.cuda.get_device_properties(
            device).multi_processor_count

    def history(self, streams):
        return StreamHistory(self.cfg, streams, self.device)

    def _attention_takes_qkv(self, streams):
        """True when the history attention also does the rotary and the ring
        update (moss_history_attention_qkv): its persistent kernel's range."""
        return (self.history_attention and streams * self.cfg.heads >= self._fused_attention_items
                and self.cfg.history_slots <= 256)

    def _linear(self, x, p, name):
        if self.owned_linear:
            return owned_linear(x, p[name + "_w_packed"], p[name + "_b16"])
        return F.linear(x, p[name + "_w16"], p[name + "_b16"])

    def native_launches(self, streams):
        """Kernels of libfast_moss_b200 that one chunk step launches: the
        first LayerNorm, then per layer the rotary (moss_rope_kv or
        moss_qkv_rope), the history attention when it replaces SDPA, the two
        residual + LayerNorm passes (the last layer's second is
        moss_scale_add) and the feed-forward activation."""
        per_layer = 4 + (1 if self.history_attention else 0)
        if self._attention_takes_qkv(streams) and not (
                self.fused_qkv and streams * self.cfg.chunk_tokens <= FUSED_QKV_MAX_ROWS):
            per_layer -= 1  # the rotary runs inside the attention kernel
        if self.owned_linear:
            per_layer += 3  # four Linears, the activation in the first feed-forward one
        return 1 + self.cfg.layers * per_layer

    @torch.inference_mode()
    def step(self, x, hist):
        """One chunk [streams, T, dim] FP32 through every layer; advances the
        history by T tokens and returns the FP32 residual stream."""
        cfg = self.cfg
        s, t, d = x.shape
        if d != cfg.dim or s != hist.streams or x.dtype != torch.float32 or x.device != self.device:
            raise ValueError("expected a [streams, tokens, dim] FP32 chunk on the stack's device")
        h, dh = cfg.heads, cfg.head_dim
        offset = hist.pos  # position of the chunk's first token (advanced at the end)
        _, slots, mask = hist.advance(t, mask=not self.history_attention)
        if not self.history_attention:
            mask = additive_mask(mask, torch.bfloat16)
        first = self.layers[0]
        x = x.contiguous()
        bf16 = torch.bfloat16
        # LayerNorm outputs go straight to the next GEMM as its bf16 input
        normed = layer_norm(x, first["norm1_w"], first["norm1_b"], cfg.eps, out_dtype=bf16)
        fused_qkv = self.fused_qkv and s * t <= FUSED_QKV_MAX_ROWS and not self.owned_linear
        fused_attention = self._attention_takes_qkv(s) and not fused_qkv
        for i, p in enumerate(self.layers):
            if fused_attention:
                # rotary, ring update and attention in one kernel
                qkv = self._linear(normed, p, "qkv")
                a = history_attention_qkv(qkv.view(s, t, 3 * d), h, offset, cfg.max_period, slots,
                                          hist.keys[i], hist.values[i], hist.slot_pos,
                                          cfg.context).view(s, t, d)
            else:
                if fused_qkv:
                    q = qkv_rope(normed, p["qkv_image"], p["qkv_b16"], h, offset, cfg.max_period,
                                 slots, hist.keys[i], hist.values[i])
                else:
                    qkv = self._linear(normed, p, "qkv")
                    qkv = qkv.view(s, t, 3, h, dh)
                    q = rope_kv(qkv[:, :, 0].transpose(1, 2), qkv[:, :, 1].transpose(1, 2),
                                qkv[:, :, 2].transpose(1, 2), offset, cfg.max_period, slots,
                                hist.keys[i], hist.values[i])
                if self.history_attention:
                    a = history_attention(q, hist.keys[i], hist.values[i], hist.slot_pos, offset,
                                          cfg.context).view(s, t, d)
                else:
                    with sdpa_kernel([SDPBackend.EFFICIENT_ATTENTION]):
                        a = F.scaled_dot_product_attention(q, hist.keys[i], hist.values[i],
                                                           attn_mask=mask)
                    a = a.transpose(1, 2).reshape(s, t, d)
            u = self._linear(a, p, "out")
            x, normed = residual_layer_norm(x, u, p["ls1"], p["norm2_w"], p["norm2_b"], cfg.eps,
                                            out_dtype=bf16)
            if self.owned_linear:
                f = owned_linear(normed, p["ffn1_w_packed"], p["ffn1_b16"],
                                 activation=cfg.activation)
            else:
                f = F.linear(normed, p["ffn1_w16"])
                f = gated_activation(f, p["ffn1_b16"], cfg.activation, cfg.gated)
            u = self._linear(f, p, "ffn2")
            if i + 1 < len(self.layers):
                nxt = self.layers[i + 1]
                x, normed = residual_layer_norm(x, u, p["ls2"], nxt["norm1_w"], nxt["norm1_b"],
                                                cfg.eps, out_dtype=bf16)
            else:
                x = scale_add(x, u, p["ls2"])
        hist.pos.add_(t)
        return x


class BatchedStreams:
    """Many streams of a StreamingTransformer advanced together under one
    CUDA graph (the scheduler that replaces fast_moss/streaming.py's one
    B=1 graph per 80 ms chunk).

    `streams` independent streams share every weight read; `chunks_per_graph`
    chunks are captured back to back in one graph, so a replay covers
    chunks_per_graph x 80 ms of every stream.  The step owns a static input
    [streams, span, dim] and a static output of the same shape: a caller
    either writes the next features into `input` (e.g. straight from pinned
    host memory) and calls `advance()`, or hands them to `push()`, which
    copies them in.  `__call__` copies every replay's output straight into
    one buffer allocated per call (no per-chunk clone, no concatenation).
    Use it on the CUDA stream and host thread that built it.
    """

    def __init__(self, stack, streams=1, chunks_per_graph=1):
        if chunks_per_graph < 1:
            raise ValueError("chunks_per_graph must be >= 1")
        self.stack = stack
        self.streams = int(streams)
        self.chunks_per_graph = int(chunks_per_graph)
        self.span = stack.cfg.chunk_tokens * self.chunks_per_graph
        self.history = stack.history(self.streams)
        t = stack.cfg.chunk_tokens
        m = self.chunks_per_graph
        features = torch.zeros(self.streams, self.span, stack.cfg.dim, device=stack.device)
        out = torch.empty_like(features)

        def run(x):
            for c in range(m):
                out[:, c * t:(c + 1) * t] = stack.step(x[:, c * t:(c + 1) * t], self.history)
            return (out,)

        self._step = CapturedStep(run, [features])
        self.history.reset()  # warm-up and capture advanced the history

    @property
    def input(self):
        """The static input [streams, span, dim] FP32 read by the next replay."""
        return self._step.inputs[0]

    @property
    def output(self):
        """The static output [streams, span, dim] FP32 of the last replay."""
        return self._step.outputs[0]

    def reset(self, streams=None):
        """Starts the given streams (all by default) afresh before the next replay."""
        self.history.reset(streams)

    def advance(self):
        """Advances every stream by one replay on the features already in
        `input`; returns `output` (valid until the next replay)."""
        return self._step.replay()[0]

    def push(self, features):
        """Copies features [streams, span, dim] FP32 (on the device) into
        `input` and advances; returns the static output."""
        if features.shape != self.input.shape or features.dtype != torch.float32:
            raise ValueError(f"expected FP32 features {tuple(self.input.shape)}")
        self.input.copy_(features)
        return self.advance()

    @torch.inference_mode()
    def __call__(self, features, *, reset=True):
        """Runs [streams, tokens, dim] features through the stack chunk by
        chunk (zero-padded to whole replays) and returns [streams, tokens, dim]."""
        if features.ndim != 3 or features.shape[0] != self.streams or \
                features.shape[2] != self.stack.cfg.dim:
            raise ValueError("expected [streams, tokens, dim] features")
        if reset:
            self.reset()
        n = features.shape[1]
        pad = (-n) % self.span
        if pad:
            features = F.pad(features, (0, 0, 0, pad))
        out = torch.empty_like(features)
        for g in range(features.shape[1] // self.span):
            sl = slice(g * self.span, (g + 1) * self.span)
            out[:, sl].copy_(self.push(features[:, sl]))
        return out[:, :n]

    @torch.inference_mode()
    def run_host(self, host_in, host_out, *, reset=True, depth=2):
        """Advances every stream through chunks held in pinned host memory.

        host_in, host_out: chunk-major pinned host tensors [chunks, streams,
        span, dim] FP32 (each chunk's block contiguous).  Chunk c's features
        are copied to the device on one copy stream and chunk c's output back
        on another while the neighbouring chunks replay (`depth` staging
        buffers each way); the replay stream only moves them between the
        staging buffers and the graph's static buffers (device to device).
        On return the current stream waits for the last copy out
        (synchronize before reading host_out)."""
        shape = (self.streams, self.span, self.stack.cfg.dim)
        if host_in.ndim != 4 or tuple(host_in.shape[1:]) != shape or host_in.is_cuda or \
                host_in.dtype != torch.float32:
            raise ValueError(f"host_in must be FP32 host features [chunks, {shape[0]}, "
                             f"{shape[1]}, {shape[2]}]")
        if host_out.shape != host_in.shape or host_out.is_cuda or host_out.dtype != torch.float32:
            raise ValueError("host_out must be an FP32 host tensor shaped like host_in")
        if depth < 1:
            raise ValueError("depth must be >= 1")
        dev = self.stack.device
        main = torch.cuda.current_stream(dev)
        h2d = torch.cuda.Stream(device=dev)
        d2h = torch.cuda.Stream(device=dev)
        stage_in = [torch.empty(shape, device=dev) for _ in range(depth)]
        stage_out = [torch.empty(shape, device=dev) for _ in range(depth)]
        # the staging buffers are used on the copy streams too: the caching
        # allocator must not hand their memory out again before those uses
        # end, and the copy streams start after the work already queued
        for buf in stage_in:
            buf.record_stream(h2d)
        for buf in stage_out:
            buf.record_stream(d2h)
        h2d.wait_stream(main)
        d2h.wait_stream(main)
        in_free = [None] * depth   # main has copied stage_in[b] into the graph input
        out_free = [None] * depth  # d2h has copied stage_out[b] to the host
        if reset:
            self.reset()
        for c in range(host_in.shape[0]):
            b = c % depth
            if in_free[b] is not None:
                h2d.wait_event(in_free[b])
            with torch.cuda.stream(h2d):
                stage_in[b].copy_(host_in[c], non_blocking=True)
                loaded = torch.cuda.Event()
                loaded.record(h2d)
            main.wait_event(loaded)
            self.input.copy_(stage_in[b])
            in_free[b] = torch.cuda.Event()
            in_free[b].record(main)
            out = self.advance()
            if out_free[b] is not None:
                main.wait_event(out_free[b])
            stage_out[b].copy_(out)
            done = torch.cuda.Event()
            done.record(main)
            d2h.wait_event(done)
            with torch.cuda.stream(d2h):
                host_out[c].copy_(stage_out[b], non_blocking=True)
                out_free[b] = torch.cuda.Event()
                out_free[b].record(d2h)
        main.wait_stream(d2h)
        main.wait_stream(h2d)

    def release(self):
        """Drops the captured graph and its static buffers."""
        self._step.release()
