"""GPU: attention of a chunk's queries over a streaming history ring.

Bars: within one bf16 unit (2^-8 relative) plus 1e-6 absolute of the same
attention evaluated in float64 from the bf16 inputs (the kernel computes in
FP32 and rounds once; the absolute term covers outputs that cancel to near
zero, where FP32 sums of ~250 terms differ from float64 by ~1e-8); the mask
is the streaming history's (slot positions in (pos + t - context, pos + t]);
the stack with the kernel in place of SDPA is bit-identical between its
graph replays and its eager steps and tracks the SDPA stack to bf16 noise.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ring(streams, heads, slots, tokens, context, seed, device):
    """A history ring after each stream has seen pos[s] + tokens positions
    (position p in slot p % slots), with random keys, values and queries."""
    g = torch.Generator().manual_seed(seed)
    pos = torch.tensor([(37 * s * s + 11 * s) % (3 * slots) for s in range(streams)])
    slot_pos = torch.full((streams, slots), -1, dtype=torch.int64)
    for s in range(streams):
        last = int(pos[s]) + tokens - 1
        for p in range(max(0, last - slots + 1), last + 1):
            slot_pos[s, p % slots] = p
    q = torch.randn(streams, heads, tokens, 64, generator=g)
    k = torch.randn(streams, heads, slots, 64, generator=g)
    v = torch.randn(streams, heads, slots, 64, generator=g)
    to = dict(device=device)
    return (q.to(**to, dtype=torch.bfloat16), k.to(**to, dtype=torch.bfloat16),
            v.to(**to, dtype=torch.bfloat16), slot_pos.to(**to), pos.to(**to))


def _close(out, ref):
    """|out - ref| <= 2^-8 |ref| + 1e-6 everywhere (NaN where ref is NaN)."""
    out = out.double().cpu()
    ref = ref.cpu()
    nan = torch.isnan(ref)
    assert torch.equal(torch.isnan(out), nan)
    err = (out - ref).abs()[~nan]
    bound = (2.0 ** -8 * ref.abs() + 1e-6)[~nan]
    assert bool((err <= bound).all()), float((err / bound).max())


def _reference(q, k, v, slot_pos, pos, context, scale):
    """float64 attention with the history mask, [S, T, H, 64]."""
    t = q.shape[2]
    qp = pos[:, None] + torch.arange(t, device=q.device)             # [S, T]
    held = slot_pos[:, None, :]                                        # [S, 1, N]
    on = (held >= 0) & (held <= qp[:, :, None]) & (held > qp[:, :, None] - context)
    sc = torch.einsum("shtd,shnd->shtn", q.double(), k.double()) * scale
    sc = sc.masked_fill(~on[:, None], float("-inf"))
    w = torch.softmax(sc, dim=-1)
    out = torch.einsum("shtn,shnd->shtd", w, v.double())
    return out.transpose(1, 2).contiguous()


@pytest.mark.parametrize("streams,heads,tokens,slots,context", [
    (1, 20, 4, 253, 250),    # the codec's stack, one stream
    (3, 4, 1, 16, 9),
    (2, 3, 8, 512, 500),
    (5, 2, 3, 257, 100),     # keys beyond the first 256 threads
    (64, 20, 4, 253, 250),   # 64 batched streams
    # the persistent kernel (at least two items per resident CTA), its tensor-
    # core scores over one or two 128-key tiles, 1 to 8 queries
    (16, 20, 1, 253, 250), (40, 8, 2, 100, 60), (20, 16, 3, 200, 150),
    (16, 20, 8, 256, 250),
])
def test_history_attention_matches_float64(moss, cuda_device, streams, heads, tokens, slots,
                                           context):
    q, k, v, slot_pos, pos = _ring(streams, heads, slots, tokens, context, 7, cuda_device)
    out = moss.history_attention(q, k, v, slot_pos, pos, context)
    ref = _reference(q, k, v, slot_pos, pos, context, 1 / 8)
    assert out.shape == (streams, tokens, heads, 64) and out.dtype == torch.bfloat16
    _close(out, ref)


def test_history_attention_agrees_with_sdpa(moss, cuda_device):
    """Against the library call it replaces (SDPA, memory-efficient
    backend, additive mask): SDPA rounds the weights to bf16 before P.V, so
    the two agree to a few bf16 units, not bit for bit."""
    from torch.nn.attention import SDPBackend, sdpa_kernel

    q, k, v, slot_pos, pos = _ring(4, 20, 253, 4, 250, 3, cuda_device)
    out = moss.history_attention(q, k, v, slot_pos, pos, 250)
    qp = pos[:, None] + torch.arange(4, device=cuda_device)
    held = slot_pos[:, None, :]
    on = (held >= 0) & (held <= qp[:, :, None]) & (held > qp[:, :, None] - 250)
    with sdpa_kernel([SDPBackend.EFFICIENT_ATTENTION]):
        ref = torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=on[:, None])
    diff = (out.float() - ref.transpose(1, 2).float()).abs().max().item()
    assert diff < 2e-2, diff


def test_history_attention_masks_and_empty_rows(moss, cuda_device):
    q, k, v, slot_pos, pos = _ring(2, 2, 16, 2, 5, 1, cuda_device)
    # stream 1: nothing in its history yet -> NaN (as SDPA with an all-false mask)
    slot_pos[1] = -1
    out = moss.history_attention(q, k, v, slot_pos, pos, 5)
    assert torch.isnan(out[1].float()).all()
    _close(out[:1], _reference(q[:1], k[:1], v[:1], slot_pos[:1], pos[:1], 5, 1 / 8))
    # an explicit scale and a caller-owned output buffer
    buf = torch.empty(1, 2, 2, 64, device=cuda_device, dtype=torch.bfloat16)
    got = moss.history_attention(q[:1], k[:1], v[:1], slot_pos[:1], pos[:1], 5, scale=0.3, out=buf)
    assert got.data_ptr() == buf.data_ptr()
    _close(buf, _reference(q[:1], k[:1], v[:1], slot_pos[:1], pos[:1], 5, 0.3))


def test_history_attention_rejects_unsupported_shapes(moss, cuda_device):
    from fast_moss_b200._lib import UnsupportedError

    q, k, v, slot_pos, pos = _ring(1, 2, 16, 2, 5, 1, cuda_device)
    with pytest.raises(ValueError):
        moss.history_attention(q.float(), k, v, slot_pos, pos, 5)
    with pytest.raises(ValueError):
        moss.history_attention(q, k, v, slot_pos.int(), pos, 5)
    q9 = torch.zeros(1, 2, 9, 64, device=cuda_device, dtype=torch.bfloat16)
    with pytest.raises(UnsupportedError):
        moss.history_attention(q9, k, v, slot_pos, pos, 5)
    k513 = torch.zeros(1, 2, 513, 64, device=cuda_device, dtype=torch.bfloat16)
    sp513 = torch.full((1, 513), -1, device=cuda_device, dtype=torch.int64)
    with pytest.raises(UnsupportedError):
        moss.history_attention(q, k513, k513, sp513, pos, 5)
    q32 = torch.zeros(1, 2, 2, 32, device=cuda_device, dtype=torch.bfloat16)
    k32 = torch.zeros(1, 2, 16, 32, device=cuda_device, dtype=torch.bfloat16)
    with pytest.raises(UnsupportedError):
        moss.history_attention(q32, k32, k32, slot_pos, pos, 5)


@pytest.mark.parametrize("fused_qkv", [False, True])
def test_stack_with_history_attention(moss, cuda_device, fused_qkv):
    from fast_moss_b200.transformer import (BatchedStreams, StackConfig, StreamingTransformer,
                                            init_weights)

    cfg = StackConfig()
    weights = init_weights(cfg, seed=2)
    plain = StreamingTransformer(cfg, weights, cuda_device)
    owned = StreamingTransformer(cfg, weights, cuda_device, fused_qkv=fused_qkv,
                                 history_attention=True)
    g = torch.Generator().manual_seed(3)
    feats = torch.randn(2, 4 * 6, cfg.dim, generator=g).to(cuda_device)
    sp = BatchedStreams(plain, streams=2)
    so = BatchedStreams(owned, streams=2)
    a, b = sp(feats), so(feats)
    hist = owned.history(2)
    eager = torch.cat([owned.step(feats[:, c * 4:(c + 1) * 4], hist) for c in range(6)], 1)
    assert torch.equal(b, eager)
    rel = float((a - b).norm() / a.norm())
    assert rel < 2e-2, rel
    sp.release()
    so.release()


@pytest.mark.parametrize("streams,heads,tokens,slots,context", [
    (64, 20, 4, 253, 250),   # the 64-stream stack
    (16, 20, 1, 253, 250), (40, 8, 2, 100, 60), (16, 20, 8, 256, 250),
])
def test_history_attention_qkv_matches_rope_kv_then_attention(moss, cuda_device, streams, heads,
                                                              tokens, slots, context):
    """The fused entry (rotary + ring update + attention) against moss_rope_kv
    followed by moss_history_attention on the same inputs: the same bits in
    the output and in both rings."""
    _, k, v, slot_pos, pos = _ring(streams, heads, slots, tokens, context, 11, cuda_device)
    g = torch.Generator().manual_seed(12)
    qkv = torch.randn(streams, tokens, 3 * heads * 64, generator=g).to(cuda_device, torch.bfloat16)
    slot_of = torch.remainder(pos[:, None] + torch.arange(tokens, device=cuda_device), slots)
    k1, v1 = k.clone(), v.clone()
    view = qkv.view(streams, tokens, 3, heads, 64)
    q = moss.rope_kv(view[:, :, 0].transpose(1, 2), view[:, :, 1].transpose(1, 2),
                     view[:, :, 2].transpose(1, 2), pos, 10000.0, slot_of, k1, v1)
    want = moss.history_attention(q, k1, v1, slot_pos, pos, context)
    k2, v2 = k.clone(), v.clone()
    got = moss.history_attention_qkv(qkv, heads, pos, 10000.0, slot_of, k2, v2, slot_pos, context)
    torch.cuda.synchronize()
    assert torch.equal(k2.view(torch.int16), k1.view(torch.int16))
    assert torch.equal(v2.view(torch.int16), v1.view(torch.int16))
    assert torch.equal(torch.isnan(got), torch.isnan(want))
    ok = ~torch.isnan(want)
    assert torch.equal(got[ok].view(torch.int16), want[ok].view(torch.int16))
    from fast_moss_b200 import _lib
    _lib.check(_lib.load().moss_check_device_error(None), "device error word")


def test_history_attention_qkv_rejects_the_per_item_range(moss, cuda_device):
    from fast_moss_b200._lib import UnsupportedError

    _, k, v, slot_pos, pos = _ring(2, 4, 16, 2, 9, 5, cuda_device)
    qkv = torch.zeros(2, 2, 3 * 4 * 64, device=cuda_device, dtype=torch.bfloat16)
    slot_of = torch.zeros(2, 2, device=cuda_device, dtype=torch.int64)
    with pytest.raises(UnsupportedError):  # too few (stream, head) items
        moss.history_attention_qkv(qkv, 4, pos, 10000.0, slot_of, k, v, slot_pos, 9)


def test_stack_fused_attention_equals_the_two_kernels(moss, cuda_device):
    """64 streams (the headline's batch): the stack whose attention also
    rotates and writes the ring gives the same bits as the stack that calls
    moss_rope_kv and moss_history_attention, under graph replay."""
    from fast_moss_b200.transformer import (BatchedStreams, StackConfig, StreamingTransformer,
                                            init_weights)

    cfg = StackConfig()
    weights = init_weights(cfg, seed=2)
    fused = StreamingTransformer(cfg, weights, cuda_device, history_attention=True)
    split = StreamingTransformer(cfg, weights, cuda_device, history_attention=True)
    split._fused_attention_items = 1 << 30  # never fused
    assert fused._attention_takes_qkv(64) and not split._attention_takes_qkv(64)
    g = torch.Generator().manual_seed(8)
    feats = torch.randn(64, 4 * 3, cfg.dim, generator=g).to(cuda_device)
    sf = BatchedStreams(fused, streams=64)
    ss = BatchedStreams(split, streams=64)
    assert torch.equal(sf(feats), ss(feats))
    sf.release()
    ss.release()
