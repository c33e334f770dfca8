"""CPU: the streaming stack's host logic -- attention-history ring buffer,
per-stream reset, configuration checks -- against the oracle's explicit
loops and against plain windowed attention over the full key list."""

import pytest
import torch
import torch.nn.functional as F

from fast_moss_b200.transformer import StackConfig, StreamHistory, init_weights
from oracle.stack import EagerStack, windowed_attention_reference


def _cfg(**kw):
    base = dict(layers=1, dim=32, heads=2, ffn=64, context=6, chunk_tokens=4)
    base.update(kw)
    return StackConfig(**base)


@pytest.mark.parametrize("context", [4, 6, 9, 12])
def test_history_slots_and_mask_match_the_oracle_loops(context):
    cfg = _cfg(context=context)
    hist = StreamHistory(cfg, 3, "cpu")
    ref = EagerStack(cfg, init_weights(cfg), "cpu", 3)
    for chunk in range(7):
        if chunk == 3:
            hist.reset([1])
            ref.reset([1])
        if chunk == 5:
            hist.reset()
            ref.reset()
        _, slots, mask = hist.advance(cfg.chunk_tokens)
        rslots, rmask = ref._mask(cfg.chunk_tokens)
        assert torch.equal(slots, rslots)
        assert torch.equal(mask, rmask)
        assert torch.equal(hist.slot_pos, ref.slot_pos)
        hist.pos.add_(cfg.chunk_tokens)
        ref.pos += cfg.chunk_tokens


def test_ring_attention_equals_windowed_attention_over_all_keys():
    """SDPA over the ring with the history mask == attention over the full
    key sequence restricted to the window (FP32 on the CPU)."""
    torch.manual_seed(0)
    cfg = _cfg(context=10, chunk_tokens=4)
    hist = StreamHistory(cfg, 1, "cpu")
    keys = torch.zeros(1, 1, cfg.history_slots, 8)
    values = torch.zeros(1, 1, cfg.history_slots, 8)
    all_k, all_v = [], []
    for chunk in range(6):  # 24 tokens through a 13-slot ring (context 10)
        q = torch.randn(1, 1, 4, 8)
        k = torch.randn(1, 1, 4, 8)
        v = torch.randn(1, 1, 4, 8)
        positions, slots, mask = hist.advance(4)
        index = slots[:, None, :, None].expand(1, 1, 4, 8)
        keys.scatter_(2, index, k)
        values.scatter_(2, index, v)
        all_k.append(k)
        all_v.append(v)
        got = F.scaled_dot_product_attention(q, keys, values, attn_mask=mask)
        ks, vs = torch.cat(all_k, 2)[0, 0], torch.cat(all_v, 2)[0, 0]
        want = windowed_attention_reference(q[0, 0], ks, vs, positions[0],
                                            torch.arange(ks.shape[0]), cfg.context)
        torch.testing.assert_close(got[0, 0], want, rtol=1e-5, atol=1e-6)
        hist.pos.add_(4)


def test_stack_config_checks():
    with pytest.raises(ValueError):
        StackConfig(dim=30, heads=4)
    with pytest.raises(ValueError):
        StackConfig(context=3, chunk_tokens=4)
    with pytest.raises(ValueError):
        StackConfig(layers=0)
    cfg = StackConfig()
    assert (cfg.layers, cfg.dim, cfg.heads, cfg.ffn, cfg.head_dim) == (24, 1280, 20, 5120, 64)


def test_weights_are_seeded_and_shaped():
    cfg = _cfg(layers=2, gated=True)
    a, b = init_weights(cfg, seed=2), init_weights(cfg, seed=2)
    assert all(torch.equal(x[k], y[k]) for x, y in zip(a, b) for k in x)
    assert a[0]["qkv_w"].shape == (96, 32)
    assert a[0]["ffn1_w"].shape == (128, 32)  # gated: twice the feed-forward width
    assert a[0]["ffn2_w"].shape == (32, 64)
    assert not torch.equal(a[0]["qkv_w"], init_weights(cfg, seed=3)[0]["qkv_w"])
