"""GPU: the streaming transformer stack on the native kernels, replayed under
CUDA graphs by the batched scheduler, against the eager-PyTorch oracle of
the same stack (stock LayerNorm, eager residual, torch rotary tables and
rotation, eager activation; the same GEMM and attention calls).  The
hot-path kernels reproduce those torch ops bit for bit, so every output of
every chunk must be bit-identical -- including after the history ring
wraps and after a per-stream reset."""

import pytest
import torch

from oracle.stack import EagerStack

pytestmark = pytest.mark.gpu


def _features(streams, tokens, dim, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(streams, tokens, dim, generator=g)


def _run_oracle(ref, feats, chunk):
    outs = []
    for c in range(feats.shape[1] // chunk):
        outs.append(ref.step(feats[:, c * chunk:(c + 1) * chunk]))
    return torch.cat(outs, 1)


@pytest.mark.parametrize("gated,activation", [(False, "gelu"), (True, "silu")])
def test_small_stack_graph_replay_is_bit_identical(moss, cuda_device, gated, activation):
    from fast_moss_b200.transformer import (BatchedStreams, StackConfig, StreamingTransformer,
                                            init_weights)

    cfg = StackConfig(layers=3, dim=256, heads=4, ffn=512, context=10, chunk_tokens=4,
                      gated=gated, activation=activation)
    weights = init_weights(cfg, seed=5)
    stack = StreamingTransformer(cfg, weights, cuda_device)
    sched = BatchedStreams(stack, streams=3, chunks_per_graph=2)
    feats = _features(3, 4 * 8, cfg.dim, 11).to(cuda_device)  # 8 chunks: the ring wraps
    got = sched(feats)
    ref = EagerStack(cfg, weights, cuda_device, 3)
    want = _run_oracle(ref, feats, 4)
    assert torch.equal(got, want)
    # a second call starts every stream afresh
    assert torch.equal(sched(feats), want)
    sched.release()


def test_config_stack_streams_bit_identical(moss, cuda_device):
    """The codec's streaming stack at its configured size: 24 layers, hidden
    1280, 20 heads, feed-forward 5120, one stream of 80 ms chunks of 4
    tokens, one graph replay per chunk."""
    from fast_moss_b200.transformer import (BatchedStreams, StackConfig, StreamingTransformer,
                                            init_weights)

    cfg = StackConfig()
    weights = init_weights(cfg, seed=2)
    stack = StreamingTransformer(cfg, weights, cuda_device)
    sched = BatchedStreams(stack, streams=1, chunks_per_graph=1)
    feats = _features(1, 4 * 6, cfg.dim, 3).to(cuda_device)
    got = sched(feats)
    ref = EagerStack(cfg, weights, cuda_device, 1)
    want = _run_oracle(ref, feats, 4)
    assert torch.isfinite(got).all()
    assert torch.equal(got, want)
    sched.release()


def test_per_stream_reset_matches_a_fresh_stream(moss, cuda_device):
    from fast_moss_b200.transformer import (BatchedStreams, StackConfig, StreamingTransformer,
                                            init_weights)

    cfg = StackConfig(layers=2, dim=128, heads=2, ffn=256, context=8, chunk_tokens=4)
    weights = init_weights(cfg, seed=7)
    stack = StreamingTransformer(cfg, weights, cuda_device)
    sched = BatchedStreams(stack, streams=2, chunks_per_graph=1)
    feats = _features(2, 4 * 5, cfg.dim, 13).to(cuda_device)
    sched.reset()
    for c in range(3):
        sched.push(feats[:, 4 * c:4 * (c + 1)])
    sched.reset([1])  # stream 1 starts a new file, stream 0 carries on
    late = torch.cat([sched.push(feats[:, 4 * c:4 * (c + 1)]).clone() for c in (3, 4)], 1)
    fresh = EagerStack(cfg, weights, cuda_device, 2)
    want_fresh = _run_oracle(fresh, feats[:, 12:20], 4)
    cont = EagerStack(cfg, weights, cuda_device, 2)
    want_cont = _run_oracle(cont, feats, 4)[:, 12:20]
    assert torch.equal(late[1], want_fresh[1])
    assert torch.equal(late[0], want_cont[0])
    sched.release()


def test_eager_step_equals_graph_replay(moss, cuda_device):
    """StreamingTransformer.step outside a graph gives the replay's bits."""
    from fast_moss_b200.transformer import (BatchedStreams, StackConfig, StreamingTransformer,
                                            init_weights)

    cfg = StackConfig(layers=2, dim=256, heads=4, ffn=512, context=12, chunk_tokens=4)
    weights = init_weights(cfg, seed=9)
    stack = StreamingTransformer(cfg, weights, cuda_device)
    feats = _features(2, 12, cfg.dim, 17).to(cuda_device)
    hist = stack.history(2)
    eager = torch.cat([stack.step(feats[:, 4 * c:4 * (c + 1)], hist) for c in range(3)], 1)
    sched = BatchedStreams(stack, streams=2, chunks_per_graph=3)
    assert torch.equal(sched(feats), eager)
    sched.release()


def test_fused_qkv_stack(moss, cuda_device):
    """The stack with the fused qkv projection (tcgen05 GEMM + rotary
    epilogue + history writes in one kernel): its graph replays equal its
    own eager steps bit for bit, and it tracks the cuBLAS-projection stack
    to bf16 noise (the projection's sums are ordered differently)."""
    from fast_moss_b200.transformer import (BatchedStreams, StackConfig, StreamingTransformer,
                                            init_weights)

    cfg = StackConfig()
    weights = init_weights(cfg, seed=2)
    plain = StreamingTransformer(cfg, weights, cuda_device)
    fused = StreamingTransformer(cfg, weights, cuda_device, fused_qkv=True)
    feats = _features(2, 4 * 6, cfg.dim, 3).to(cuda_device)
    sp = BatchedStreams(plain, streams=2)
    sf = BatchedStreams(fused, streams=2)
    a, b = sp(feats), sf(feats)
    hist = fused.history(2)
    eager = torch.cat([fused.step(feats[:, c * 4:(c + 1) * 4], hist) for c in range(6)], 1)
    assert torch.equal(b, eager)
    rel = float((a - b).norm() / a.norm())
    assert rel < 2e-2, rel
    sp.release()
    sf.release()


def test_owned_linear_stack(moss, cuda_device):
    """The stack on the tcgen05 Linear (all four projections; the first
    feed-forward one with bias + GELU in its epilogue), with and without the
    history attention: graph replays equal the stack's own eager steps bit
    for bit, and it tracks the cuBLAS stack to bf16 noise (the projections'
    sums are ordered differently)."""
    from fast_moss_b200.transformer import (BatchedStreams, StackConfig, StreamingTransformer,
                                            init_weights)

    cfg = StackConfig()
    weights = init_weights(cfg, seed=2)
    plain = StreamingTransformer(cfg, weights, cuda_device)
    feats = _features(3, 4 * 6, cfg.dim, 5).to(cuda_device)
    sp = BatchedStreams(plain, streams=3)
    a = sp(feats)
    sp.release()
    for opts in ({"owned_linear": True}, {"owned_linear": True, "history_attention": True}):
        owned = StreamingTransformer(cfg, weights, cuda_device, **opts)
        so = BatchedStreams(owned, streams=3)
        b = so(feats)
        hist = owned.history(3)
        eager = torch.cat([owned.step(feats[:, c * 4:(c + 1) * 4], hist) for c in range(6)], 1)
        assert torch.equal(b, eager), opts
        rel = float((a - b).norm() / a.norm())
        assert rel < 2e-2, (opts, rel)
        so.release()


def test_batched_streams_run_host_matches_the_device_path(moss, cuda_device):
    """run_host (copies in and out overlapped with the replays) gives the
    same bits as pushing the same chunks from device memory."""
    from fast_moss_b200.transformer import BatchedStreams, StackConfig, StreamingTransformer
    from fast_moss_b200.transformer import init_weights

    cfg = StackConfig(layers=2)
    stack = StreamingTransformer(cfg, init_weights(cfg, seed=2), cuda_device,
                                 history_attention=True)
    sched = BatchedStreams(stack, streams=3)
    g = torch.Generator().manual_seed(9)
    feats = torch.randn(7, 3, cfg.chunk_tokens, cfg.dim, generator=g)
    host_in = feats.pin_memory()
    host_out = torch.empty_like(host_in).pin_memory()
    sched.run_host(host_in, host_out)
    torch.cuda.synchronize()
    sched.reset()
    want = torch.stack([sched.push(feats[c].to(cuda_device)).cpu() for c in range(7)])
    assert torch.equal(host_out, want)
    with pytest.raises(ValueError):
        sched.run_host(host_in[:, :2], host_out[:, :2])
    sched.release()
