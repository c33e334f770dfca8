"""GPU: the drop-in patch layer (`optimized`) on a stand-in model.

The upstream model classes are remote code that is not available here, so
this test builds stand-ins with the same class names and attributes the
runtime patches (transformer layer, rotary embedding, LFQ decode), whose
forward methods state the eager computation of the upstream modules.  Under
`optimized(model)` the patched methods must return the same bits, and on
exit every original method must be back."""

import math

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


class MossAudioTokenizerLayerScale(nn.Module):
    def __init__(self, dim):
        super().__init__()
        self.scale = nn.Parameter(0.01 * torch.randn(dim))
        self.channel_last = True

    def forward(self, x):
        return self.scale * x


class MossAudioTokenizerTransformerLayer(nn.Module):
    def __init__(self, dim):
        super().__init__()
        self.norm1 = nn.LayerNorm(dim)
        self.norm2 = nn.LayerNorm(dim)
        with torch.no_grad():
            for n in (self.norm1, self.norm2):
                n.weight.copy_(1 + 0.1 * torch.randn(dim))
                n.bias.copy_(0.1 * torch.randn(dim))
        self.self_attn = nn.Linear(dim, dim)
        self.ffn = nn.Linear(dim, dim)
        self.layer_scale_1 = MossAudioTokenizerLayerScale(dim)
        self.layer_scale_2 = MossAudioTokenizerLayerScale(dim)

    def forward(self, x, **kwargs):
        x = x + self.layer_scale_1(self.self_attn(self.norm1(x)))
        return x + self.layer_scale_2(self.ffn(self.norm2(x)))


class MossAudioTokenizerRotaryEmbedding(nn.Module):
    def __init__(self, max_period=10000.0):
        super().__init__()
        self.max_period = max_period

    def forward(self, q, k, offset, time_before_heads=False):
        b, h, t, d = q.shape
        ds = torch.arange(d // 2, device=q.device, dtype=torch.float32)
        freq = torch.exp(ds * (-math.log(self.max_period) * 2 / d))
        ts = offset.float().view(-1, 1) + torch.arange(t, device=q.device, dtype=torch.float32)
        phase = freq * ts.view(b, t, 1)
        c, s = torch.cos(phase).view(b, 1, t, d // 2), torch.sin(phase).view(b, 1, t, d // 2)

        def rot(x):
            xr, xi = x.float()[..., 0::2], x.float()[..., 1::2]
            out = torch.stack([xr * c - xi * s, xr * s + xi * c], dim=-1)
            return out.reshape(b, h, t, d).to(x.dtype)

        return rot(q), rot(k)


class MossAudioTokenizerLFQ(nn.Module):
    def __init__(self, k):
        super().__init__()
        self.codebook = nn.Embedding(k, 8)

    def decode_latents(self, x):
        b, _, t = x.shape
        enc = F.normalize(x.transpose(1, 2).reshape(-1, 8).float())
        book = F.normalize(self.codebook.weight.float())
        dist = (enc.pow(2).sum(1, keepdim=True) - (2 * enc) @ book.T) + book.pow(2).sum(1)[None]
        idx = dist.argmin(1)
        values = self.codebook.weight[idx].view(b, t, 8)
        return values.transpose(1, 2), idx.view(b, t)


class MossAudioTokenizerModel(nn.Module):
    def __init__(self, revision, dim=256, k=1024):
        super().__init__()
        self.config = type("Config", (), {"_commit_hash": revision})()
        self.sampling_rate, self.number_channels, self.downsample_rate = 48000, 2, 3840
        self.enable_channel_interleave = True
        self.attention_implementation = "sdpa"
        self.layer = MossAudioTokenizerTransformerLayer(dim)
        self.rope = MossAudioTokenizerRotaryEmbedding()
        self.lfq = MossAudioTokenizerLFQ(k)


@pytest.fixture()
def model(moss, cuda_device):
    from fast_moss_b200.v2_loading import REVISION

    torch.manual_seed(0)
    m = MossAudioTokenizerModel(REVISION).to(cuda_device).eval()
    m.requires_grad_(False)
    return m


def test_optimized_patches_are_bit_identical_and_restored(moss, model, cuda_device):
    torch.manual_seed(1)
    x = torch.randn(3, 37, 256, device=cuda_device)
    q = torch.randn(2, 4, 50, 64, device=cuda_device).to(torch.bfloat16)
    k = torch.randn(2, 4, 50, 64, device=cuda_device).to(torch.bfloat16)
    offset = torch.tensor([0, 9], device=cuda_device)
    lat = torch.randn(2, 8, 33, device=cuda_device)
    with torch.inference_mode():
        want_x = model.layer(x)
        want_q, want_k = model.rope(q, k, offset)
        want_v, want_i = model.lfq.decode_latents(lat)
        with moss.optimized(model, cache_linear=False) as rt:
            assert rt.residual_modules == 1 and rt.rope_modules == 1 and rt.quantizer_modules == 1
            got_x = model.layer(x)
            got_q, got_k = model.rope(q, k, offset)
            got_v, got_i = model.lfq.decode_latents(lat)
            assert rt.fused_norm_calls == 1 and rt.rope_calls == 1 and rt.select_calls == 1
    assert torch.equal(got_x, want_x)
    assert torch.equal(got_q.view(torch.int16), want_q.view(torch.int16))
    assert torch.equal(got_k.view(torch.int16), want_k.view(torch.int16))
    assert torch.equal(got_i, want_i)
    assert torch.equal(got_v, want_v)
    for mod, name in ((model.layer, "forward"), (model.rope, "forward"),
                      (model.lfq, "decode_latents")):
        assert name not in mod.__dict__  # the class method is back


def test_optimized_falls_back_where_the_reference_does(moss, model, cuda_device):
    q = torch.randn(2, 4, 50, 64, device=cuda_device)
    k = torch.randn(2, 4, 50, 64, device=cuda_device)
    offset = torch.tensor([0, 9], device=cuda_device)
    with torch.inference_mode(), moss.optimized(model, cache_linear=False) as rt:
        model.rope(q, k, offset, time_before_heads=True)  # not covered: upstream path
        assert rt.rope_calls == 0
    with pytest.raises(RuntimeError):
        with moss.optimized(model) as rt:
            with moss.optimized(model):
                pass


def test_graph_captured_in_context_stops_replaying_after_it(moss, model, cuda_device):
    """A graph captured inside optimized(model) holds the context's cached
    resources; once the context closes the graph refuses to replay, while
    a graph captured outside any context keeps working."""
    q = torch.randn(2, 4, 16, 64, device=cuda_device).to(torch.bfloat16)
    offset = torch.tensor([0, 3], device=cuda_device)

    def rotary(x):
        return model.rope(x, x, offset)

    with moss.optimized(model, cache_linear=False) as rt:
        inside = moss.GraphedCallable(rotary, q)
        first = inside(q)
        assert rt.rope_calls >= 1
    with pytest.raises(RuntimeError, match="released or rebuilt"):
        inside(q)
    outside = moss.GraphedCallable(rotary, q)  # the upstream path, no context
    again = outside(q)
    assert torch.equal(again[0].view(torch.int16), first[0].view(torch.int16))
    outside.release()
