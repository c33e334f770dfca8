"""GPU: the streaming scheduler (`StreamingCodec`) and the offline adapters
(`encode_fixed`, `codec`) on a stand-in model.

The upstream model is remote code that is not available here, so this test
builds a small stand-in with the interface those adapters drive
(fast_moss/v2_codec.py:36-61, fast_moss/streaming.py:14-133): the channel
flattening, the bf16 inference autocast, an encoder whose attention module
keeps a bounded history in a native streaming state (reset in place, and an
upstream-style `_update_streaming_cache` that rebinds new tensors), a
quantizer of LFQ stages, `_decode_frame`, `streaming(batch_size)` and
`_stop_streaming`.  Inside `optimized(model)`, graph replays of 80 ms
chunks must give the bits of the same chunks run eagerly one by one."""

import contextlib
import math
import threading

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

FRAME = 3840
CH = 16


class MossAudioTokenizerEncoderOutput:
    def __init__(self, audio_codes, audio_codes_lengths, encoder_hidden_states):
        self.audio_codes = audio_codes
        self.audio_codes_lengths = audio_codes_lengths
        self.encoder_hidden_states = encoder_hidden_states


class DecoderOutput:
    def __init__(self, audio):
        self.audio = audio


class StreamState:
    """Attention history of one module: fixed-size window, reset in place."""

    def __init__(self, batch, channels, context, device):
        self.cached_keys = torch.zeros(batch, channels, context, device=device)
        self.cached_values = torch.zeros(batch, channels, context, device=device)
        self.cached_positions = torch.full((batch, context), -1, device=device, dtype=torch.long)
        self.exec_mask = torch.ones(batch, device=device, dtype=torch.bool)
        self.offset = torch.zeros(batch, device=device, dtype=torch.long)

    def reset(self, exec_mask):
        self.cached_keys.zero_()
        self.cached_values.zero_()
        self.cached_positions.fill_(-1)
        self.offset.zero_()


class StandInAttention(nn.Module):
    """Single-head attention over a bounded history of frames."""

    def __init__(self, channels, context):
        super().__init__()
        self.context = context
        self.qkv = nn.Linear(channels, 3 * channels)
        self._streaming_state = None
        self.is_streaming = False

    def _update_streaming_cache(self, state, keys, values, positions, k_new, v_new, p_new):
        # the upstream form: new tensors for the window (the scheduler keeps
        # the addresses stable around this)
        state.cached_keys = torch.cat([keys, k_new], -1)[..., -self.context:]
        state.cached_values = torch.cat([values, v_new], -1)[..., -self.context:]
        state.cached_positions = torch.cat([positions, p_new], -1)[..., -self.context:]

    def forward(self, x, lengths):
        b, c, t = x.shape
        st = self._streaming_state
        if st is None:  # offline: a fresh history for this call
            st = StreamState(b, c, self.context, x.device)
        q, k, v = self.qkv(x.transpose(1, 2)).float().transpose(1, 2).chunk(3, dim=1)
        pos = st.offset[:, None] + torch.arange(t, device=x.device)
        keys = torch.cat([st.cached_keys, k], -1)
        values = torch.cat([st.cached_values, v], -1)
        held = torch.cat([st.cached_positions, pos], -1)
        allowed = (held[:, None, :] >= 0) & (held[:, None, :] <= pos[:, :, None]) & \
                  (held[:, None, :] > pos[:, :, None] - self.context)
        scores = torch.einsum("bct,bcs->bts", q, keys) / math.sqrt(c)
        attn = torch.softmax(scores.masked_fill(~allowed, float("-inf")), -1)
        out = x.float() + torch.einsum("bts,bcs->bct", attn, values)
        self._update_streaming_cache(st, st.cached_keys, st.cached_values, st.cached_positions,
                                     k, v, pos)
        st.offset.add_(t)
        return out, lengths


class FrameEmbed(nn.Module):
    def __init__(self):
        super().__init__()
        self.proj = nn.Linear(2 * FRAME, CH)

    def forward(self, audio, lengths):
        b, _, n = audio.shape
        frames = audio.view(b, 2, n // FRAME, FRAME).permute(0, 2, 1, 3).reshape(b, n // FRAME, -1)
        return self.proj(frames).transpose(1, 2), lengths // FRAME


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


class StandInQuantizer(nn.Module):
    def __init__(self, stages=3, k=64):
        super().__init__()
        self.proj_in = nn.ModuleList(nn.Linear(CH, 8) for _ in range(stages))
        self.proj_out = nn.ModuleList(nn.Linear(8, CH) for _ in range(stages))
        self.lfq = nn.ModuleList(MossAudioTokenizerLFQ(k) for _ in range(stages))

    def forward(self, hidden, lengths, n_q):
        residual = hidden
        codes = []
        for pin, pout, lfq in zip(self.proj_in, self.proj_out, self.lfq):
            z = pin(residual.transpose(1, 2)).transpose(1, 2).contiguous()
            values, idx = lfq.decode_latents(z)
            residual = residual - pout(values.transpose(1, 2)).transpose(1, 2)
            codes.append(idx)
        return None, torch.stack(codes), lengths


class MossAudioTokenizerModel(nn.Module):
    def __init__(self, revision):
        super().__init__()
        self.config = type("Config", (), {"_commit_hash": revision})()
        self.sampling_rate, self.number_channels, self.downsample_rate = 48000, 2, FRAME
        self.enable_channel_interleave = True
        self.attention_implementation = "sdpa"
        self.encoder = nn.ModuleList([FrameEmbed(), StandInAttention(CH, context=3)])
        self.quantizer = StandInQuantizer()
        self.decoder = nn.Linear(CH, 2 * FRAME)

    def _flatten_channels_for_codec(self, audio, lengths):
        return audio, lengths

    def _codec_inference_autocast(self):
        return torch.autocast("cuda", dtype=torch.bfloat16)

    def _decode_frame(self, codes):
        emb = sum(lfq.codebook(c) for lfq, c in zip(self.quantizer.lfq, codes))  # [B, T, 8]
        emb = F.pad(emb, (0, CH - 8))
        out = self.decoder(emb.float())  # [B, T, 2 * FRAME]
        b, t, _ = out.shape
        audio = out.view(b, t, 2, FRAME).permute(0, 2, 1, 3).reshape(b, 2, t * FRAME)
        return DecoderOutput(audio)

    @contextlib.contextmanager
    def streaming(self, batch_size):
        for m in self.modules():
            if isinstance(m, StandInAttention):
                m._streaming_state = StreamState(batch_size, CH, m.context,
                                                 next(self.parameters()).device)
                m.is_streaming = True
        try:
            yield
        finally:
            self._stop_streaming()

    def _stop_streaming(self):
        for m in self.modules():
            if isinstance(m, StandInAttention):
                m._streaming_state = None
                m.is_streaming = False


@pytest.fixture()
def model(moss, cuda_device):
    from fast_moss_b200.v2_loading import REVISION

    torch.manual_seed(0)
    m = MossAudioTokenizerModel(REVISION).to(cuda_device).eval()
    m.requires_grad_(False)
    return m


def _audio(cuda_device, samples, seed=1, batch=1):
    g = torch.Generator().manual_seed(seed)
    return (0.5 * torch.randn(batch, 2, samples, generator=g)).to(cuda_device)


@torch.inference_mode()
def _eager_stream(model, audio):
    from fast_moss_b200.v2_codec import _encode_complete

    length = audio.shape[-1]
    audio = F.pad(audio, (0, (-length) % FRAME))
    parts = []
    with model.streaming(batch_size=1):
        for chunk in audio.split(FRAME, dim=-1):
            enc = _encode_complete(model, chunk)
            parts.append((enc.audio_codes, enc.encoder_hidden_states,
                          model._decode_frame(enc.audio_codes).audio))
    codes, hidden, rec = (torch.cat(p, -1) for p in zip(*parts))
    return codes, hidden, rec[..., :length]


@pytest.mark.parametrize("chunks_per_graph", [1, 3])
def test_streaming_codec_replays_match_eager_chunks(moss, model, cuda_device, chunks_per_graph):
    from fast_moss_b200.streaming import StreamingCodec
    from fast_moss_b200.v2_runtime import optimized

    audio = _audio(cuda_device, 7 * FRAME + 1234)  # 8 chunks, the last one padded
    with optimized(model):
        want = _eager_stream(model, audio)
        with StreamingCodec(model, chunks_per_graph=chunks_per_graph) as sc:
            got = sc(audio)
            again = sc(audio)  # every call starts a fresh file
            short = sc(audio[..., :FRAME])
    assert got[0].shape == want[0].shape == (3, 1, 8)
    assert got[2].shape == audio.shape
    for g, w in zip(got, want):
        assert torch.equal(g, w)
    for g, w in zip(again, want):
        assert torch.equal(g, w)
    # a one-chunk file: its codes are the first chunk's codes of the longer file
    assert torch.equal(short[0], want[0][..., :1])
    # the history really carries across chunks: the second chunk differs
    # from encoding it as the first chunk of a file
    solo = _eager_stream(model, audio[..., FRAME:2 * FRAME].contiguous())
    assert not torch.equal(solo[1], want[1][..., 1:2])


def test_streaming_codec_ownership_and_errors(moss, model, cuda_device):
    from fast_moss_b200.streaming import StreamingCodec

    sc = StreamingCodec(model)
    with pytest.raises(RuntimeError):
        sc(_audio(cuda_device, FRAME))  # not entered
    with sc:
        with pytest.raises(ValueError):
            sc(_audio(cuda_device, FRAME, batch=2))
        with pytest.raises(ValueError):
            sc(_audio(cuda_device, FRAME).double())
        errors = []

        def other_thread():
            try:
                sc(_audio(cuda_device, FRAME))
            except RuntimeError as e:
                errors.append(e)

        th = threading.Thread(target=other_thread)
        th.start()
        th.join()
        assert errors, "a call from another thread must be refused"
        with pytest.raises(RuntimeError):
            StreamingCodec(model).__enter__()  # a second live session
    with pytest.raises(RuntimeError):
        sc.__enter__()  # not re-enterable
    assert not any(getattr(m, "is_streaming", False) for m in model.modules())
    assert all("_update_streaming_cache" not in m.__dict__ for m in model.modules())


def test_encode_fixed_and_codec(moss, model, cuda_device):
    from fast_moss_b200.v2_codec import _encode_complete, codec, encode_fixed
    from fast_moss_b200.v2_runtime import optimized

    audio = _audio(cuda_device, 4 * FRAME, batch=2)
    with optimized(model), torch.inference_mode():
        enc = encode_fixed(model, audio)
        ref = _encode_complete(model, audio)
        assert torch.equal(enc.audio_codes, ref.audio_codes)
        assert torch.equal(enc.encoder_hidden_states, ref.encoder_hidden_states)
        codes, hidden, rec = codec(model, audio)
        assert torch.equal(codes, ref.audio_codes)
        assert torch.equal(rec, model._decode_frame(ref.audio_codes).audio)
        assert rec.shape == audio.shape
        with pytest.raises(ValueError):
            encode_fixed(model, audio[..., :FRAME + 5])
        with model.streaming(batch_size=1):
            with pytest.raises(RuntimeError):
                encode_fixed(model, audio[:1])


def test_command_line_reconstructs_a_wav(moss, model, cuda_device, tmp_path, monkeypatch):
    """`python -m fast_moss_b200 in.wav out.wav` (fast_moss/__main__.py:13-36)
    on the stand-in model: the FP32 output file holds the bits of the
    streaming codec's reconstruction of the file's samples."""
    import numpy as np

    from fast_moss_b200 import __main__ as cli
    from fast_moss_b200 import wav
    from fast_moss_b200.streaming import StreamingCodec
    from fast_moss_b200.v2_runtime import optimized

    monkeypatch.setattr(cli, "load_model", lambda: model)
    audio = _audio(cuda_device, 2 * FRAME + 777, seed=5)
    src, dst = tmp_path / "in.wav", tmp_path / "out.wav"
    wav.write_wav(src, audio[0].T.cpu().numpy(), 48000)
    cli.main([str(src), str(dst)])
    got, rate = wav.read_wav(dst)
    assert rate == 48000 and got.shape == (audio.shape[-1], 2)
    with torch.inference_mode(), optimized(model), StreamingCodec(model) as sc:
        want = sc(audio)[2][0].float().cpu().T.numpy()
    assert np.array_equal(got.view(np.uint32), np.ascontiguousarray(want).view(np.uint32))
