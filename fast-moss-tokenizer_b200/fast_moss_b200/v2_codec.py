"""Offline (whole-clip) encode and decode of native 48 kHz stereo clips.

Drop-in for fast_moss/v2_codec.py: `encode_fixed(model, audio)` and
`codec(model, audio)`, plus the complete-frame encoder step
`_encode_complete` that StreamingCodec captures and replays.  A batch is
admitted only as whole 80 ms frames (3840 samples) of stereo audio, so
every code length follows from the tensor shape and nothing waits on the
device.  The upstream model's own modules do the arithmetic; inside
`optimized(model)` their patched methods run the B200 kernels.
"""

import importlib
from dataclasses import dataclass

import torch

FRAME = 3840  # samples per codec frame: 80 ms at 48 kHz


@dataclass(frozen=True)
class ClipSpec:
    """The clips the fixed-frame adapters accept: `channels`-channel audio
    at `rate` Hz in whole frames of `frame` samples, on a model built for
    that rate and channel count with SDPA attention."""

    rate: int = 48000
    channels: int = 2
    frame: int = FRAME

    def refusal(self, model, audio):
        """Why `audio` [B, C, T] cannot be encoded as fixed frames, or None."""
        if audio.ndim != 3 or audio.shape[0] < 1 or audio.shape[1] != self.channels:
            return f"expected a B,{self.channels},T batch of clips, got {tuple(audio.shape)}"
        samples = audio.shape[-1]
        if samples < self.frame or samples % self.frame:
            return (f"clips must hold whole {self.frame}-sample frames, got {samples} samples "
                    f"per channel")
        if model.sampling_rate != self.rate or model.number_channels != self.channels:
            return f"the model is not a {self.rate} Hz {self.channels}-channel codec"
        if model.attention_implementation != "sdpa":
            return "the fixed-frame path is validated with SDPA attention only"
        return None


STEREO_48K = ClipSpec()


def _encoder_output_type(model):
    """The upstream module's encoder-output record class."""
    return importlib.import_module(type(model).__module__).MossAudioTokenizerEncoderOutput


def _encode_complete(model, audio):
    """Encoder and quantizer over complete frames of `audio` [B, 2, T]
    (also valid inside a live stream, which StreamingCodec relies on).
    Every clip has the full length, so the lengths are a constant tensor."""
    full = torch.full((audio.shape[0],), audio.shape[-1], device=audio.device, dtype=torch.long)
    hidden, lengths = model._flatten_channels_for_codec(audio, full)
    with model._codec_inference_autocast():
        for block in model.encoder:
            hidden, lengths = block(hidden, lengths)
    hidden = hidden.float()  # the quantizer runs in FP32 (its autocast is off)
    _, codes, code_lengths = model.quantizer(hidden, lengths, None)
    return _encoder_output_type(model)(audio_codes=codes, audio_codes_lengths=code_lengths,
                                       encoder_hidden_states=hidden)


@torch.no_grad()
def encode_fixed(model, audio):
    """Encodes a batch of equal-length stereo clips of whole frames; safe
    to capture in a CUDA graph (no host synchronisation)."""
    reason = STEREO_48K.refusal(model, audio)
    if reason is not None:
        raise ValueError(reason)
    if any(getattr(m, "is_streaming", False) for m in model.modules()):
        raise RuntimeError("a streaming session is active on this model; fixed-frame encoding is "
                           "offline only (use StreamingCodec for stateful input)")
    return _encode_complete(model, audio)


def codec(model, audio):
    """(codes, encoder hidden states, reconstruction) of `audio`, all owned
    by the caller."""
    encoded = encode_fixed(model, audio)
    decoded = model._decode_frame(encoded.audio_codes)
    return encoded.audio_codes, encoded.encoder_hidden_states, decoded.audio
