"""Fixed-frame offline encode/decode adapters for native stereo v2.

Same contract as fast_moss/v2_codec.py:8-61: complete 3840-sample frames
only, valid code lengths known from the shape (no host sync), and the
upstream arithmetic unchanged around the optimized modules.
"""

import sys

import torch

FRAME = 3840


@torch.no_grad()
def encode_fixed(model, audio):
    """Graph-safe full-frame v2 encoding of complete equal-length stereo clips."""
    if (
        audio.ndim != 3
        or audio.shape[1] != 2
        or audio.shape[0] < 1
        or audio.shape[-1] < FRAME
        or audio.shape[-1] % FRAME
        or model.sampling_rate != 48000
        or model.number_channels != 2
        or model.attention_implementation != "sdpa"
    ):
        raise ValueError("Expected complete equal-length B,2,T 48 kHz stereo frames with SDPA")
    if any(getattr(m, "is_streaming", False) for m in model.modules()):
        raise RuntimeError("Fixed v2 graphs are offline; use StreamingCodec for stateful input")
    return _encode_complete(model, audio)


def _encode_complete(model, audio):
    """Native arithmetic for complete frames, including an active stream."""
    lengths = torch.full((audio.shape[0],), audio.shape[-1], device=audio.device,
                         dtype=torch.long)
    hidden, lengths = model._flatten_channels_for_codec(audio, lengths)
    with model._codec_inference_autocast():
        for module in model.encoder:
            hidden, lengths = module(hidden, lengths)
    _, codes, code_lengths = model.quantizer(hidden.float(), lengths, None)
    output_type = sys.modules[type(model).__module__].MossAudioTokenizerEncoderOutput
    return output_type(audio_codes=codes, audio_codes_lengths=code_lengths,
                       encoder_hidden_states=hidden.float())


def codec(model, audio):
    """Return owned-by-caller codes, hidden states and stereo reconstruction."""
    enc = encode_fixed(model, audio)
    return enc.audio_codes, enc.encoder_hidden_states, model._decode_frame(enc.audio_codes).audio
