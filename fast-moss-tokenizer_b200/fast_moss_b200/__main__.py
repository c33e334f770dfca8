"""Reconstruct a 48 kHz stereo WAV file with the B200 codec.

`python -m fast_moss_b200 input.wav output.wav` -- the command line of
fast_moss/__main__.py: the input is read and checked first (different
files, a .wav output, 48 kHz, two channels, at least one sample; any
failure is a usage error before the model is loaded), then coded by
`StreamingCodec` inside `optimized(model)`, and the reconstruction is
written as an FP32 WAV file.
"""

import argparse
from pathlib import Path

import torch

from .streaming import StreamingCodec
from .v2_loading import load_model
from .v2_runtime import optimized
from .wav import read_wav, write_wav

RATE = 48_000
CHANNELS = 2


def _usage_problem(src, dst):
    """Reads `src` and returns (samples [n, 2] float32, None), or (None,
    the reason the command cannot run)."""
    if src.resolve() == dst.resolve():
        return None, "the input and output must be different files"
    if dst.suffix.lower() != ".wav":
        return None, "the output must be a .wav file"
    samples, rate = read_wav(src)
    if rate != RATE or samples.shape[1] != CHANNELS:
        return None, f"the input must be {RATE} Hz audio with {CHANNELS} channels"
    if samples.shape[0] == 0:
        return None, "the input holds no samples"
    return samples, None


def reconstruct(samples, model):
    """Codes `samples` [n, 2] (float32, host) with the model on its device
    and returns the reconstruction [n, 2] float32 on the host."""
    device = next(model.parameters()).device
    waveform = torch.from_numpy(samples.T.copy())[None].to(device)
    with torch.inference_mode(), optimized(model), StreamingCodec(model) as session:
        _, _, decoded = session(waveform)
        return decoded[0].float().T.cpu().numpy()


def main(argv=None):
    parser = argparse.ArgumentParser(prog="python -m fast_moss_b200",
                                     description=__doc__.splitlines()[0])
    parser.add_argument("input", type=Path, help="48 kHz stereo WAV to code")
    parser.add_argument("output", type=Path, help="reconstruction, written as FP32 WAV")
    args = parser.parse_args(argv)
    samples, problem = _usage_problem(args.input, args.output)
    if problem is not None:
        parser.error(problem)
    decoded = reconstruct(samples, load_model())
    write_wav(args.output, decoded, RATE)
    print(f"Saved {args.output}: {RATE} Hz stereo, {len(decoded)} samples")


if __name__ == "__main__":
    main()
