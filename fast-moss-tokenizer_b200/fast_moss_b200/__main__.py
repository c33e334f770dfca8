"""Reconstruct a 48 kHz stereo WAV file with the B200 codec.

Same command line, checks and output as fast_moss/__main__.py:13-36:
`python -m fast_moss_b200 input.wav output.wav` reads the input, encodes and
decodes it through `StreamingCodec` inside `optimized(model)` and writes the
reconstruction as FP32 WAV.  The argument errors (same file, output not .wav,
not 48 kHz stereo, empty input) are reported before the model is loaded.
"""

import argparse
from pathlib import Path

import torch

from .streaming import StreamingCodec
from .v2_loading import load_model
from .v2_runtime import optimized
from .wav import read_wav, write_wav


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("input", type=Path, help="Input 48 kHz stereo WAV")
    parser.add_argument("output", type=Path, help="Output WAV, saved as FP32")
    args = parser.parse_args(argv)

    if args.input.resolve() == args.output.resolve():
        parser.error("Input and output must be different files")
    if args.output.suffix.lower() != ".wav":
        parser.error("Output must have a .wav extension")
    audio, sample_rate = read_wav(args.input)
    if sample_rate != 48_000 or audio.shape[1] != 2:
        parser.error("Input must be 48 kHz stereo (two channels)")
    if not len(audio):
        parser.error("Input audio is empty")

    model = load_model()
    waveform = torch.from_numpy(audio.T.copy()).unsqueeze(0).cuda()
    with torch.inference_mode(), optimized(model), StreamingCodec(model) as codec:
        _, _, reconstructed = codec(waveform)
        output = reconstructed[0].float().cpu().T.numpy()

    write_wav(args.output, output, sample_rate)
    print(f"Saved {args.output}: {sample_rate} Hz stereo, {len(output)} samples")


if __name__ == "__main__":
    main()
