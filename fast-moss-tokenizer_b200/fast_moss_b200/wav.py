"""WAV file input and output for the command-line codec.

The reference reads with soundfile (`sf.read(path, dtype="float32",
always_2d=True)`) and writes FP32 WAV (`subtype="FLOAT"`), in
fast_moss/__main__.py:22-35.  This module reads and writes the same data
through scipy's RIFF/WAVE reader, with soundfile's float conversion of
integer samples: unsigned 8-bit as (x - 128) / 128, signed 16/24/32-bit as
x / 2^(bits - 1) (scipy returns 24-bit samples left-justified in int32, so
they share the 32-bit scale); float samples are returned as float32.
"""

import numpy as np
from scipy.io import wavfile


def read_wav(path):
    """Returns (samples [frames, channels] float32, sample rate)."""
    rate, data = wavfile.read(path)
    if data.ndim == 1:
        data = data[:, None]
    if data.dtype == np.uint8:
        out = (data.astype(np.float32) - 128.0) / 128.0
    elif data.dtype == np.int16:
        out = data.astype(np.float32) / 32768.0
    elif data.dtype == np.int32:
        out = (data.astype(np.float64) / 2147483648.0).astype(np.float32)
    elif data.dtype == np.int64:
        out = (data.astype(np.float64) / 9223372036854775808.0).astype(np.float32)
    elif data.dtype in (np.float32, np.float64):
        out = data.astype(np.float32)
    else:
        raise ValueError(f"Unsupported WAV sample type {data.dtype}")
    return np.ascontiguousarray(out), int(rate)


def write_wav(path, samples, rate):
    """Writes [frames, channels] samples as IEEE float32 WAV."""
    samples = np.ascontiguousarray(np.asarray(samples, dtype=np.float32))
    if samples.ndim != 2:
        raise ValueError("Expected samples shaped [frames, channels]")
    wavfile.write(path, int(rate), samples)
