"""WAV input/output and the command line's argument checks (CPU).

The conversions follow soundfile's float32 reading of integer WAV samples,
which the reference's command line uses (fast_moss/__main__.py:22); the
argument errors must come before any model is loaded (the reference's
order, fast_moss/__main__.py:19-28)."""

import numpy as np
import pytest
from scipy.io import wavfile

from fast_moss_b200 import wav


def test_float_wav_round_trip_keeps_bits(tmp_path):
    rng = np.random.default_rng(0)
    x = rng.standard_normal((4801, 2)).astype(np.float32)
    x[0, 0], x[1, 1], x[2, 0] = -0.0, np.float32(1e-42), np.float32(3.4e38)
    p = tmp_path / "a.wav"
    wav.write_wav(p, x, 48000)
    y, rate = wav.read_wav(p)
    assert rate == 48000 and y.dtype == np.float32 and y.shape == x.shape
    assert np.array_equal(y.view(np.uint32), x.view(np.uint32))


@pytest.mark.parametrize("dtype,scale", [(np.int16, 2.0 ** 15), (np.int32, 2.0 ** 31)])
def test_integer_wav_is_scaled_like_soundfile(tmp_path, dtype, scale):
    info = np.iinfo(dtype)
    x = np.array([[info.min, info.max], [0, 1], [-1, 12345]], dtype=dtype)
    p = tmp_path / "i.wav"
    wavfile.write(p, 44100, x)
    y, rate = wav.read_wav(p)
    assert rate == 44100
    assert np.array_equal(y, (x.astype(np.float64) / scale).astype(np.float32))
    assert y[0, 0] == -1.0


def test_unsigned_8bit_and_mono(tmp_path):
    x = np.array([0, 128, 255], dtype=np.uint8)
    p = tmp_path / "u8.wav"
    wavfile.write(p, 8000, x)
    y, _ = wav.read_wav(p)
    assert y.shape == (3, 1)
    assert np.array_equal(y[:, 0], np.array([-1.0, 0.0, 127 / 128], dtype=np.float32))


def test_24bit_pcm(tmp_path):
    # a hand-built 24-bit PCM file: two frames, stereo
    samples = [-(2 ** 23), 2 ** 23 - 1, 1, -2]
    data = b"".join(int(v).to_bytes(3, "little", signed=True) for v in samples)
    fmt = (1).to_bytes(2, "little") + (2).to_bytes(2, "little") + (48000).to_bytes(4, "little")
    fmt += (48000 * 6).to_bytes(4, "little") + (6).to_bytes(2, "little") + (24).to_bytes(2, "little")
    body = b"WAVE" + b"fmt " + len(fmt).to_bytes(4, "little") + fmt + b"data" + len(data).to_bytes(4, "little") + data
    p = tmp_path / "p24.wav"
    p.write_bytes(b"RIFF" + len(body).to_bytes(4, "little") + body)
    y, rate = wav.read_wav(p)
    assert rate == 48000 and y.shape == (2, 2)
    want = (np.array(samples, dtype=np.float64) / 2 ** 23).astype(np.float32).reshape(2, 2)
    assert np.array_equal(y, want)


def test_cli_rejects_bad_arguments_before_loading(tmp_path, monkeypatch):
    from fast_moss_b200 import __main__ as cli

    def no_model():
        raise AssertionError("the model must not be loaded for a rejected call")

    monkeypatch.setattr(cli, "load_model", no_model)
    good = tmp_path / "in.wav"
    wav.write_wav(good, np.zeros((10, 2), np.float32), 48000)
    mono = tmp_path / "mono.wav"
    wav.write_wav(mono, np.zeros((10, 1), np.float32), 48000)
    slow = tmp_path / "44k.wav"
    wav.write_wav(slow, np.zeros((10, 2), np.float32), 44100)
    empty = tmp_path / "empty.wav"
    wav.write_wav(empty, np.zeros((0, 2), np.float32), 48000)
    for argv in ([str(good), str(good)],
                 [str(good), str(tmp_path / "out.flac")],
                 [str(mono), str(tmp_path / "out.wav")],
                 [str(slow), str(tmp_path / "out.wav")],
                 [str(empty), str(tmp_path / "out.wav")]):
        with pytest.raises(SystemExit) as e:
            cli.main(argv)
        assert e.value.code == 2, argv
    assert not (tmp_path / "out.wav").exists()
