"""mt_write_wav_f32: the reference's float32 WAV layout (main.swift:134-144), checked byte for byte
against a header packed here from the RIFF/WAVE format."""
from __future__ import annotations

import struct

import numpy as np
import pytest


def expected_wav(samples: np.ndarray, rate: int) -> bytes:
    data = samples.astype("<f4").tobytes()
    return (b"RIFF" + struct.pack("<I", 36 + len(data)) + b"WAVE" + b"fmt " +
            struct.pack("<IHHIIHH", 16, 3, 1, rate, rate * 4, 4, 32) + b"data" + struct.pack("<I", len(data)) + data)


@pytest.mark.parametrize("n,rate", [(0, 44100), (1, 44100), (4851, 44100), (1000, 16000)])
def test_wav_bytes(mt, tmp_path, n, rate):
    x = np.random.default_rng(n).standard_normal(n).astype(np.float32)
    path = tmp_path / "out.wav"
    mt.write_wav(path, x, sample_rate=rate)
    assert path.read_bytes() == expected_wav(x, rate)


def test_wav_default_rate_is_the_models(mt, tmp_path):
    mt.write_wav(tmp_path / "a.wav", np.zeros(3, np.float32))
    assert struct.unpack("<I", (tmp_path / "a.wav").read_bytes()[24:28])[0] == 44100 == mt.SAMPLE_RATE


def test_wav_unwritable_path(mt, tmp_path):
    with pytest.raises(mt.MingError) as e:
        mt.write_wav(tmp_path / "no" / "such" / "dir.wav", np.zeros(4, np.float32))
    assert e.value.status == mt.MT_ERR_ARG
