"""The batch reader / writer stages (host only, no GPU) against the reference host's conversions.

``vocalarc_b200_read_track`` is the reader stage of
``vocalarc_b200_separate_files``: wav_read, to_stereo and resample_linear of
the reference host (native/vocalarc_separation.c:1152-1222).  The oracle
restates them in numpy and is pinned to the reference executable itself: the
STFT of its conversion of a PCM16 mono 22.05 kHz WAV equals the executable's
own "source" dump (tests/golden/wav_pcm16_mono_22k.npz).
"""

import math
import os

import numpy as np
import pytest

from karaoke_platform_sidecar_native_b200 import fixtures, native
from oracle import vocalarc_oracle as O
from tests.conftest import GOLDEN


def snr_db(ref, test):
    ref = np.asarray(ref, dtype=np.float64)
    err = ref - np.asarray(test, dtype=np.float64)
    return 10 * math.log10((ref ** 2).sum() / max((err ** 2).sum(), 1e-300))


def test_oracle_input_conversion_matches_reference_dump():
    g = np.load(os.path.join(GOLDEN, "wav_pcm16_mono_22k.npz"))
    audio = O.read_track(g["wav"].tobytes())
    assert audio.shape == (2, g["vocals"].shape[1])
    assert snr_db(g["source"], O.stft(audio)) > 120


CASES = [
    # (channels, rate, bits, pcm, extra chunk)
    (1, 22050, 16, True, b"LIST" + (3).to_bytes(4, "little") + b"abc\0"),
    (2, 48000, 24, True, b""),
    (1, 44100, 32, True, b"junk" + (4).to_bytes(4, "little") + b"wxyz"),
    (2, 44100, 32, False, b""),
    (2, 8000, 32, False, b""),
    (1, 96000, 16, True, b""),
]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_library_reader_equals_oracle(tmp_path, case):
    channels, rate, bits, pcm, extra = CASES[case]
    rng = np.random.default_rng(case)
    audio = (rng.standard_normal((channels, 3001 + case)) * 0.3).astype(np.float32)
    raw = fixtures.wav_bytes(audio, rate=rate, bits=bits, pcm=pcm, extra_chunk=extra)
    path = tmp_path / "in.wav"
    path.write_bytes(raw)
    ours = native.read_track(str(path))
    ref = O.read_track(raw)
    assert ours.shape == ref.shape
    assert np.array_equal(ours, ref)


def test_reader_refuses_unsupported(tmp_path):
    bad = {
        "8bit": fixtures.wav_bytes(np.zeros((1, 100), np.float32), bits=16, pcm=True).replace(
            b"\x10\x00data", b"\x08\x00data"),
        "3ch": fixtures.wav_bytes(np.zeros((3, 100), np.float32)),
        "notwav": b"RIFX" + b"\0" * 60,
    }
    for name, raw in bad.items():
        path = tmp_path / f"{name}.wav"
        path.write_bytes(raw)
        with pytest.raises(native.ProviderError):
            native.read_track(str(path))


def test_writer_stage_round_trip(tmp_path):
    rng = np.random.default_rng(7)
    audio = (rng.standard_normal((2, 999)) * 0.2).astype(np.float32)
    audio[0, 5] = np.nan
    audio[1, 7] = np.inf
    path = tmp_path / "out.wav"
    native.write_track(str(path), audio)
    back = fixtures.read_wav_f32(str(path))
    expect = np.where(np.isfinite(audio), audio, 0.0).astype(np.float32)
    assert np.array_equal(back, expect)
    assert np.array_equal(native.read_track(str(path)), expect)
