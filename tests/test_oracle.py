"""The CPU oracle pinned against the reference executable's own outputs.

The golden fixtures come from the unchanged reference CPU build
(tests/golden/make_golden.py); these tests need no GPU and no checkout of the reference.
"""

import os

import numpy as np
import pytest

from karaoke_platform_sidecar_native_b200 import modelpack
from oracle import vocalarc_oracle as O
from tests.conftest import GOLDEN

CASES = ("clip_a", "clip_t1", "clip_t2")


def snr_db(ref, test):
    ref = np.asarray(ref, dtype=np.float64)
    err = ref - np.asarray(test, dtype=np.float64)
    return 10.0 * np.log10(max((ref ** 2).sum(), 1e-300) / max((err ** 2).sum(), 1e-300))


def load(case):
    return np.load(os.path.join(GOLDEN, f"{case}.npz"))


def test_pack_regenerates_bit_identical(test_pack_sha256):
    # The golden outputs were produced with this exact synthetic pack.
    for case in CASES:
        assert str(load(case)["pack_sha256"]) == test_pack_sha256


def test_pack_size_matches_manifest(test_pack_blob):
    assert len(test_pack_blob) == modelpack.PACK_BYTES == 267_386_408


def test_pack_round_trip():
    rng = np.random.default_rng(1)
    for fin, fout in ((256, 1536), (256, 8), (1024, 1032), (8, 256), (1024, 16)):
        w = rng.standard_normal((fout, fin)).astype(np.float32)
        assert np.array_equal(modelpack.unpack_matrix(modelpack.pack_matrix(w), fin, fout), w)


def test_bad_header_rejected(test_pack_blob):
    bad = bytearray(test_pack_blob[:200])
    bad[8 + 4 * 9] = 0xB9  # HOP field no longer 512
    with pytest.raises(ValueError):
        modelpack.parse_pack(bytes(bad))


@pytest.mark.parametrize("case", CASES)
def test_oracle_matches_reference_stages(case, test_model):
    g = load(case)
    stages = {}
    vocals = O.forward(test_model, g["audio"], keep=(1, 16), stages=stages)
    frames = int(g["frames"])
    assert stages["source"].shape[2] == frames
    # STFT: reference uses a double radix-2 FFT; float32 rounding only.
    assert snr_db(g["source"], stages["source"]) > 120
    kept = list(g["bands_kept"])
    assert snr_db(g["band"], stages["band"][kept]) > 110
    fk = list(g["frames_kept"])
    assert snr_db(g["features1"], stages["dumps"][1][fk]) > 105
    assert snr_db(g["features16"], stages["dumps"][16][fk]) > 100
    assert snr_db(g["mask"], stages["mask"]) > 100
    assert snr_db(g["vocals"], vocals) > 100
    assert np.abs(g["vocals"] - vocals).max() < 1e-6


def test_reflect_index_matches_definition():
    # reflect_index (vocalarc_separation.c:1027-1034) applied repeatedly.
    def scalar(i, n):
        if n <= 1:
            return 0
        while i < 0 or i >= n:
            i = -i if i < 0 else 2 * n - 2 - i
        return i
    idx = np.arange(-3000, 3000)
    for n in (1, 2, 3, 300, 1000):
        assert list(O.reflect_index(idx, n)) == [scalar(int(i), n) for i in idx]


def test_chunk_plan_counts():
    # 240 s -> 27 chunks, 180 s -> 21 chunks (reflect-padded by the border).
    for seconds, count in ((240, 27), (180, 21)):
        border, padded, plan = O.chunk_plan(seconds * 44100)
        assert border == O.CHUNK_SAMPLES - O.STEP_SAMPLES
        assert padded == seconds * 44100 + 2 * border
        assert len(plan) == count
    assert O.frames_for(O.CHUNK_SAMPLES) == modelpack.MODEL_FRAMES


def test_chunk_weights_first_and_final_batches():
    w1 = O.chunk_weights(5, 100, batch=1)
    assert np.all(w1[0] == 1) and np.all(w1[4] == 1)
    assert w1[2, -1] == pytest.approx(0.1) and w1[2, 0] == 1
    w2 = O.chunk_weights(5, 100, batch=2)
    # With a model batch of two the first batch is not forced to 1
    # (position - step != 0 after it, onnx_sidecar.cpp:762).
    assert w2[0, -1] == pytest.approx(0.1) and np.all(w2[4] == 1)


def test_demix_identity_predict_reconstructs_input():
    # An identity "model" must give back the input: fade weights cancel in the
    # result / counter division, and the border crop restores alignment.
    rng = np.random.default_rng(0)
    mix = rng.standard_normal((2, 5000)).astype(np.float32)
    out = O.demix(lambda chunk: chunk, mix, chunk=1200)
    assert np.allclose(out, mix, atol=1e-6)
