"""The oracle's chunk assembly pinned against the reference's Python twin.

The C++ sidecar's chunked overlap-add, bigshifts and TTA
(onnx/native/onnx_sidecar.cpp:725-790, :556-575) need onnxruntime and cannot
run here.  The reference's Python twin of the same loop (onnx/audio.py:133-232)
can: tests/golden/make_demix_twin.py ran it, unchanged, with a deterministic
stand-in network and stored its outputs.  The oracle runs the same stand-in
here.  Where the two reference implementations agree, the oracle must agree
with the twin bit for bit; where they differ (the fade ramp, the first-batch
rule, the TTA sign), the oracle follows the C++ sidecar and each difference is
checked to be exactly the documented one.  The GPU chunked path is compared
with this oracle in tests/test_gpu_model.py and tests/test_gpu_tta.py.
"""

import hashlib
import json
import os

import numpy as np
import pytest

from oracle import vocalarc_oracle as O
from tests.conftest import GOLDEN
from tests.golden import make_demix_twin as twin

GOLD = np.load(os.path.join(GOLDEN, "demix_twin.npz"))
CASES = json.loads(str(GOLD["cases"]))


def setup(case):
    chunk, length, batch, shifts, tta, seed = CASES[case]
    mix = twin.mix_for(length, seed)
    assert hashlib.sha256(mix.tobytes()).hexdigest() == str(GOLD[f"{case}/mix_sha256"])
    ramp = twin.ramp_for(chunk)
    twin_fade = GOLD[f"ramp/{chunk}"]

    def separate(audio, fade_ramp=twin_fade):
        return O.demix(lambda part: twin.stand_in_numpy(part, ramp), audio, chunk, batch, fade_ramp=fade_ramp)

    return mix, separate, GOLD[f"{case}/out"]


@pytest.mark.parametrize("case", [c for c, v in CASES.items() if v[3] == 0 and v[2] >= 2])
def test_demix_matches_twin_bit_for_bit(case):
    # Model batch >= 2: the first-batch rule is off in both implementations
    # (position - step != 0 after the first batch), so with the twin's fade
    # ramp every sample must be identical: border reflection, pad_chunk's
    # reflect/zero fill, chunk positions, the final-batch weights, the
    # counter division and the crop.
    mix, separate, expected = setup(case)
    np.testing.assert_array_equal(separate(mix), expected)


@pytest.mark.parametrize("case", [c for c, v in CASES.items() if v[3] == 0 and v[2] >= 2])
def test_sidecar_fade_ramp_is_the_only_other_difference(case):
    # With its own ramp 1 - i/fade the oracle differs from the twin only by the
    # ramp's spacing (1/fade against 1/(fade - 1)): at most a few 1e-3 of the
    # signal inside a fade and nothing where the weights are forced to 1.
    mix, separate, expected = setup(case)
    got = separate(mix, fade_ramp=None)
    bound = 4.0 / (CASES[case][0] // 10) * float(np.abs(expected).max() + 1)
    assert float(np.abs(got - expected).max()) <= bound
    if CASES[case][2] >= 64:   # one batch: all weights forced to 1, no fade at all
        np.testing.assert_array_equal(got, expected)


def test_first_batch_rule_differs_only_in_the_first_chunks_fade():
    # Model batch 1: the sidecar sets the first chunk's weight to 1 over the
    # whole chunk (onnx_sidecar.cpp:762-765); in the twin the same rule sets
    # the window's first chunk/10 samples, which are 1 already (audio.py:170-171),
    # so the first chunk keeps its fade-out.  Everything outside that fade
    # (output samples [chunk - fade - border, chunk - border)) is identical.
    mix, separate, expected = setup("b1")
    chunk = CASES["b1"][0]
    fade, border = chunk // 10, chunk - chunk // 2
    got = separate(mix)
    lo, hi = chunk - fade - border, chunk - border
    outside = np.ones(got.shape[1], dtype=bool)
    outside[lo:hi] = False
    np.testing.assert_array_equal(got[:, outside], expected[:, outside])
    assert np.abs(got[:, lo + 1:hi] - expected[:, lo + 1:hi]).min() > 0


@pytest.mark.parametrize("case", [c for c, v in CASES.items() if v[3] > 0 and not v[4]])
def test_bigshift_matches_twin(case):
    # Rotation, inverse rotation and the mean of the shifted separations.  The
    # sidecar scales the sum by 1/count and the twin divides it (np.mean), so
    # three shifts may differ in the last bit.
    mix, separate, expected = setup(case)
    got = O.bigshift(separate, mix, CASES[case][3])
    if CASES[case][3] == 2:
        np.testing.assert_array_equal(got, expected)
    else:
        np.testing.assert_allclose(got, expected, rtol=0, atol=2 ** -22 * float(np.abs(expected).max()))


def test_tta_matches_twin_up_to_the_sidecars_polarity_sign():
    # The twin subtracts the estimate of -mix (audio.py:231); the sidecar
    # forms inverted = -bigshift(-mix) and adds it with right_scale = -1
    # (onnx_sidecar.cpp:572-573), i.e. it adds bigshift(-mix).  So the
    # sidecar's result is the twin's plus 2/3 of bigshift(-mix); the base and
    # the negated estimates themselves match the twin bit for bit.
    mix, separate, expected = setup("tta_b2")
    shifts = CASES["tta_b2"][3]
    np.testing.assert_array_equal(O.bigshift(separate, mix, shifts), GOLD["tta_b2/base"])
    negated = GOLD["tta_b2/negated"]
    np.testing.assert_array_equal(O.bigshift(separate, (mix * np.float32(-1.0)).astype(np.float32), shifts), negated)
    got = O.separate_tta(separate, mix, shifts, True)
    np.testing.assert_allclose(got, expected + np.float32(2.0 / 3.0) * negated, rtol=0,
                               atol=2 ** -20 * float(np.abs(expected).max() + np.abs(negated).max()))
