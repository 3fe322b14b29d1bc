"""The ONNX sidecar's bigshift + TTA quality pass on the device.

``vocalarc_b200_separate_tta`` runs all rotated / channel-swapped / polarity-
flipped copies of the mix through the chunked forward as one batch and combines
them on the device.  Two checks: (1) the combination equals the oracle's float32
restatement of ``Separator::separate`` (onnx_sidecar.cpp:556-575, :784-790)
applied to this provider's own chunked separations of each copy, bit for bit;
(2) end to end against the oracle forward, at the north-star bar.
"""
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from karaoke_platform_sidecar_native_b200 import fixtures, native  # noqa: E402
from oracle import vocalarc_oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def provider(test_pack_blob):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    p = native.Provider(0)
    p.load_model(test_pack_blob)
    yield p
    p.close()


def snr_db(ref, test):
    ref = np.asarray(ref, dtype=np.float64)
    err = ref - np.asarray(test, dtype=np.float64)
    return 10 * math.log10((ref ** 2).sum() / max((err ** 2).sum(), 1e-300))


@pytest.mark.parametrize("bigshifts,tta,batch", [(2, True, 1), (3, False, 1), (1, True, 2)])
def test_tta_combination_matches_restatement(provider, bigshifts, tta, batch):
    chunk = 16384
    audio = fixtures.tone_mix(1.3, seed=21)
    got = provider.separate_tta(audio, bigshifts=bigshifts, tta=tta, chunk=chunk, model_batch=batch)
    ref = O.separate_tta(lambda a: provider.separate_chunked(a, chunk=chunk, model_batch=batch), audio,
                         bigshifts, tta)
    assert np.array_equal(got, ref)


def test_tta_matches_oracle_forward(provider, test_model):
    chunk = 16384
    audio = fixtures.tone_mix(0.9, seed=22)
    ref = O.separate_tta(lambda a: O.demix(lambda c: O.forward(test_model, c), a, chunk=chunk), audio, 2, True)
    got = provider.separate_tta(audio, bigshifts=2, tta=True, chunk=chunk)
    assert snr_db(ref, got) >= 50.0
    assert np.abs(ref - got).max() <= 2e-3
