"""Sequence parallelism on the B200: one clip split across providers equals the whole-clip forward.

``vocalarc_b200_separate_sp`` runs the time-axis blocks on band ranges and the
band-axis blocks on frame ranges of one clip, exchanging x, its 16-bit copy and
the row norm factor between the axes.  Every row sees the arithmetic of the
single-provider forward, so the vocals must match ``vocalarc_b200_separate``
bit for bit.  On one GPU the providers share the device (the copies are then
device-local); with two or more GPUs, one provider per GPU.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from karaoke_platform_sidecar_native_b200 import fixtures, native  # noqa: E402

pytestmark = pytest.mark.gpu


def providers(blob, devices):
    out = []
    for d in devices:
        p = native.Provider(d)
        p.load_model(blob)
        out.append(p)
    return out


@pytest.mark.parametrize("count", [1, 2, 3])
def test_split_on_one_gpu_equals_whole_clip(test_pack_blob, count):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    audio = fixtures.tone_mix(seconds=1.0, seed=9)
    ps = providers(test_pack_blob, [0] * count)
    ref = ps[0].separate(audio)
    for _ in range(2):   # buffers are reused by the second call
        np.testing.assert_array_equal(native.separate_sp(ps, audio), ref)
    for p in ps:
        p.close()


def test_split_across_gpus_equals_whole_clip(test_pack_blob):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    n = min(torch.cuda.device_count(), 4)
    audio = fixtures.tone_mix(seconds=2.0, seed=10)
    ps = providers(test_pack_blob, list(range(n)))
    ref = ps[0].separate(audio)
    np.testing.assert_array_equal(native.separate_sp(ps, audio), ref)
    for p in ps:
        p.close()


def test_split_rejects_too_few_frames(test_pack_blob):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ps = providers(test_pack_blob, [0, 0])
    with pytest.raises(native.ProviderError):
        native.separate_sp(ps, np.zeros((2, 100), dtype=np.float32))   # 1 frame, 2 providers
    for p in ps:
        p.close()


def test_split_rejects_different_models(test_pack_blob):
    # Every provider of a split must hold the same pack (compared by content hash).
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from karaoke_platform_sidecar_native_b200 import modelpack
    a = native.Provider(0)
    a.load_model(test_pack_blob)
    b = native.Provider(0)
    b.load_model(modelpack.synthetic_pack(**modelpack.BENCH_RECIPE))
    with pytest.raises(native.ProviderError):
        native.separate_sp([a, b], fixtures.tone_mix(seconds=1.0, seed=9))
    a.close()
    b.close()
