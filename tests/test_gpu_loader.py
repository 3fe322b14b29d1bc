"""Load fast path on the B200: converted vs cached vs mmap'd-file loads give the same forward.

The first load of a pack converts it on several threads and writes the device
image to the cache directory; later loads of the same bytes (or the same file
through vocalarc_b200_load_model_file) copy that image instead.  A damaged
image fails its hash check and is rebuilt.
"""

import glob
import os
import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from karaoke_platform_sidecar_native_b200 import fixtures, native  # noqa: E402

pytestmark = pytest.mark.gpu


def timed_load(provider, loader, arg):
    t = time.perf_counter()
    loader(arg)
    return (time.perf_counter() - t) * 1000.0


def test_image_cache_round_trip(test_pack_blob, test_pack_path, tmp_path, monkeypatch):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    monkeypatch.setenv("VOCALARC_B200_IMAGE_CACHE", str(tmp_path))
    audio = fixtures.tone_mix(seconds=1.0, seed=5)
    outs, times, cached = [], [], []
    for how in ("convert", "cached", "file", "damaged"):
        if how == "damaged":
            (path,) = glob.glob(str(tmp_path / "*.fp16.vbimg"))
            with open(path, "r+b") as handle:
                handle.seek(64 + 12345)
                byte = handle.read(1)
                handle.seek(64 + 12345)
                handle.write(bytes([byte[0] ^ 0x40]))
        p = native.Provider(0)
        if how == "file":
            times.append(timed_load(p, p.load_model_file, test_pack_path))
        else:
            times.append(timed_load(p, p.load_model, test_pack_blob))
        cached.append(p.model_from_cache)
        outs.append(p.separate(audio))
        p.close()
    print("load ms (convert, cached, file, damaged):", [round(t, 1) for t in times])
    assert cached == [False, True, True, False]
    for out in outs[1:]:
        np.testing.assert_array_equal(out, outs[0])
    assert len(glob.glob(str(tmp_path / "*.vbimg"))) == 1


def test_image_cache_off(test_pack_blob, tmp_path, monkeypatch):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    monkeypatch.setenv("VOCALARC_B200_IMAGE_CACHE", "off")
    monkeypatch.setenv("HOME", str(tmp_path))
    p = native.Provider(0)
    p.load_model(test_pack_blob)
    assert not p.model_from_cache
    p.load_model(test_pack_blob)
    assert not p.model_from_cache
    p.close()
    assert not os.listdir(tmp_path)
