"""Load fast path on the host: the converted device image and its on-disk cache (no GPU).

``vocalarc_b200_load_model`` uploads one image of the device allocation: per
axial block the 16-bit q|k|v|gate rows (attention gamma folded), out, FF1 (FF
gamma folded) and FF2 matrices and three fp32 vectors; the band split in fp32;
the mask head with the final gamma folded and layer-2 rows interleaved.  The
image is built on several threads and can come from a cache file.  These tests
check the bytes against a numpy conversion of the parsed pack.
"""

import os
import struct

import numpy as np
import pytest

from karaoke_platform_sidecar_native_b200 import modelpack as mp
from karaoke_platform_sidecar_native_b200 import native


def round4k(x):
    return (x + 4095) & ~4095


QKV_ROWS = mp.QKV_DIM + 16
BLOCK_BYTES = (QKV_ROWS * mp.DIM + mp.DIM * mp.DIM_INNER + 2 * mp.FF_DIM * mp.DIM) * 2 + \
    (mp.HEADS + mp.FF_DIM + mp.DIM) * 4 + 16 * 1024
BAND_BYTES = 4100 * 256 * 4 + 4100 * 4 + 90 * 256 * 4 + 90 * 8 + 91 * 4 + 16 * 1024
MASK_BYTES = 90 * 1024 * 256 * 2 + 90 * 1024 * 4 + 8400 * 1024 * 2 + 8400 * 4 + 256 * 4 + 256 * 1024
BLOCK_REGION, BAND_REGION, MASK_REGION = round4k(BLOCK_BYTES), round4k(BAND_BYTES), round4k(MASK_BYTES)


def align(x):
    return (x + 1023) & ~1023


def bf16_bits(x):
    bits = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)


@pytest.fixture(scope="module")
def lib():
    from karaoke_platform_sidecar_native_b200 import build
    build.build()
    return native.load()


@pytest.fixture(scope="module")
def image_fp16(lib, test_pack_blob):
    return native.model_image(test_pack_blob, bf16=False, threads=8)


def test_image_size(image_fp16):
    assert image_fp16.size == 32 * BLOCK_REGION + BAND_REGION + MASK_REGION


def test_image_is_independent_of_thread_count(test_pack_blob, image_fp16):
    np.testing.assert_array_equal(native.model_image(test_pack_blob, bf16=False, threads=1), image_fp16)


@pytest.mark.parametrize("layer,axis", [(0, 0), (7, 1), (15, 1)])
def test_block_bytes_match_numpy_conversion(test_model, image_fp16, layer, axis):
    w = test_model.layers[layer][axis]
    base = (2 * layer + axis) * BLOCK_REGION
    qkv = np.zeros((QKV_ROWS, mp.DIM), dtype=np.float32)
    qkv[:mp.QKV_DIM] = w["qkv"] * w["gamma"][None, :]
    qkv[mp.QKV_DIM:mp.QKV_DIM + mp.HEADS] = w["gate_weight"] * w["gamma"][None, :]
    off = 0
    for want in (qkv, w["out_weight"], w["ff1_weight"] * w["ff_gamma"][None, :], w["ff2_weight"]):
        n = want.size * 2
        got = image_fp16[base + off:base + off + n].view(np.float16).reshape(want.shape)
        np.testing.assert_array_equal(got, want.astype(np.float16))
        off = align(off + n)
    for vec in (w["gate_bias"], w["ff1_bias"], w["ff2_bias"]):
        got = image_fp16[base + off:base + off + vec.size * 4].view(np.float32)
        np.testing.assert_array_equal(got, vec)
        off = align(off + vec.size * 4)


def test_band_split_and_mask_bytes(test_model, image_fp16):
    band = 32 * BLOCK_REGION
    # W^T of band 0 ([8][256]) first, then band 1.
    wt0 = image_fp16[band:band + 8 * 256 * 4].view(np.float32).reshape(8, 256)
    np.testing.assert_array_equal(wt0, test_model.bands[0]["weight"].T)
    mask = band + BAND_REGION
    w1 = image_fp16[mask:mask + 1024 * 256 * 2].view(np.float16).reshape(1024, 256)
    want = (test_model.masks[0]["first_weight"] * test_model.final_gamma[None, :]).astype(np.float16)
    np.testing.assert_array_equal(w1, want)


def test_bf16_image_rounds_to_nearest_even(lib, test_pack_blob, test_model):
    image = native.model_image(test_pack_blob, bf16=True, threads=4)
    w = test_model.layers[0][0]
    got = image[:mp.QKV_DIM * mp.DIM * 2].view(np.uint16).reshape(mp.QKV_DIM, mp.DIM)
    np.testing.assert_array_equal(got, bf16_bits(w["qkv"] * w["gamma"][None, :]))


def test_rejects_foreign_pack(lib, test_pack_blob):
    bad = b"XXXXXXXX" + test_pack_blob[8:]
    with pytest.raises(native.ProviderError):
        native.model_image(bad)
    with pytest.raises(native.ProviderError):
        native.model_image(test_pack_blob[:len(test_pack_blob) // 2])


def test_store_writes_header_and_image(lib, test_pack_blob, image_fp16, tmp_path, monkeypatch):
    monkeypatch.setenv("VOCALARC_B200_IMAGE_CACHE", str(tmp_path / "cache"))
    path = native.store_model_image(test_pack_blob, bf16=False)
    assert path.startswith(str(tmp_path / "cache")) and path.endswith(".fp16.vbimg")
    data = open(path, "rb").read()
    assert len(data) == 64 + image_fp16.size
    magic, pack_hash, pack_bytes, layout, image_bytes, image_hash, bf16 = struct.unpack_from("<8sQQQQQI", data)
    assert magic == b"VBIMG001" and pack_bytes == len(test_pack_blob) and image_bytes == image_fp16.size
    assert bf16 == 0 and layout != 0 and image_hash != 0
    np.testing.assert_array_equal(np.frombuffer(data, dtype=np.uint8, offset=64), image_fp16)
    # The file name is the pack's content hash: a one-byte change gives another entry.
    changed = bytearray(test_pack_blob)
    changed[-1] ^= 1
    other = native.store_model_image(bytes(changed), bf16=False)
    assert other != path and os.path.exists(other)
    assert native.store_model_image(test_pack_blob, bf16=True).endswith(".bf16.vbimg")


def test_cache_can_be_switched_off(lib, test_pack_blob, monkeypatch):
    monkeypatch.setenv("VOCALARC_B200_IMAGE_CACHE", "off")
    with pytest.raises(native.ProviderError):
        native.store_model_image(test_pack_blob)
