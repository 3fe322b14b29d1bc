"""Configurable stack: weight layout, configuration checks and the oracle's pin (no GPU).

The stack oracle (oracle/stack_oracle.py) composes the reference-pinned
operations of oracle/vocalarc_oracle.py at a configuration's sizes.  With the
bundled sizes it must reproduce vocalarc_oracle.forward exactly; that is what
ties the config-3 oracle (dim 512, 62 bands, hop 441, GEGLU) to the reference.
"""

import numpy as np
import pytest

from karaoke_platform_sidecar_native_b200 import fixtures, stack as st
from oracle import stack_oracle as SO
from oracle import vocalarc_oracle as O


@pytest.fixture(scope="module")
def built():
    from karaoke_platform_sidecar_native_b200 import build
    build.build()


def test_config3_shape():
    cfg = st.CONFIG3
    assert cfg.bands == 62 and sum(cfg.band_bins) == 1025
    assert cfg.frames(st.CONFIG3_CLIP) == 801            # 8 s at hop 441
    assert cfg.ff1_rows == 2 * 2048 and cfg.dim == 512 and cfg.depth == 12
    # Parameter count: 24 blocks of 4.20 M, band split 2.10 M, mask head 81.8 M.
    assert st.weight_count(cfg) == 24 * (512 + 1536 * 512 + 8 * 512 + 8 + 512 * 512 + 512 + 4096 * 512 + 4096
                                         + 512 * 2048 + 512) + (4100 + 4100 * 512 + 62 * 512) + 512 + \
        (62 * (2048 * 512 + 2048) + 2 * 4100 * 2048 + 2 * 4100)


@pytest.mark.parametrize("cfg", [st.CONFIG3, st.BUNDLED, st.CONFIG3.replace(depth=2, bf16=False),
                                 st.BUNDLED.replace(geglu=True, ff_inner=384, mask_hidden=512, hop=300)])
def test_library_weight_count_matches(built, cfg):
    assert st.library_weight_count(cfg) == st.weight_count(cfg)


@pytest.mark.parametrize("change", [dict(dim=384), dict(heads=4), dict(dim_head=32), dict(n_fft=1024),
                                    dict(ff_inner=200), dict(geglu=False, ff_inner=384), dict(mask_hidden=300),
                                    dict(hop=0), dict(hop=4096), dict(depth=0),
                                    dict(band_bins=st.BSROFORMER_62_BANDS[:-1]),
                                    dict(band_bins=(130,) + (129,) * 6 + (121,))])
def test_library_rejects_unsupported(built, change):
    assert st.library_weight_count(st.CONFIG3.replace(**change)) == 0


def test_bundled_weights_round_trip(test_model):
    flat = st.weights_from_model(test_model)
    assert flat.size == st.weight_count(st.BUNDLED)
    w = st.split_weights(st.BUNDLED, flat)
    np.testing.assert_array_equal(w["layers.3.1.ff1_weight"], test_model.layers[3][1]["ff1_weight"])
    np.testing.assert_array_equal(w["bands.89.weight"], test_model.bands[89]["weight"])
    np.testing.assert_array_equal(w["masks.0.second_bias"], test_model.masks[0]["second_bias"])
    np.testing.assert_array_equal(w["final_gamma"], test_model.final_gamma)


def test_stack_oracle_with_bundled_sizes_is_the_pinned_oracle(test_model):
    audio = fixtures.tone_mix(seed=0, seconds=0.2)
    ref = O.forward(test_model, audio)
    got = SO.forward(st.BUNDLED, st.weights_from_model(test_model), audio)
    np.testing.assert_array_equal(got, ref)


def test_stft_hop441_matches_direct_frames():
    rng = np.random.default_rng(3)
    audio = rng.standard_normal((2, 441 * 20 + 17), dtype=np.float32) * np.float32(0.1)
    spec = O.stft(audio, 441)
    assert spec.shape == (1025, 2, audio.shape[1] // 441 + 1, 2)
    win = O.window().astype(np.float64)
    for f in (0, 3, 12, spec.shape[2] - 1):
        idx = O.reflect_index(np.arange(2048) + f * 441 - 1024, audio.shape[1])
        direct = np.fft.fft(audio[1][idx].astype(np.float64) * win)[:1025]
        np.testing.assert_allclose(spec[:, 1, f, 0], direct.real, atol=2e-5)
        np.testing.assert_allclose(spec[:, 1, f, 1], direct.imag, atol=2e-5)


def test_istft_hop441_inverts_stft():
    # With an all-ones mask the window-envelope division makes the round trip exact.
    rng = np.random.default_rng(4)
    audio = rng.standard_normal((2, 441 * 30), dtype=np.float32) * np.float32(0.1)
    spec = O.stft(audio, 441)
    ones = np.zeros_like(spec)
    ones[..., 0] = 1.0
    back = O.istft(spec, ones, audio.shape[1], 441)
    np.testing.assert_allclose(back, audio, atol=2e-6)


def test_geglu_block_uses_value_times_gelu_gate():
    cfg = st.BUNDLED.replace(depth=1, geglu=True, ff_inner=128, mask_hidden=256)
    flat = st.synthetic_weights(cfg, seed=5, gamma_sigma=0.1, bias_sigma=0.02)
    w = st.split_weights(cfg, flat)
    x = np.random.default_rng(6).standard_normal((3, 7, cfg.dim), dtype=np.float32)
    out = SO.transformer(cfg, w, "layers.0.0.", x)
    # The same block with the FFN written out by hand.
    p = "layers.0.0."
    zero_ffn = dict(w)
    zero_ffn[p + "ff2_weight"] = np.zeros_like(w[p + "ff2_weight"])
    zero_ffn[p + "ff2_bias"] = np.zeros_like(w[p + "ff2_bias"])
    attn_only = SO.transformer(cfg, zero_ffn, p, x)
    normed = O.rms_norm(attn_only, w[p + "ff_gamma"])
    pre = normed @ w[p + "ff1_weight"].T + w[p + "ff1_bias"]
    hidden = pre[..., :128] * O.gelu(pre[..., 128:])
    expect = attn_only + hidden @ w[p + "ff2_weight"].T + w[p + "ff2_bias"]
    np.testing.assert_allclose(out, expect, rtol=1e-5, atol=1e-5)


def test_synthetic_weights_recipe():
    cfg = st.BUNDLED.replace(depth=1)
    flat = st.synthetic_weights(cfg, seed=2)
    w = st.split_weights(cfg, flat)
    assert np.all(w["final_gamma"] == 1.0) and np.all(w["layers.0.1.ff2_bias"] == 0.0)
    assert abs(float(np.std(w["layers.0.0.qkv"])) - 0.02) < 1e-3
    again = st.synthetic_weights(cfg, seed=2)
    np.testing.assert_array_equal(flat, again)
