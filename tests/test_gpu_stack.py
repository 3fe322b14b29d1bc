"""Configurable stack on the B200 against the stack oracle (config 3 and the bundled sizes).

Config 3 (dim 512, 62 bands, hop 441, GEGLU FFN, bf16) has no reference
implementation; its oracle (oracle/stack_oracle.py) composes the
reference-pinned operations and is itself pinned by reproducing the bundled
oracle exactly (tests/test_stack.py).  Tolerances, per stage on the same
inputs: spectral stages are fp32 SIMT (> 100 dB); one axial block through
16-bit tensor-core operands > 60 dB with fp16 and > 45 dB with bf16 (7-bit
significand); the depth-2 forward end to end >= 50 dB with fp16 and >= 35 dB
with bf16.
"""

import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from karaoke_platform_sidecar_native_b200 import fixtures, native, stack as st  # noqa: E402
from oracle import stack_oracle as SO  # noqa: E402
from oracle import vocalarc_oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu

SMALL3 = st.CONFIG3.replace(depth=2)
LENGTH = 441 * 100 + 123          # 101 frames


def snr_db(ref, test):
    ref = np.asarray(ref, dtype=np.float64)
    err = ref - np.asarray(test, dtype=np.float64)
    return 10 * math.log10((ref ** 2).sum() / max((err ** 2).sum(), 1e-300))


@pytest.fixture(scope="module")
def weights3():
    return st.synthetic_weights(SMALL3, seed=2, gamma_sigma=0.1, bias_sigma=0.02)


@pytest.fixture(scope="module", params=[True, False], ids=["bf16", "fp16"])
def stack3(request, weights3):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    s = st.Stack(SMALL3.replace(bf16=request.param), weights3)
    yield s
    s.close()


@pytest.fixture(scope="module")
def clips():
    a = fixtures.tone_mix(seconds=LENGTH / 44100, seed=11)[:, :LENGTH]
    b = (np.random.default_rng(12).standard_normal((2, LENGTH), dtype=np.float32) * np.float32(0.1))
    return np.ascontiguousarray(np.stack([a, b]), dtype=np.float32)    # [2][2][LENGTH]


def run(s, fn, *args):
    torch.cuda.synchronize()
    fn(*args)
    s.synchronize()
    assert s.lib.vocalarc_b200_stack_take_device_error(s.handle) == 0


def test_stft_hop441(stack3, clips):
    frames = SMALL3.frames(LENGTH)
    spec = torch.empty(2, frames, 1025, 2, 2, device="cuda")
    run(stack3, stack3.stage_stft, torch.from_numpy(clips).cuda(), 2, LENGTH, spec)
    for c in range(2):
        ref = SO.frame_major(O.stft(clips[c], 441))
        assert snr_db(ref, spec[c].cpu().numpy()) > 100


def test_band_split_62_bands_dim512(stack3, weights3, clips):
    w = st.split_weights(SMALL3, weights3)
    frames = SMALL3.frames(LENGTH)
    sources = [O.stft(clips[c], 441) for c in range(2)]
    spec = torch.from_numpy(np.stack([SO.frame_major(s) for s in sources])).cuda()
    x = torch.zeros(2, 62, frames, 512, device="cuda")
    run(stack3, stack3.stage_band_split, spec, 2, frames, x)
    for c in range(2):
        assert snr_db(SO.band_split(SMALL3, w, sources[c]), x[c].cpu().numpy()) > 100


@pytest.mark.parametrize("layer,axis", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_block_geglu_dim512(stack3, weights3, clips, layer, axis):
    w = st.split_weights(SMALL3, weights3)
    frames = SMALL3.frames(LENGTH)
    xs = [SO.band_split(SMALL3, w, O.stft(clips[c], 441)) for c in range(2)]
    x = torch.from_numpy(np.stack(xs)).cuda()
    run(stack3, stack3.stage_block, x, 2, frames, layer, axis)
    bar = 45 if stack3.cfg.bf16 else 60
    for c in range(2):
        ref = SO.block(SMALL3, w, layer, axis, xs[c])
        assert snr_db(ref, x[c].cpu().numpy()) > bar


def test_mask_62_bands(stack3, weights3, clips):
    w = st.split_weights(SMALL3, weights3)
    frames = SMALL3.frames(LENGTH)
    xs = [SO.block(SMALL3, w, 0, 0, SO.band_split(SMALL3, w, O.stft(clips[c], 441))) for c in range(2)]
    mask = torch.zeros(2, frames, 1025, 2, 2, device="cuda")
    run(stack3, stack3.stage_mask, torch.from_numpy(np.stack(xs)).cuda(), 2, frames, mask)
    bar = 45 if stack3.cfg.bf16 else 60
    for c in range(2):
        ref = SO.frame_major(SO.mask_estimate(SMALL3, w, xs[c]))
        assert snr_db(ref, mask[c].cpu().numpy()) > bar


def test_istft_hop441(stack3, clips):
    frames = SMALL3.frames(LENGTH)
    rng = np.random.default_rng(13)
    sources = [O.stft(clips[c], 441) for c in range(2)]
    masks = [rng.uniform(-1, 1, s.shape).astype(np.float32) for s in sources]
    out = torch.zeros(2, 2, LENGTH, device="cuda")
    spec = torch.from_numpy(np.stack([SO.frame_major(s) for s in sources])).cuda()
    mk = torch.from_numpy(np.stack([SO.frame_major(m) for m in masks])).cuda()
    run(stack3, stack3.stage_istft, spec, mk, 2, LENGTH, out)
    assert frames == sources[0].shape[2]
    for c in range(2):
        assert snr_db(O.istft(sources[c], masks[c], LENGTH, 441), out[c].cpu().numpy()) > 100


def test_forward_depth2(stack3, weights3, clips):
    got = stack3.separate(clips)
    bar = 35 if stack3.cfg.bf16 else 50
    for c in range(2):
        ref = SO.forward(SMALL3, weights3, clips[c])
        assert snr_db(ref, got[c]) >= bar
        assert np.isfinite(got[c]).all()


def test_bundled_sizes_match_the_provider(test_pack_blob, test_model):
    # The stack at the reference's sizes runs the same forward as the bundled path.
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    audio = fixtures.tone_mix(seconds=1.0, seed=3)
    p = native.Provider(0)
    p.load_model(test_pack_blob)
    ref = p.separate(audio)
    p.close()
    s = st.Stack(st.BUNDLED, st.weights_from_model(test_model))
    got = s.separate(audio)
    s.close()
    np.testing.assert_array_equal(got, ref)


def test_config3_full_size_is_deterministic():
    # Config 3 as benchmarked: 16 clips x 8 s, depth 12, bf16.
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    cfg = st.CONFIG3
    weights = st.synthetic_weights(cfg, seed=2)
    s = st.Stack(cfg, weights)
    g = torch.Generator(device="cuda").manual_seed(2)
    audio = torch.randn(st.CONFIG3_CLIPS, 2, st.CONFIG3_CLIP, device="cuda", generator=g) * 0.1
    outs = []
    for _ in range(2):
        out = torch.empty_like(audio)
        before = s.launch_count
        s.forward_device(audio, st.CONFIG3_CLIPS, st.CONFIG3_CLIP, out)
        s.synchronize()
        # stft, band split, row stats, 12 x 2 x (qkv, attention, out, norm, ff1, ff2, norm), 2 mask, istft, ola
        assert s.launch_count - before == 3 + 24 * 7 + 4
        outs.append(out.cpu())
    s.close()
    assert torch.isfinite(outs[0]).all()
    assert torch.equal(outs[0], outs[1])
    assert float(outs[0].abs().max()) > 0


SMALL_BUNDLED = st.BUNDLED.replace(depth=1)


@pytest.mark.parametrize("bf16", [True, False], ids=["bf16", "fp16"])
@pytest.mark.parametrize("axis", [0, 1])
def test_block_fused_ffn_dim256(bf16, axis):
    # Width 256 with a GELU FFN runs the fused FFN kernel (FF1, GELU and FF2
    # with the hidden on chip); both operand types against the stack oracle.
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    cfg = SMALL_BUNDLED.replace(bf16=bf16)
    weights = st.synthetic_weights(cfg, seed=4, gamma_sigma=0.1, bias_sigma=0.02)
    w = st.split_weights(cfg, weights)
    length = 512 * 150 + 77
    audio = fixtures.tone_mix(seconds=length / 44100 + 0.01, seed=21)[:, :length]
    clips2 = np.ascontiguousarray(np.stack([audio, audio[::-1]]), dtype=np.float32)
    frames = cfg.frames(length)
    xs = [SO.band_split(cfg, w, O.stft(clips2[c], cfg.hop)) for c in range(2)]
    s = st.Stack(cfg, weights)
    try:
        x = torch.from_numpy(np.stack(xs)).cuda()
        run(s, s.stage_block, x, 2, frames, 0, axis)
        bar = 45 if bf16 else 60
        for c in range(2):
            assert snr_db(SO.block(cfg, w, 0, axis, xs[c]), x[c].cpu().numpy()) > bar
    finally:
        s.close()
