"""The allocation-free iSTFT entry point agrees with the regular one.

``vocalarc_b200_stage_istft_noalloc`` exists for callers that cannot call
cudaMalloc while processing audio (real-time audio threads, hosts with a GPU
memory budget fixed at load time).  It keeps its frame scratch in a fixed
device array instead of a buffer sized on demand.  This file is collected last
so that a run stopping at the first failure has run every other test before it.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from karaoke_platform_sidecar_native_b200 import native  # noqa: E402
from oracle import vocalarc_oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu


def _inputs(seed, segments, length):
    rng = np.random.default_rng(seed)
    specs, masks = [], []
    for _ in range(segments):
        audio = (rng.standard_normal((2, length)) * 0.1).astype(np.float32)
        source = O.stft(audio)                                            # [1025][2][T][2]
        mask = (rng.standard_normal(source.shape) * 0.3).astype(np.float32)
        specs.append(source.transpose(2, 0, 1, 3))                         # frame-major
        masks.append(mask.transpose(2, 0, 1, 3))
    return (torch.from_numpy(np.ascontiguousarray(np.stack(specs))).cuda(),
            torch.from_numpy(np.ascontiguousarray(np.stack(masks))).cuda())


def test_noalloc_istft_matches_regular_entry_point_twice():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    provider = native.Provider(0)
    try:
        # Two calls in a row with different shapes and data: the shared scratch
        # keeps the first call's contents, which must not leak into the second.
        for seed, segments, length in ((1, 2, 44100), (2, 1, 881559)):
            spec, mask = _inputs(seed, segments, length)
            regular = torch.zeros(segments, 2, length, device="cuda")
            noalloc = torch.full((segments, 2, length), float("nan"), device="cuda")
            torch.cuda.synchronize()
            provider.stage_istft(spec, mask, segments, length, regular)
            provider.synchronize()
            provider.stage_istft_noalloc(spec, mask, segments, length, noalloc)
            provider.synchronize()
            assert provider.take_device_error() == 0
            a = regular.cpu().numpy().astype(np.float64)
            b = noalloc.cpu().numpy().astype(np.float64)
            assert np.isfinite(b).all()
            # Same kernels on the same inputs: the tolerance used for iSTFT
            # parity elsewhere (SNR > 100 dB) holds with room to spare.
            snr = 10 * np.log10((a ** 2).sum() / max(((a - b) ** 2).sum(), 1e-300))
            assert snr > 100
        # A request beyond the fixed scratch (2048 frames) is refused, not run.
        # The buffers have the requested size (3 x 1722 frames, about 85 MB
        # each), so even a broken size check could not read past them.
        frames = 881559 // 512 + 1
        spec = torch.zeros(3, frames, 1025, 2, 2, device="cuda")
        mask = torch.zeros_like(spec)
        out = torch.zeros(3, 2, 881559, device="cuda")
        ok = provider.lib.vocalarc_b200_stage_istft_noalloc(provider.handle, native.dptr(spec), native.dptr(mask), 3,
                                                            881559, native.dptr(out))
        assert ok == 0
    finally:
        provider.close()
