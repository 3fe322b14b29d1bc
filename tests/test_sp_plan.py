"""Sequence parallelism: the exchange plan moves every token row to its owner (no GPU).

``vocalarc_b200_separate_sp`` splits one clip across providers: band ranges for
the time-axis blocks, frame ranges for the band-axis blocks.  The library's own
copy plan (``vocalarc_b200_sp_plan``) is applied here to arrays of token ids
with numpy, exactly as the provider applies it with 2-D copies, and every
buffer must end up in the layout its next block expects.
"""

import numpy as np
import pytest

from karaoke_platform_sidecar_native_b200 import native

BANDS = 90


@pytest.fixture(scope="module", autouse=True)
def built():
    from karaoke_platform_sidecar_native_b200 import build
    build.build()


def ranges(n, total):
    return [(total * r // n, total * (r + 1) // n) for r in range(n)]


def band_shard(frames, lo, hi):
    """Token ids (band * frames + frame) of bands [lo, hi), band-major [nb][T]."""
    return np.arange(lo * frames, hi * frames, dtype=np.int64)


def frame_shard(frames, lo, hi):
    """Token ids of frames [lo, hi) over all bands, band-major [90][nf]."""
    b = np.arange(BANDS)[:, None]
    t = np.arange(lo, hi)[None, :]
    return (b * frames + t).reshape(-1).astype(np.int64)


def apply(plan, src_bufs, dst_bufs):
    for s, d, sr, sp, dr, dp, w, h in plan:
        for row in range(h):
            dst_bufs[d][dr + row * dp: dr + row * dp + w] = src_bufs[s][sr + row * sp: sr + row * sp + w]


@pytest.mark.parametrize("n,frames", [(1, 5), (2, 87), (3, 87), (4, 862), (8, 862), (7, 13), (90, 90)])
def test_exchanges_route_every_row(n, frames):
    full = np.arange(BANDS * frames, dtype=np.int64)
    bands, fr = ranges(n, BANDS), ranges(n, frames)
    size = BANDS * frames
    # Phase 0: provider 0's full band-major x to the band ranges (provider 0 keeps rows [0, nb0 T)).
    bufs = [full.copy()] + [np.full(size, -1, np.int64) for _ in range(n - 1)]
    apply(native.sp_plan(n, frames, 0), [b.copy() for b in bufs], bufs)
    for r, (lo, hi) in enumerate(bands):
        np.testing.assert_array_equal(bufs[r][:(hi - lo) * frames], band_shard(frames, lo, hi))
    # Phase 1: band ranges -> frame ranges (into fresh buffers).
    src = [b.copy() for b in bufs]
    dst = [np.full(size, -1, np.int64) for _ in range(n)]
    apply(native.sp_plan(n, frames, 1), src, dst)
    for r, (lo, hi) in enumerate(fr):
        np.testing.assert_array_equal(dst[r][:BANDS * (hi - lo)], frame_shard(frames, lo, hi))
    # Phase 2: frame ranges -> band ranges.
    back = [np.full(size, -1, np.int64) for _ in range(n)]
    apply(native.sp_plan(n, frames, 2), dst, back)
    for r, (lo, hi) in enumerate(bands):
        np.testing.assert_array_equal(back[r][:(hi - lo) * frames], band_shard(frames, lo, hi))
    # Phase 3: frame ranges -> provider 0's full band-major x.
    gathered = [np.full(size, -1, np.int64) for _ in range(n)]
    apply(native.sp_plan(n, frames, 3), dst, gathered)
    np.testing.assert_array_equal(gathered[0], full)


def test_each_copy_is_one_block_per_pair():
    plan = native.sp_plan(4, 862, 1)
    assert len(plan) == 16 and len({(p[0], p[1]) for p in plan}) == 16
    assert len(native.sp_plan(4, 862, 0)) == 3 and len(native.sp_plan(4, 862, 3)) == 4


@pytest.mark.parametrize("n,frames,phase", [(0, 10, 1), (91, 200, 1), (4, 3, 1), (2, 10, 4)])
def test_plan_rejects(n, frames, phase):
    with pytest.raises(native.ProviderError):
        native.sp_plan(n, frames, phase)
