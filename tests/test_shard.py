"""Chunk scheduler (one track's chunks sharded across GPUs) on the CPU.

The scheduler logic and the seam exchange protocol run as ``gloo`` ranks with a
numpy stand-in for the provider: per-chunk "model outputs" are seeded arrays and
the range forward / seam / finish arithmetic restates the device kernel
(``demix_range_kernel``: accumulators start from the previous range's seam and
add this range's chunks in ascending order).  The sharded result must equal the
single-process overlap-add bit for bit, the property the device test checks on
the GPU.  No GPU is used here.
"""
import os
import pickle

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

from karaoke_platform_sidecar_native_b200 import shard  # noqa: E402
from oracle import vocalarc_oracle as O  # noqa: E402

F32 = np.float32


def plan_of(length, chunk):
    border, padded, starts = O.chunk_plan(length, chunk)
    step = chunk // 2
    return {"chunks": len(starts), "step": step, "border": border if padded != length else 0,
            "seam": chunk - step, "padded": padded}


def chunk_output(c, chunk):
    return np.random.default_rng(1000 + c).standard_normal((2, chunk)).astype(F32)


def accumulate(plan, chunk, batch, c0, c1, p0, p1, init=None, init_p0=0):
    """Accumulators of padded samples [p0, p1) over chunks [c0, c1), ascending."""
    weights = O.chunk_weights(plan["chunks"], chunk, batch)
    n = p1 - p0
    res = np.zeros((2, n), F32)
    cnt = np.zeros(n, F32)
    if init is not None:
        k0 = max(p0, init_p0) - init_p0
        k1 = min(p1, init_p0 + init.shape[1]) - init_p0
        if k1 > k0:
            res[:, k0 + init_p0 - p0:k1 + init_p0 - p0] = init[:2, k0:k1]
            cnt[k0 + init_p0 - p0:k1 + init_p0 - p0] = init[2, k0:k1]
    for c in range(c0, c1):
        start = c * plan["step"]
        valid = min(chunk, plan["padded"] - start)
        a, b = max(p0, start), min(p1, start + valid)
        if b <= a:
            continue
        i = np.arange(a - start, b - start)
        w = weights[c, i]
        res[:, a - p0:b - p0] += chunk_output(c, chunk)[:, i] * w
        cnt[a - p0:b - p0] += w
    return res, cnt


class FakeProvider:
    """numpy stand-in with the provider's chunk-range methods."""

    def __init__(self, plan, chunk, batch):
        self.plan, self.chunk, self.batch = plan, chunk, batch

    def range_forward(self, d_audio, length, c0, c1, chunk, model_batch):
        self.length, self.c0, self.c1 = length, c0, c1
        self.seam_in = None
        if c1 < self.plan["chunks"]:
            p0 = c1 * self.plan["step"]
            res, cnt = accumulate(self.plan, self.chunk, self.batch, c0, c1, p0, p0 + self.plan["seam"])
            self.seam_out = np.concatenate([res, cnt[None]])

    def range_seam_export(self):
        return pickle.dumps(self.seam_out)   # stands in for the 64-byte CUDA IPC handle

    def range_seam_import(self, handle):
        self.seam_in = pickle.loads(handle)

    def _owned_padded(self):
        p0 = self.c0 * self.plan["step"]
        p1 = self.c1 * self.plan["step"] if self.c1 < self.plan["chunks"] else self.plan["padded"]
        return p0, p1

    def range_finish(self, vocals):
        assert self.c0 == 0 or self.seam_in is not None
        p0, p1 = self._owned_padded()
        res, cnt = accumulate(self.plan, self.chunk, self.batch, self.c0, self.c1, p0, p1, self.seam_in, p0)
        out = (res / np.maximum(cnt, F32(1e-12))).astype(F32)
        s = np.arange(p0, p1) - self.plan["border"]
        keep = (s >= 0) & (s < self.length)
        vocals[:, s[keep]] = out[:, keep]

    def range_owned(self):
        p0, p1 = self._owned_padded()
        b = self.plan["border"]
        return max(0, min(self.length, p0 - b)), max(0, min(self.length, p1 - b))


def reference(plan, chunk, batch, length):
    res, cnt = accumulate(plan, chunk, batch, 0, plan["chunks"], 0, plan["padded"])
    out = (res / np.maximum(cnt, F32(1e-12))).astype(F32)
    b = plan["border"]
    return out[:, b:b + length]


def _rank_main(rank, world, port, length, chunk, batch, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = plan_of(length, chunk)
        provider = FakeProvider(plan, chunk, batch)
        vocals = np.zeros((2, length), F32)
        owned = shard.separate_range(provider, None, length, rank, world, chunk=chunk, model_batch=batch,
                                     d_vocals=vocals, plan=plan)
        full = shard.gather_output(vocals, owned, rank, world)
        if rank == 0:
            np.save(result_path, full)
    finally:
        dist.destroy_process_group()


def test_chunk_ranges_cover_and_hold_two_chunks():
    for chunks in range(1, 40):
        for world in range(1, 10):
            ranges = shard.chunk_ranges(chunks, world)
            assert len(ranges) == world
            nonempty = [r for r in ranges if r[1] > r[0]]
            assert nonempty[0][0] == 0 and nonempty[-1][1] == chunks
            for (a0, a1), (b0, b1) in zip(nonempty, nonempty[1:]):
                assert a1 == b0
            if len(nonempty) > 1:
                assert all(b - a >= 2 for a, b in nonempty)
            assert all(r == (chunks, chunks) for r in ranges[len(nonempty):])


def test_chunk_plan_matches_oracle():
    from karaoke_platform_sidecar_native_b200 import native
    for length in (1000, 881559, 881560 * 2 + 1, 44100 * 60, 44100 * 240):
        plan = native.chunk_plan(length)
        ref = plan_of(length, O.CHUNK_SAMPLES)
        assert (plan["chunks"], plan["step"], plan["border"], plan["seam"]) == \
            (ref["chunks"], ref["step"], ref["border"], ref["seam"])


@pytest.mark.parametrize("world,batch", [(2, 1), (3, 2)])
def test_sharded_overlap_add_is_bit_identical(tmp_path, world, batch):
    # A small chunk keeps the numpy work short; the plan has the bundled shape
    # (step = chunk // 2, seam = chunk - step, reflect border).
    chunk = 2001
    length = 9000
    port = 29500 + os.getpid() % 1000 + world
    result = str(tmp_path / "full.npy")
    mp.start_processes(_rank_main, args=(world, port, length, chunk, batch, result), nprocs=world,
                       start_method="spawn")
    full = np.load(result)
    ref = reference(plan_of(length, chunk), chunk, batch, length)
    assert np.array_equal(full, ref)
