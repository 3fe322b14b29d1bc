"""One track's chunks sharded across providers: bit-identical to the single-GPU demix.

Single GPU: three providers on cuda:0 each run a chunk range and hand their
seam to the next (same-process peer copy), exactly the multi-GPU sequence.
Two GPUs: two processes, one per GPU, exchange the seam through CUDA IPC over
NVLink (skipped when fewer than two GPUs are visible).
"""
import os
import tempfile

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from karaoke_platform_sidecar_native_b200 import fixtures, native, shard  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def providers(test_pack_blob):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ps = []
    for _ in range(3):
        p = native.Provider(0)
        p.load_model(test_pack_blob)
        ps.append(p)
    yield ps
    for p in ps:
        p.close()


def single_gpu_vocals(provider, d_audio, length, batch):
    d_out = torch.zeros_like(d_audio)
    torch.cuda.synchronize()
    provider.separate_device(d_audio, 1, length, d_out, chunked=True, model_batch=batch)
    provider.synchronize()
    return d_out


@pytest.mark.parametrize("seconds,batch", [(60.0, 1), (47.0, 2)])
def test_sharded_ranges_match_single_gpu(providers, seconds, batch):
    audio = fixtures.long_mix(seconds, seed=11)
    length = audio.shape[1]
    d_audio = torch.from_numpy(audio).cuda()
    plan = native.chunk_plan(length)
    ranges = shard.chunk_ranges(plan["chunks"], len(providers))
    assert all(b - a >= 2 for a, b in ranges)
    d_sharded = torch.full_like(d_audio, float("nan"))
    torch.cuda.synchronize()
    for p, (c0, c1) in zip(providers, ranges):
        p.range_forward(d_audio, length, c0, c1, model_batch=batch)
    for prev, p in zip(providers, providers[1:]):
        p.range_seam_from(prev)
    covered = []
    for p in providers:
        p.range_finish(d_sharded)
        covered.append(p.range_owned())
    assert covered[0][0] == 0 and covered[-1][1] == length
    assert all(a[1] == b[0] for a, b in zip(covered, covered[1:]))
    ref = single_gpu_vocals(providers[0], d_audio, length, batch)
    assert torch.equal(d_sharded, ref)


def _ipc_rank(rank, world, port, pack_path, seconds, result_path):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.cuda.set_device(rank)
        p = native.Provider(rank)
        with open(pack_path, "rb") as handle:
            p.load_model(handle.read())
        audio = fixtures.long_mix(seconds, seed=11)
        length = audio.shape[1]
        d_audio = torch.from_numpy(audio).cuda(rank)
        d_vocals = torch.zeros_like(d_audio)
        torch.cuda.synchronize()
        owned = shard.separate_range(p, d_audio, length, rank, world, d_vocals=d_vocals)
        full = shard.gather_output(d_vocals.cpu().numpy(), owned, rank, world)
        if rank == 0:
            ref = single_gpu_vocals(p, d_audio, length, 1).cpu().numpy()
            np.save(result_path, np.stack([full, ref]))
        p.close()
    finally:
        dist.destroy_process_group()


def test_sharded_ipc_two_gpus(test_pack_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as tmp:
        result = os.path.join(tmp, "r.npy")
        mp.start_processes(_ipc_rank, args=(2, 29650 + os.getpid() % 200, test_pack_path, 60.0, result), nprocs=2,
                           start_method="spawn")
        full, ref = np.load(result)
    assert np.array_equal(full, ref)
