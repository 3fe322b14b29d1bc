"""Chunk scheduler: one track's chunks sharded across the GPUs of a node.

The chunked forward (``vocalarc_b200_separate_chunked``; the ONNX sidecar's
``Separator::demix``, onnx/native/onnx_sidecar.cpp:725-782) cuts a track into
chunks of 881,559 samples at a step of 440,779.  Chunks are independent given
the padded input, so each GPU (one process per GPU) takes a contiguous range of
them.  The only exchange is the overlap-add seam: the partial sums of the
``seam`` = chunk - step samples that a range's last chunk reaches into the next
range's samples (three float arrays, 5.3 MB).  The next range pulls it over
NVLink with a CUDA IPC peer copy -- no NCCL -- and starts its accumulators
from it, so the merged result is bit-identical to the single-GPU demix.

The process group (any ``torch.distributed`` backend) only carries the 64-byte
IPC handles and the barriers; the output gather goes through it too.
"""
from __future__ import annotations

from typing import Optional, Sequence

import numpy as np


def chunk_ranges(chunks: int, world: int) -> list:
    """Contiguous chunk ranges [c0, c1), one per rank.

    Every non-empty range holds at least two chunks (a seam then only reaches
    the next range), unless a single range covers the whole track.  Ranks past
    ``chunks // 2`` get an empty range.
    """
    if chunks <= 0 or world <= 0:
        raise ValueError("chunks and world must be positive")
    active = max(1, min(world, chunks // 2))
    base, extra = divmod(chunks, active)
    ranges, c = [], 0
    for r in range(world):
        if r < active:
            n = base + (1 if r < extra else 0)
            ranges.append((c, c + n))
            c += n
        else:
            ranges.append((chunks, chunks))
    return ranges


def separate_range(provider, d_audio, length: int, rank: int, world: int, group=None, chunk: int = 0,
                   model_batch: int = 1, d_vocals=None, plan: Optional[dict] = None):
    """This rank's part of a sharded chunked forward.

    Runs the rank's chunk range, exchanges seams with its neighbours and writes
    the rank's own output samples into ``d_vocals`` (device, [2][length]).
    Every rank of ``group`` must call it (collective).  Returns the owned
    output sample range (s0, s1), empty for a rank without chunks.
    """
    import torch.distributed as dist

    if plan is None:
        from . import native
        plan = native.chunk_plan(length, chunk)
    c0, c1 = chunk_ranges(plan["chunks"], world)[rank]
    active = c1 > c0
    if active:
        provider.range_forward(d_audio, length, c0, c1, chunk, model_batch)
    handle = provider.range_seam_export() if active and c1 < plan["chunks"] else None
    handles = [None] * world
    dist.all_gather_object(handles, handle, group=group)
    if active and c0 > 0:
        provider.range_seam_import(handles[rank - 1])
    owned = (0, 0)
    if active:
        provider.range_finish(d_vocals)
        owned = provider.range_owned()
    # The previous range's seam buffer may be reused only after every import.
    dist.barrier(group=group)
    return owned


def gather_output(vocals_host: np.ndarray, owned: Sequence[int], rank: int, world: int, group=None, dst: int = 0):
    """Assembles the full track on rank ``dst`` from every rank's owned slice.

    ``vocals_host`` is this rank's [2][length] host copy (only the owned slice
    is read).  Returns the full [2][length] array on ``dst``, None elsewhere.
    """
    import torch.distributed as dist

    s0, s1 = owned
    piece = (s0, s1, np.ascontiguousarray(vocals_host[:, s0:s1]))
    pieces = [None] * world if rank == dst else None
    dist.gather_object(piece, pieces, dst=dst, group=group)
    if rank != dst:
        return None
    out = np.zeros_like(vocals_host)
    for a, b, data in pieces:
        out[:, a:b] = data
    return out
