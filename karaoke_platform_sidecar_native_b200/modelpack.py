"""VSCNAT01 model pack: layout constants, a seeded synthetic writer and a reader.

The bundled ``bs_leap_xe_voc`` pack is a Git-LFS object that is not available to
this build, so every run uses a seeded synthetic pack written in exactly the
reference layout.  The layout follows ``model_parse``
(native/vocalarc_separation.c:528-589):

* 8-byte magic ``VSCNAT01`` and 14 little-endian u32 fields; fields 0..11 are
  checked against the compile-time constants (vocalarc_separation.c:535-542);
* 16 layers x 2 axes (axis 0 = time, axis 1 = band) of ten transformer tensors
  (vocalarc_separation.c:543-563);
* 90 band-split triples (gamma, weight, bias) (vocalarc_separation.c:564-571);
* the final gamma, then 90 mask-MLP quadruples (vocalarc_separation.c:572-583).

Each tensor is a u64 element count followed by that many f32 values.  Matrices
are stored in the reference's 32-lane packed layout: for every full block of 32
outputs an ``[in][32]`` slab, then an ``[in][out % 32]`` tail slab
(``matmul_row_scalar`` vocalarc_separation.c:428-457; decoded by
``unpack_weight`` native/native_gpu_cuda.cu:104-124).  With the reference
constants the pack is exactly 267,386,408 bytes, the size recorded in
native/assets/manifest.json:6.
"""

from __future__ import annotations

import os
import struct
import tempfile
from dataclasses import dataclass, field

import numpy as np

MAGIC = b"VSCNAT01"
DIM = 256
DEPTH = 16
BANDS = 90
HEADS = 8
DIM_HEAD = 64
DIM_INNER = 512
QKV_DIM = 1536
FF_DIM = 1024
FREQ_BINS = 1025
CHANNELS = 2
NFFT = 2048
HOP = 512
WIN_LENGTH = 2048
MODEL_FRAMES = 1722
SAMPLE_RATE = 44100
PACK_BYTES = 267_386_408

#: Band widths in STFT bins (vocalarc_separation.c:50-57); they sum to 1025.
BAND_FREQS = (2,) * 24 + (4,) * 36 + (12,) * 16 + (24,) * 8 + (48,) * 4 + (128, 129)
assert len(BAND_FREQS) == BANDS and sum(BAND_FREQS) == FREQ_BINS
#: Band-split input width d_b = bins x channels x (re, im).
BAND_DIMS = tuple(4 * w for w in BAND_FREQS)
BAND_FIRST = tuple(int(x) for x in np.concatenate([[0], np.cumsum(BAND_FREQS)[:-1]]))

#: (name, in_features, out_features or None for vectors) of one transformer, in
#: pack order (vocalarc_separation.c:551-560).
TRANSFORMER_TENSORS = (
    ("gamma", None, DIM),
    ("qkv", DIM, QKV_DIM),
    ("gate_weight", DIM, HEADS),
    ("gate_bias", None, HEADS),
    ("out_weight", DIM_INNER, DIM),
    ("ff_gamma", None, DIM),
    ("ff1_weight", DIM, FF_DIM),
    ("ff1_bias", None, FF_DIM),
    ("ff2_weight", FF_DIM, DIM),
    ("ff2_bias", None, DIM),
)


def pack_matrix(weight: np.ndarray) -> np.ndarray:
    """Logical ``W[out][in]`` -> the reference's 32-lane packed flat layout."""
    out_features, in_features = weight.shape
    full = (out_features // 32) * 32
    pieces = []
    for tile in range(0, full, 32):
        pieces.append(np.ascontiguousarray(weight[tile:tile + 32].T).reshape(-1))
    if full < out_features:
        pieces.append(np.ascontiguousarray(weight[full:].T).reshape(-1))
    return np.concatenate(pieces).astype(np.float32, copy=False)


def unpack_matrix(packed: np.ndarray, in_features: int, out_features: int) -> np.ndarray:
    """Inverse of :func:`pack_matrix`: packed flat layout -> ``W[out][in]``."""
    packed = np.asarray(packed, dtype=np.float32).reshape(-1)
    full = (out_features // 32) * 32
    weight = np.empty((out_features, in_features), dtype=np.float32)
    cursor = 0
    for tile in range(0, full, 32):
        block = packed[cursor:cursor + in_features * 32].reshape(in_features, 32)
        weight[tile:tile + 32] = block.T
        cursor += in_features * 32
    tail = out_features - full
    if tail:
        block = packed[cursor:cursor + in_features * tail].reshape(in_features, tail)
        weight[full:] = block.T
        cursor += in_features * tail
    assert cursor == packed.size
    return weight


def tensor_plan():
    """Yield ``(label, in_features, out_features, kind)`` for every tensor in order.

    ``kind`` is ``"gamma"``, ``"bias"`` or ``"matrix"``; vectors have
    ``in_features`` None.
    """
    for layer in range(DEPTH):
        for axis in range(2):
            for name, fin, fout in TRANSFORMER_TENSORS:
                kind = "matrix" if fin is not None else ("gamma" if "gamma" in name else "bias")
                yield (f"layers.{layer}.{axis}.{name}", fin, fout, kind)
    for band in range(BANDS):
        d = BAND_DIMS[band]
        yield (f"bands.{band}.gamma", None, d, "gamma")
        yield (f"bands.{band}.weight", d, DIM, "matrix")
        yield (f"bands.{band}.bias", None, DIM, "bias")
    yield ("final_gamma", None, DIM, "gamma")
    for band in range(BANDS):
        d = BAND_DIMS[band]
        yield (f"masks.{band}.first_weight", DIM, FF_DIM, "matrix")
        yield (f"masks.{band}.first_bias", None, FF_DIM, "bias")
        yield (f"masks.{band}.second_weight", FF_DIM, 2 * d, "matrix")
        yield (f"masks.{band}.second_bias", None, 2 * d, "bias")


def header_bytes() -> bytes:
    fields = [1, DIM, DEPTH, BANDS, HEADS, DIM_HEAD, FREQ_BINS, CHANNELS, NFFT, HOP,
              WIN_LENGTH, MODEL_FRAMES, 0, 0]
    return MAGIC + struct.pack("<14I", *fields)


def synthetic_pack(seed: int = 0, weight_sigma: float = 0.02, gamma_sigma: float = 0.0,
                   bias_sigma: float = 0.0) -> bytes:
    """Seeded synthetic VSCNAT01 pack (numpy PCG64).

    Matrices ~ N(0, weight_sigma) (drawn logically and packed), gammas
    ``1 + N(0, gamma_sigma)``, biases ``N(0, bias_sigma)``.  The default is the
    benchmark recipe (gamma 1, biases 0); parity tests use nonzero gamma and
    bias spreads so that every tensor influences the output.
    """
    rng = np.random.default_rng(seed)
    chunks = [header_bytes()]
    for _label, fin, fout, kind in tensor_plan():
        if kind == "matrix":
            w = rng.standard_normal((fout, fin), dtype=np.float32) * np.float32(weight_sigma)
            values = pack_matrix(w)
        elif kind == "gamma":
            values = np.ones(fout, dtype=np.float32)
            if gamma_sigma:
                values += rng.standard_normal(fout, dtype=np.float32) * np.float32(gamma_sigma)
        else:
            values = np.zeros(fout, dtype=np.float32)
            if bias_sigma:
                values += rng.standard_normal(fout, dtype=np.float32) * np.float32(bias_sigma)
        chunks.append(struct.pack("<Q", values.size))
        chunks.append(values.astype("<f4", copy=False).tobytes())
    blob = b"".join(chunks)
    assert len(blob) == PACK_BYTES, len(blob)
    return blob


#: Recipe used by parity tests: nonzero gamma/bias spread, weights N(0, 0.02).
TEST_RECIPE = dict(seed=7, weight_sigma=0.02, gamma_sigma=0.1, bias_sigma=0.02)
#: Recipe used by the benchmark (gamma 1, biases 0, weights N(0, 0.02), seed 0).
BENCH_RECIPE = dict(seed=0, weight_sigma=0.02, gamma_sigma=0.0, bias_sigma=0.0)


def pack_path(recipe: dict, directory: str | None = None) -> str:
    """Write (once) the pack for ``recipe`` to a cache file and return its path."""
    directory = directory or os.environ.get("VOCALARC_B200_CACHE") or os.path.join(
        tempfile.gettempdir(), "vocalarc_b200_cache")
    os.makedirs(directory, exist_ok=True)
    name = "pack-" + "-".join(f"{k}{recipe[k]}" for k in sorted(recipe)) + ".f32"
    path = os.path.join(directory, name)
    if not os.path.exists(path) or os.path.getsize(path) != PACK_BYTES:
        blob = synthetic_pack(**recipe)
        tmp = path + f".tmp{os.getpid()}"
        with open(tmp, "wb") as handle:
            handle.write(blob)
        os.replace(tmp, path)
    return path


@dataclass
class Model:
    """Parsed pack with logical (unpacked) ``W[out][in]`` matrices, all float32."""

    layers: list = field(default_factory=list)   # [DEPTH][2] dicts
    bands: list = field(default_factory=list)    # [BANDS] dicts gamma/weight/bias
    final_gamma: np.ndarray | None = None
    masks: list = field(default_factory=list)    # [BANDS] dicts


def parse_pack(blob: bytes) -> Model:
    """Parse a VSCNAT01 blob following ``model_parse`` (vocalarc_separation.c:528)."""
    if len(blob) < 64 or blob[:8] != MAGIC:
        raise ValueError("not a VSCNAT01 pack")
    fields = struct.unpack_from("<14I", blob, 8)
    expected = (1, DIM, DEPTH, BANDS, HEADS, DIM_HEAD, FREQ_BINS, CHANNELS, NFFT, HOP,
                WIN_LENGTH, MODEL_FRAMES)
    if tuple(fields[:12]) != expected:
        raise ValueError("unsupported native model header")
    cursor = 64
    model = Model()
    model.layers = [[{}, {}] for _ in range(DEPTH)]
    model.bands = [{} for _ in range(BANDS)]
    model.masks = [{} for _ in range(BANDS)]
    for label, fin, fout, kind in tensor_plan():
        (count,) = struct.unpack_from("<Q", blob, cursor)
        cursor += 8
        need = fout if fin is None else fin * fout
        if count != need:
            raise ValueError(f"tensor mismatch for {label}: {count} != {need}")
        values = np.frombuffer(blob, dtype="<f4", count=count, offset=cursor).astype(np.float32)
        cursor += 4 * count
        if fin is not None:
            values = unpack_matrix(values, fin, fout)
        parts = label.split(".")
        if parts[0] == "layers":
            model.layers[int(parts[1])][int(parts[2])][parts[3]] = values
        elif parts[0] == "bands":
            model.bands[int(parts[1])][parts[2]] = values
        elif parts[0] == "masks":
            model.masks[int(parts[1])][parts[2]] = values
        else:
            model.final_gamma = values
    if cursor != len(blob):
        raise ValueError(f"{len(blob) - cursor} trailing bytes")
    return model
