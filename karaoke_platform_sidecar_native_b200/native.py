"""ctypes binding of libvocalarc_b200.so (the sm_100a provider).

The library exposes the reference's provider ABI (``native_gpu.h``; the host
``native/vocalarc_separation.c`` links it unchanged) and the additive
``vocalarc_b200.h`` extension.  This module is a thin Python mirror of both,
used by the tests and ``bench.py``.  There is no fallback: when the library is
missing or no sm_100 device is present the calls fail loudly.
"""

from __future__ import annotations

import ctypes
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "libvocalarc_b200.so")
HEADERS = (os.path.join(ROOT, "include", "native_gpu.h"), os.path.join(ROOT, "include", "vocalarc_b200.h"),
           os.path.join(ROOT, "include", "vocalarc_b200_stack.h"))

_f32p = ctypes.POINTER(ctypes.c_float)
_vp = ctypes.c_void_p
_ip = ctypes.POINTER(ctypes.c_int)


class TransformerWeights(ctypes.Structure):
    """``native_gpu_transformer_weights`` (native_gpu.h:30-41)."""

    _fields_ = [(name, _f32p) for name in (
        "gamma", "qkv", "gate_weight", "gate_bias", "out_weight", "ff_gamma",
        "ff1_weight", "ff1_bias", "ff2_weight", "ff2_bias")]


class MaskBand(ctypes.Structure):
    """``native_gpu_mask_band`` (native_gpu.h:60-67)."""

    _fields_ = [("first_weight", _f32p), ("first_bias", _f32p), ("second_weight", _f32p),
                ("second_bias", _f32p), ("input_dim", ctypes.c_int), ("first_frequency", ctypes.c_int)]


_SIGNATURES = {
    "native_gpu_create": (_vp, []),
    "native_gpu_destroy": (None, [_vp]),
    "native_gpu_matmul": (ctypes.c_int, [_vp, ctypes.c_int64, ctypes.c_int, ctypes.c_int, _f32p, _f32p, _f32p, _f32p]),
    "native_gpu_backend": (ctypes.c_char_p, [_vp]),
    "native_gpu_device": (ctypes.c_char_p, [_vp]),
    "native_gpu_uses_full_batches": (ctypes.c_int, [_vp]),
    "native_gpu_can_use_full_batches": (ctypes.c_int, [_vp, ctypes.c_int]),
    "native_gpu_transformer": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _f32p, _f32p, _f32p, _f32p, _f32p,
                                              ctypes.POINTER(TransformerWeights)]),
    "native_gpu_resident_begin": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _f32p]),
    "native_gpu_resident_transformer": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int,
                                                       ctypes.POINTER(TransformerWeights)]),
    "native_gpu_resident_transpose": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int]),
    "native_gpu_resident_end": (ctypes.c_int, [_vp, _f32p]),
    "native_gpu_resident_mask": (ctypes.c_int, [_vp, ctypes.c_int, _f32p, _f32p, ctypes.POINTER(MaskBand),
                                                ctypes.c_int]),
    "vocalarc_b200_create": (_vp, [ctypes.c_int]),
    "vocalarc_b200_load_model": (ctypes.c_int, [_vp, ctypes.c_void_p, ctypes.c_size_t]),
    "vocalarc_b200_load_model_file": (ctypes.c_int, [_vp, ctypes.c_char_p]),
    "vocalarc_b200_model_from_cache": (ctypes.c_int, [_vp]),
    "vocalarc_b200_model_image": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int,
                                                 ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    "vocalarc_b200_store_model_image": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                                       ctypes.c_char_p, ctypes.c_int]),
    "vocalarc_b200_separate": (ctypes.c_int, [_vp, _f32p, ctypes.c_int, _f32p]),
    "vocalarc_b200_separate_chunked": (ctypes.c_int, [_vp, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p]),
    "vocalarc_b200_separate_device": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                     ctypes.c_int, ctypes.c_int, _vp]),
    "vocalarc_b200_synchronize": (ctypes.c_int, [_vp]),
    "vocalarc_b200_separate_sp": (ctypes.c_int, [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, _f32p, ctypes.c_int,
                                                 _f32p]),
    "vocalarc_b200_sp_plan": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             ctypes.POINTER(ctypes.c_longlong), ctypes.c_int]),
    "vocalarc_b200_stream": (_vp, [_vp]),
    "vocalarc_b200_take_device_error": (ctypes.c_int, [_vp]),
    "vocalarc_b200_set_precision": (ctypes.c_int, [_vp, ctypes.c_int]),
    "vocalarc_b200_launch_count": (ctypes.c_longlong, [_vp]),
    "vocalarc_b200_trace_begin": (ctypes.c_int, [_vp]),
    "vocalarc_b200_trace_mark": (ctypes.c_int, [_vp, ctypes.c_char_p]),
    "vocalarc_b200_trace_end": (ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.c_int]),
    "vocalarc_b200_stage_gemm": (ctypes.c_int, [_vp, ctypes.c_int, _vp, _vp, ctypes.c_int, ctypes.c_int,
                                                ctypes.c_int, _vp, _vp]),
    "vocalarc_b200_separate_tta": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                  ctypes.c_int, _vp]),
    "vocalarc_b200_chunk_plan": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, _ip, _ip, _ip, _ip]),
    "vocalarc_b200_range_forward": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                   ctypes.c_int]),
    "vocalarc_b200_range_owned": (ctypes.c_int, [_vp, _ip, _ip]),
    "vocalarc_b200_range_seam_export": (ctypes.c_int, [_vp, _vp]),
    "vocalarc_b200_range_seam_import": (ctypes.c_int, [_vp, _vp]),
    "vocalarc_b200_range_seam_from": (ctypes.c_int, [_vp, _vp]),
    "vocalarc_b200_range_finish": (ctypes.c_int, [_vp, _vp]),
    "vocalarc_b200_stage_attention": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                     ctypes.c_int]),
    "vocalarc_b200_stage_stft": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp]),
    "vocalarc_b200_stage_istft": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp]),
    "vocalarc_b200_stage_istft_noalloc": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp]),
    "vocalarc_b200_stage_wait_check": (ctypes.c_int, [_vp, ctypes.c_int]),
    "vocalarc_b200_separate_files": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.POINTER(ctypes.c_char_p),
                                                    ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_char_p),
                                                    ctypes.c_int]),
    "vocalarc_b200_read_track": (ctypes.c_int, [ctypes.c_char_p, _f32p, ctypes.c_longlong,
                                                ctypes.POINTER(ctypes.c_int)]),
    "vocalarc_b200_write_track": (ctypes.c_int, [ctypes.c_char_p, _f32p, ctypes.c_int]),
    "vocalarc_b200_stage_band_split": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp]),
    "vocalarc_b200_stage_block": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "vocalarc_b200_stage_mask": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp]),
}

_LIB = None


def chunk_plan(length: int, chunk: int = 0) -> dict:
    """Chunk plan of vocalarc_b200_separate_chunked (chunks, step, border, seam)."""
    lib = load()
    vals = [ctypes.c_int(0) for _ in range(4)]
    if not lib.vocalarc_b200_chunk_plan(length, chunk, *[ctypes.byref(v) for v in vals]):
        raise ProviderError(f"chunk_plan({length}, {chunk}) failed")
    return dict(zip(("chunks", "step", "border", "seam"), (v.value for v in vals)))


def read_track(path: str) -> np.ndarray:
    """The batch reader stage: a WAV decoded to planar stereo float32 at 44.1 kHz (no GPU)."""
    lib = load()
    n = ctypes.c_int(0)
    if not lib.vocalarc_b200_read_track(os.fsencode(path), None, 0, ctypes.byref(n)):
        raise ProviderError(f"cannot read {path}")
    out = np.zeros((2, n.value), dtype=np.float32)
    if not lib.vocalarc_b200_read_track(os.fsencode(path), fptr(out), out.size, ctypes.byref(n)):
        raise ProviderError(f"cannot read {path}")
    return out


def write_track(path: str, audio: np.ndarray) -> None:
    """The batch writer stage: float32 stereo 44.1 kHz WAV, non-finite samples as 0 (no GPU)."""
    audio = np.ascontiguousarray(audio, dtype=np.float32)
    if not load().vocalarc_b200_write_track(os.fsencode(path), fptr(audio), audio.shape[1]):
        raise ProviderError(f"cannot write {path}")


def sp_plan(count: int, frames: int, phase: int) -> np.ndarray:
    """Copies of one sequence-parallel exchange: rows of (src, dst, src_row, src_pitch,
    dst_row, dst_pitch, width, height), in token rows."""
    lib = load()
    n = lib.vocalarc_b200_sp_plan(count, frames, phase, None, 0)
    if n < 0:
        raise ProviderError(f"sp_plan({count}, {frames}, {phase}) rejected")
    out = np.zeros((max(n, 1), 8), dtype=np.int64)
    lib.vocalarc_b200_sp_plan(count, frames, phase, out.ctypes.data_as(ctypes.POINTER(ctypes.c_longlong)), n)
    return out[:n]


def separate_sp(providers: list, audio: np.ndarray) -> np.ndarray:
    """One clip's whole-clip forward split across the providers (one per GPU)."""
    lib = load()
    audio = np.ascontiguousarray(audio, dtype=np.float32)
    out = np.zeros_like(audio)
    handles = (ctypes.c_void_p * len(providers))(*[p.handle for p in providers])
    if not lib.vocalarc_b200_separate_sp(handles, len(providers), fptr(audio), audio.shape[1], fptr(out)):
        raise ProviderError("vocalarc_b200_separate_sp failed")
    return out


def model_image(blob: bytes, bf16: bool = False, threads: int = 0) -> np.ndarray:
    """The converted device image of a VSCNAT01 pack, built on the host (no GPU)."""
    lib = load()
    size = ctypes.c_size_t(0)
    lib.vocalarc_b200_model_image(None, 0, 0, 0, None, 0, ctypes.byref(size))
    out = np.zeros(size.value, dtype=np.uint8)
    ok = lib.vocalarc_b200_model_image(blob, len(blob), int(bf16), threads, out.ctypes.data_as(ctypes.c_void_p),
                                       out.size, ctypes.byref(size))
    if not ok:
        raise ProviderError("vocalarc_b200_model_image failed")
    return out


def store_model_image(blob: bytes, bf16: bool = False) -> str:
    """Convert a pack and write its image to the cache directory (no GPU); returns the file."""
    lib = load()
    path = ctypes.create_string_buffer(4096)
    if not lib.vocalarc_b200_store_model_image(blob, len(blob), int(bf16), path, len(path)):
        raise ProviderError("vocalarc_b200_store_model_image failed")
    return path.value.decode()


def declared_functions() -> list:
    """Every function name declared in include/*.h."""
    names = []
    for path in HEADERS:
        text = open(path).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"\b((?:native_gpu|vocalarc_b200)_\w+)\s*\(", text)
    return sorted(set(names))


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the provider library; raises when it has not been built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: run python -m karaoke_platform_sidecar_native_b200.build")
    lib = ctypes.CDLL(path)
    for name, (restype, argtypes) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _LIB = lib
    return lib


def fptr(array: np.ndarray):
    assert array.dtype == np.float32 and array.flags["C_CONTIGUOUS"]
    return array.ctypes.data_as(_f32p)


def dptr(tensor) -> int:
    """Raw device pointer of a torch tensor (plumbing only)."""
    return ctypes.c_void_p(tensor.data_ptr())


class ProviderError(RuntimeError):
    pass


class Provider:
    """One ``native_gpu`` context bound to a CUDA device."""

    def __init__(self, device: int = 0):
        self.lib = load()
        self.handle = self.lib.vocalarc_b200_create(device)
        if not self.handle:
            raise ProviderError(f"vocalarc_b200_create({device}) failed: no sm_100 device")
        self._keep = []

    # ---- reference ABI -------------------------------------------------
    @property
    def backend(self) -> str:
        return self.lib.native_gpu_backend(self.handle).decode()

    @property
    def device_name(self) -> str:
        return self.lib.native_gpu_device(self.handle).decode()

    def close(self):
        if self.handle:
            self.lib.native_gpu_destroy(self.handle)
            self.handle = None

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass

    def check(self, ok: int, what: str):
        if not ok:
            raise ProviderError(f"{what} failed (device error {self.lib.vocalarc_b200_take_device_error(self.handle)})")

    # ---- extension -----------------------------------------------------
    def load_model(self, blob: bytes):
        # A bytes object is passed as a pointer to its own buffer (no copy).
        self.check(self.lib.vocalarc_b200_load_model(self.handle, bytes(blob), len(blob)), "load_model")

    def load_model_file(self, path: str):
        self.check(self.lib.vocalarc_b200_load_model_file(self.handle, os.fsencode(path)), "load_model_file")

    @property
    def model_from_cache(self) -> bool:
        return bool(self.lib.vocalarc_b200_model_from_cache(self.handle))

    def set_precision(self, bf16: bool):
        self.check(self.lib.vocalarc_b200_set_precision(self.handle, 1 if bf16 else 0), "set_precision")

    def separate(self, audio: np.ndarray) -> np.ndarray:
        audio = np.ascontiguousarray(audio, dtype=np.float32)
        out = np.zeros_like(audio)
        self.check(self.lib.vocalarc_b200_separate(self.handle, fptr(audio), audio.shape[1], fptr(out)), "separate")
        return out

    def separate_chunked(self, audio: np.ndarray, chunk: int = 0, model_batch: int = 1) -> np.ndarray:
        audio = np.ascontiguousarray(audio, dtype=np.float32)
        out = np.zeros_like(audio)
        self.check(self.lib.vocalarc_b200_separate_chunked(self.handle, fptr(audio), audio.shape[1], chunk,
                                                           model_batch, fptr(out)), "separate_chunked")
        return out

    def separate_tta(self, audio: np.ndarray, bigshifts: int = 2, tta: bool = True, chunk: int = 0,
                     model_batch: int = 1) -> np.ndarray:
        """The ONNX sidecar's bigshift + TTA pass over the chunked forward."""
        audio = np.ascontiguousarray(audio, dtype=np.float32)
        out = np.zeros_like(audio)
        self.check(self.lib.vocalarc_b200_separate_tta(self.handle, fptr(audio), audio.shape[1], chunk, model_batch,
                                                       bigshifts, 1 if tta else 0, fptr(out)), "separate_tta")
        return out

    def separate_device(self, d_audio, tracks: int, length: int, d_vocals, chunked: bool = False, chunk: int = 0,
                        model_batch: int = 1):
        self.check(self.lib.vocalarc_b200_separate_device(self.handle, dptr(d_audio), tracks, length,
                                                          1 if chunked else 0, chunk, model_batch,
                                                          dptr(d_vocals)), "separate_device")

    def synchronize(self):
        self.check(self.lib.vocalarc_b200_synchronize(self.handle), "synchronize")

    @property
    def stream(self) -> int:
        return self.lib.vocalarc_b200_stream(self.handle) or 0

    def take_device_error(self) -> int:
        return self.lib.vocalarc_b200_take_device_error(self.handle)

    @property
    def launch_count(self) -> int:
        return int(self.lib.vocalarc_b200_launch_count(self.handle))

    def trace_begin(self):
        self.check(self.lib.vocalarc_b200_trace_begin(self.handle), "trace_begin")

    def trace_mark(self, what: str):
        self.lib.vocalarc_b200_trace_mark(self.handle, what.encode())

    def trace_end(self) -> dict:
        buf = ctypes.create_string_buffer(1 << 16)
        self.check(self.lib.vocalarc_b200_trace_end(self.handle, buf, len(buf)), "trace_end")
        out = {}
        for line in buf.value.decode().splitlines():
            name, count, ms = line.split("\t")
            out[name] = (int(count), float(ms))
        return out

    # ---- one track's chunks sharded across providers (chunk ranges) -----
    def range_forward(self, d_audio, length: int, chunk_begin: int, chunk_end: int, chunk: int = 0,
                      model_batch: int = 1):
        self.check(self.lib.vocalarc_b200_range_forward(self.handle, dptr(d_audio), length, chunk, model_batch,
                                                        chunk_begin, chunk_end), "range_forward")

    def range_owned(self) -> tuple:
        s0, s1 = ctypes.c_int(0), ctypes.c_int(0)
        self.check(self.lib.vocalarc_b200_range_owned(self.handle, ctypes.byref(s0), ctypes.byref(s1)), "range_owned")
        return s0.value, s1.value

    def range_seam_export(self) -> bytes:
        buf = ctypes.create_string_buffer(64)
        self.check(self.lib.vocalarc_b200_range_seam_export(self.handle, buf), "range_seam_export")
        return buf.raw

    def range_seam_import(self, handle: bytes):
        buf = ctypes.create_string_buffer(bytes(handle), 64)
        self.check(self.lib.vocalarc_b200_range_seam_import(self.handle, buf), "range_seam_import")

    def range_seam_from(self, prev: "Provider"):
        self.check(self.lib.vocalarc_b200_range_seam_from(self.handle, prev.handle), "range_seam_from")

    def range_finish(self, d_vocals):
        self.check(self.lib.vocalarc_b200_range_finish(self.handle, dptr(d_vocals)), "range_finish")

    # ---- stages (device pointers) --------------------------------------
    def stage_gemm(self, epilogue, a, b, m, n, k, bias, out):
        self.check(self.lib.vocalarc_b200_stage_gemm(self.handle, epilogue, dptr(a), dptr(b), m, n, k,
                                                     dptr(bias) if bias is not None else None, dptr(out)),
                   "stage_gemm")

    def stage_attention(self, qkv, gates, out, d1, d2, d3, pos_dim):
        self.check(self.lib.vocalarc_b200_stage_attention(self.handle, dptr(qkv), dptr(gates), dptr(out), d1, d2,
                                                          d3, pos_dim), "stage_attention")

    def stage_stft(self, audio, segments, length, spec):
        self.check(self.lib.vocalarc_b200_stage_stft(self.handle, dptr(audio), segments, length, dptr(spec)),
                   "stage_stft")

    def stage_istft(self, spec, mask, segments, length, audio):
        self.check(self.lib.vocalarc_b200_stage_istft(self.handle, dptr(spec), dptr(mask), segments, length,
                                                      dptr(audio)), "stage_istft")

    def stage_istft_noalloc(self, spec, mask, segments, length, audio):
        self.check(self.lib.vocalarc_b200_stage_istft_noalloc(self.handle, dptr(spec), dptr(mask), segments, length,
                                                              dptr(audio)), "stage_istft_noalloc")

    def separate_files(self, inputs, vocals, instrumentals=None, chunked: bool = False) -> int:
        """Separate WAV files with the reader and writer stages running beside the device work."""
        n = len(inputs)
        arr = lambda paths: (ctypes.c_char_p * n)(*[os.fsencode(p) if p else None for p in paths])
        return int(self.lib.vocalarc_b200_separate_files(self.handle, n, arr(inputs), arr(vocals),
                                                         arr(instrumentals) if instrumentals else None,
                                                         1 if chunked else 0))

    def stage_wait_check(self, limit_us: int) -> int:
        """Run the bounded-wait check; returns the raw C-ABI result (0 = the wait ran out and was reported)."""
        return int(self.lib.vocalarc_b200_stage_wait_check(self.handle, limit_us))

    def stage_band_split(self, spec, segments, frames, x):
        self.check(self.lib.vocalarc_b200_stage_band_split(self.handle, dptr(spec), segments, frames, dptr(x)),
                   "stage_band_split")

    def stage_block(self, x, segments, frames, layer, axis):
        self.check(self.lib.vocalarc_b200_stage_block(self.handle, dptr(x), segments, frames, layer, axis),
                   "stage_block")

    def stage_mask(self, x, segments, frames, mask):
        self.check(self.lib.vocalarc_b200_stage_mask(self.handle, dptr(x), segments, frames, dptr(mask)),
                   "stage_mask")


def transformer_weights_from_blob(blob_array: np.ndarray, offsets: dict) -> TransformerWeights:
    """Build a ``native_gpu_transformer_weights`` pointing into a float32 view of a pack."""
    base = blob_array.ctypes.data
    w = TransformerWeights()
    for name in TransformerWeights._fields_:
        setattr(w, name[0], ctypes.cast(base + offsets[name[0]], _f32p))
    return w


def pack_offsets(blob: bytes) -> dict:
    """Byte offsets of every tensor's data in a VSCNAT01 blob (model_parse order)."""
    import struct

    from .modelpack import tensor_plan

    cursor = 64
    offsets = {}
    for label, _fin, _fout, _kind in tensor_plan():
        (count,) = struct.unpack_from("<Q", blob, cursor)
        offsets[label] = cursor + 8
        cursor += 8 + 4 * count
    return offsets
