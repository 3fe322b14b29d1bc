"""Configurable BS-RoFormer stack: configurations, weight layout and the ctypes binding.

The library's ``vocalarc_b200_stack_*`` entry points (``include/vocalarc_b200_stack.h``)
run the bundled model's forward with its sizes as parameters.  Two
configurations matter here:

* :data:`CONFIG3` -- the layer-level tensor-core benchmark model: dim 512,
  depth 12, 8 heads x 64, GEGLU FFN with mult 4, 62 bands over the 1025 STFT
  bins, n_fft 2048, hop 441 (8 s clips = 801 frames), bf16 operands.  The 62
  band widths are BS-RoFormer's published default split (24 x 2, 12 x 4,
  8 x 12, 8 x 24, 8 x 48, 128, 129 bins).
* :data:`BUNDLED` -- the reference's own sizes (vocalarc_separation.c:33-57),
  used to cross-check the stack against the bundled-model path.

The weight array is float32, every matrix logical ``W[out][in]``, in the
order of :func:`weight_plan` (the VSCNAT01 order of ``model_parse``,
vocalarc_separation.c:528-589, without the count prefixes or the 32-lane
packing).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import modelpack as mp
from .native import ProviderError, dptr, fptr, load

MAX_BANDS = 128
BSROFORMER_62_BANDS = (2,) * 24 + (4,) * 12 + (12,) * 8 + (24,) * 8 + (48,) * 8 + (128, 129)
assert len(BSROFORMER_62_BANDS) == 62 and sum(BSROFORMER_62_BANDS) == mp.FREQ_BINS


@dataclass(frozen=True)
class StackConfig:
    dim: int
    depth: int
    ff_inner: int
    geglu: bool
    mask_hidden: int
    band_bins: tuple
    hop: int
    bf16: bool
    heads: int = mp.HEADS
    dim_head: int = mp.DIM_HEAD
    n_fft: int = mp.NFFT

    @property
    def bands(self) -> int:
        return len(self.band_bins)

    @property
    def band_dims(self) -> tuple:
        return tuple(4 * w for w in self.band_bins)

    @property
    def band_first(self) -> tuple:
        return tuple(int(x) for x in np.concatenate([[0], np.cumsum(self.band_bins)[:-1]]))

    @property
    def ff1_rows(self) -> int:
        return self.ff_inner * (2 if self.geglu else 1)

    def frames(self, length: int) -> int:
        return length // self.hop + 1

    def replace(self, **changes) -> "StackConfig":
        values = {k: getattr(self, k) for k in self.__dataclass_fields__}
        values.update(changes)
        return StackConfig(**values)


CONFIG3 = StackConfig(dim=512, depth=12, ff_inner=2048, geglu=True, mask_hidden=2048,
                      band_bins=BSROFORMER_62_BANDS, hop=441, bf16=True)
BUNDLED = StackConfig(dim=mp.DIM, depth=mp.DEPTH, ff_inner=mp.FF_DIM, geglu=False, mask_hidden=mp.FF_DIM,
                      band_bins=mp.BAND_FREQS, hop=mp.HOP, bf16=False)

#: Config 3's clip: 8 s at 44.1 kHz (801 frames at hop 441), 16 clips per batch.
CONFIG3_CLIP = 8 * mp.SAMPLE_RATE
CONFIG3_CLIPS = 16


def weight_plan(cfg: StackConfig):
    """Yield ``(label, shape, kind)`` of every tensor in array order (kind: matrix, gamma, bias)."""
    d, inner = cfg.dim, cfg.heads * cfg.dim_head
    for layer in range(cfg.depth):
        for axis in range(2):
            p = f"layers.{layer}.{axis}."
            yield p + "gamma", (d,), "gamma"
            yield p + "qkv", (3 * inner, d), "matrix"
            yield p + "gate_weight", (cfg.heads, d), "matrix"
            yield p + "gate_bias", (cfg.heads,), "bias"
            yield p + "out_weight", (d, inner), "matrix"
            yield p + "ff_gamma", (d,), "gamma"
            yield p + "ff1_weight", (cfg.ff1_rows, d), "matrix"
            yield p + "ff1_bias", (cfg.ff1_rows,), "bias"
            yield p + "ff2_weight", (d, cfg.ff_inner), "matrix"
            yield p + "ff2_bias", (d,), "bias"
    for band, db in enumerate(cfg.band_dims):
        yield f"bands.{band}.gamma", (db,), "gamma"
        yield f"bands.{band}.weight", (d, db), "matrix"
        yield f"bands.{band}.bias", (d,), "bias"
    yield "final_gamma", (d,), "gamma"
    for band, db in enumerate(cfg.band_dims):
        yield f"masks.{band}.first_weight", (cfg.mask_hidden, d), "matrix"
        yield f"masks.{band}.first_bias", (cfg.mask_hidden,), "bias"
        yield f"masks.{band}.second_weight", (2 * db, cfg.mask_hidden), "matrix"
        yield f"masks.{band}.second_bias", (2 * db,), "bias"


def weight_count(cfg: StackConfig) -> int:
    return sum(int(np.prod(shape)) for _l, shape, _k in weight_plan(cfg))


def synthetic_weights(cfg: StackConfig, seed: int = 2, weight_sigma: float = 0.02, gamma_sigma: float = 0.0,
                      bias_sigma: float = 0.0) -> np.ndarray:
    """Seeded weights (numpy PCG64): matrices N(0, weight_sigma), gammas 1 + N(0, gamma_sigma), biases N(0, bias_sigma)."""
    rng = np.random.default_rng(seed)
    flat = np.empty(weight_count(cfg), dtype=np.float32)
    cursor = 0
    for _label, shape, kind in weight_plan(cfg):
        n = int(np.prod(shape))
        view = flat[cursor:cursor + n]
        if kind == "matrix":
            rng.standard_normal(n, dtype=np.float32, out=view)
            view *= np.float32(weight_sigma)
        elif kind == "gamma":
            if gamma_sigma:
                rng.standard_normal(n, dtype=np.float32, out=view)
                view *= np.float32(gamma_sigma)
                view += np.float32(1.0)
            else:
                view.fill(1.0)
        else:
            if bias_sigma:
                rng.standard_normal(n, dtype=np.float32, out=view)
                view *= np.float32(bias_sigma)
            else:
                view.fill(0.0)
        cursor += n
    return flat


def split_weights(cfg: StackConfig, flat: np.ndarray) -> dict:
    """Views of the flat array by label (``{label: ndarray}``)."""
    out, cursor = {}, 0
    for label, shape, _kind in weight_plan(cfg):
        n = int(np.prod(shape))
        out[label] = flat[cursor:cursor + n].reshape(shape)
        cursor += n
    if cursor != flat.size:
        raise ValueError(f"weight array has {flat.size} floats, the configuration needs {cursor}")
    return out


def weights_from_model(model: mp.Model) -> np.ndarray:
    """The flat :data:`BUNDLED` weight array of a parsed VSCNAT01 pack."""
    names = {"gamma": "gamma", "qkv": "qkv", "gate_weight": "gate_weight", "gate_bias": "gate_bias",
             "out_weight": "out_weight", "ff_gamma": "ff_gamma", "ff1_weight": "ff1_weight",
             "ff1_bias": "ff1_bias", "ff2_weight": "ff2_weight", "ff2_bias": "ff2_bias"}
    parts = []
    for label, shape, _kind in weight_plan(BUNDLED):
        p = label.split(".")
        if p[0] == "layers":
            value = model.layers[int(p[1])][int(p[2])][names[p[3]]]
        elif p[0] == "bands":
            value = model.bands[int(p[1])][p[2]]
        elif p[0] == "masks":
            value = model.masks[int(p[1])][p[2]]
        else:
            value = model.final_gamma
        parts.append(np.asarray(value, dtype=np.float32).reshape(shape).reshape(-1))
    return np.concatenate(parts)


# ------------------------------------------------------------------ ctypes binding
class StackConfigC(ctypes.Structure):
    """``vocalarc_b200_stack_config`` (include/vocalarc_b200_stack.h)."""

    _fields_ = [("dim", ctypes.c_int), ("depth", ctypes.c_int), ("heads", ctypes.c_int),
                ("dim_head", ctypes.c_int), ("ff_inner", ctypes.c_int), ("geglu", ctypes.c_int),
                ("mask_hidden", ctypes.c_int), ("bands", ctypes.c_int), ("band_bins", ctypes.c_int * MAX_BANDS),
                ("n_fft", ctypes.c_int), ("hop", ctypes.c_int), ("bf16", ctypes.c_int)]

    @classmethod
    def of(cls, cfg: StackConfig) -> "StackConfigC":
        if not 1 <= cfg.bands <= MAX_BANDS:
            raise ValueError(f"{cfg.bands} bands; the library takes 1..{MAX_BANDS}")
        c = cls()
        c.dim, c.depth, c.heads, c.dim_head = cfg.dim, cfg.depth, cfg.heads, cfg.dim_head
        c.ff_inner, c.geglu, c.mask_hidden, c.bands = cfg.ff_inner, int(cfg.geglu), cfg.mask_hidden, cfg.bands
        for i, w in enumerate(cfg.band_bins):
            c.band_bins[i] = w
        c.n_fft, c.hop, c.bf16 = cfg.n_fft, cfg.hop, int(cfg.bf16)
        return c


_vp = ctypes.c_void_p
_cfgp = ctypes.POINTER(StackConfigC)
STACK_SIGNATURES = {
    "vocalarc_b200_stack_weight_count": (ctypes.c_size_t, [_cfgp]),
    "vocalarc_b200_stack_create": (_vp, [ctypes.c_int, _cfgp, ctypes.POINTER(ctypes.c_float), ctypes.c_size_t]),
    "vocalarc_b200_stack_destroy": (None, [_vp]),
    "vocalarc_b200_stack_forward_device": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp]),
    "vocalarc_b200_stack_separate": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_float), ctypes.c_int, ctypes.c_int,
                                                    ctypes.POINTER(ctypes.c_float)]),
    "vocalarc_b200_stack_stage_stft": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp]),
    "vocalarc_b200_stack_stage_band_split": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp]),
    "vocalarc_b200_stack_stage_block": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                       ctypes.c_int]),
    "vocalarc_b200_stack_stage_mask": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp]),
    "vocalarc_b200_stack_stage_istft": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp]),
    "vocalarc_b200_stack_synchronize": (ctypes.c_int, [_vp]),
    "vocalarc_b200_stack_stream": (_vp, [_vp]),
    "vocalarc_b200_stack_take_device_error": (ctypes.c_int, [_vp]),
    "vocalarc_b200_stack_launch_count": (ctypes.c_longlong, [_vp]),
    "vocalarc_b200_stack_trace_begin": (ctypes.c_int, [_vp]),
    "vocalarc_b200_stack_trace_end": (ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.c_int]),
}


def bind(lib=None):
    lib = lib or load()
    for name, (restype, argtypes) in STACK_SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


def library_weight_count(cfg: StackConfig) -> int:
    """The library's own count for ``cfg`` (0 = configuration rejected)."""
    lib = bind()
    c = StackConfigC.of(cfg)
    return int(lib.vocalarc_b200_stack_weight_count(ctypes.byref(c)))


class Stack:
    """One ``vocalarc_b200_stack`` on a CUDA device."""

    def __init__(self, cfg: StackConfig, weights: np.ndarray, device: int = 0):
        self.lib = bind()
        self.cfg = cfg
        weights = np.ascontiguousarray(weights, dtype=np.float32)
        c = StackConfigC.of(cfg)
        self.handle = self.lib.vocalarc_b200_stack_create(device, ctypes.byref(c), fptr(weights), weights.size)
        if not self.handle:
            raise ProviderError("vocalarc_b200_stack_create failed")

    def close(self):
        if self.handle:
            self.lib.vocalarc_b200_stack_destroy(self.handle)
            self.handle = None

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass

    def check(self, ok: int, what: str):
        if not ok:
            raise ProviderError(f"{what} failed (device error {self.lib.vocalarc_b200_stack_take_device_error(self.handle)})")

    @property
    def stream(self) -> int:
        return self.lib.vocalarc_b200_stack_stream(self.handle) or 0

    @property
    def launch_count(self) -> int:
        return int(self.lib.vocalarc_b200_stack_launch_count(self.handle))

    def synchronize(self):
        self.check(self.lib.vocalarc_b200_stack_synchronize(self.handle), "stack synchronize")

    def separate(self, audio: np.ndarray) -> np.ndarray:
        """Host ``[clips][2][length]`` (or ``[2][length]``) -> vocals of the same shape."""
        audio = np.ascontiguousarray(audio, dtype=np.float32)
        batch = audio if audio.ndim == 3 else audio[None]
        out = np.zeros_like(batch)
        self.check(self.lib.vocalarc_b200_stack_separate(self.handle, fptr(batch), batch.shape[0], batch.shape[2],
                                                         fptr(out)), "stack separate")
        return out if audio.ndim == 3 else out[0]

    def forward_device(self, d_audio, clips: int, length: int, d_vocals):
        self.check(self.lib.vocalarc_b200_stack_forward_device(self.handle, dptr(d_audio), clips, length,
                                                               dptr(d_vocals)), "stack forward")

    def stage_stft(self, d_audio, clips: int, length: int, d_spec):
        self.check(self.lib.vocalarc_b200_stack_stage_stft(self.handle, dptr(d_audio), clips, length, dptr(d_spec)),
                   "stack stft")

    def stage_band_split(self, d_spec, clips: int, frames: int, d_x):
        self.check(self.lib.vocalarc_b200_stack_stage_band_split(self.handle, dptr(d_spec), clips, frames, dptr(d_x)),
                   "stack band split")

    def stage_block(self, d_x, clips: int, frames: int, layer: int, axis: int):
        self.check(self.lib.vocalarc_b200_stack_stage_block(self.handle, dptr(d_x), clips, frames, layer, axis),
                   "stack block")

    def stage_mask(self, d_x, clips: int, frames: int, d_mask):
        self.check(self.lib.vocalarc_b200_stack_stage_mask(self.handle, dptr(d_x), clips, frames, dptr(d_mask)),
                   "stack mask")

    def stage_istft(self, d_spec, d_mask, clips: int, length: int, d_audio):
        self.check(self.lib.vocalarc_b200_stack_stage_istft(self.handle, dptr(d_spec), dptr(d_mask), clips, length,
                                                            dptr(d_audio)), "stack istft")

    def trace_begin(self):
        self.check(self.lib.vocalarc_b200_stack_trace_begin(self.handle), "stack trace_begin")

    def trace_end(self) -> dict:
        buf = ctypes.create_string_buffer(1 << 16)
        self.check(self.lib.vocalarc_b200_stack_trace_end(self.handle, buf, len(buf)), "stack trace_end")
        out = {}
        for line in buf.value.decode().splitlines():
            name, count, ms = line.split("\t")
            out[name] = (int(count), float(ms))
        return out


def forward_flops(cfg: StackConfig, clips: int, frames: int) -> dict:
    """Algorithmic FLOPs of one forward by kernel class (multiply-add = 2)."""
    tokens = clips * cfg.bands * frames
    inner = cfg.heads * cfg.dim_head
    d = cfg.dim
    per_block = {
        "qkv gemm": 2 * tokens * d * (3 * inner + cfg.heads),
        "out gemm": 2 * tokens * inner * d,
        "ff1 gemm": 2 * tokens * d * cfg.ff1_rows,
        "ff2 gemm": 2 * tokens * cfg.ff_inner * d,
    }
    if d == 256 and cfg.ff1_rows == cfg.ff_inner and cfg.ff_inner % 128 == 0:
        # One fused launch (FF1, GELU and FF2 with the hidden on chip).
        per_block["ffn"] = per_block.pop("ff1 gemm") + per_block.pop("ff2 gemm")
    out = {k: v * 2 * cfg.depth for k, v in per_block.items()}
    out["attention (L>128)"] = cfg.depth * 4 * inner * clips * cfg.bands * frames * frames
    out["attention (L<=128)"] = cfg.depth * 4 * inner * clips * frames * cfg.bands * cfg.bands
    split = sum(cfg.band_dims)
    out["band split"] = 2 * clips * frames * split * d
    out["mask gemm 1"] = 2 * tokens * d * cfg.mask_hidden
    out["mask gemm 2"] = 2 * clips * frames * cfg.mask_hidden * 2 * split
    return out
