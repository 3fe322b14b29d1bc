"""CPU oracle of the configurable BS-RoFormer stack (TEST INFRASTRUCTURE).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may
import this module; it is the checker, never the product.

The stack is the bundled model's forward (``forward_model``,
native/vocalarc_separation.c:1342-1445) with the sizes as parameters.  Every
operation here is a call into the reference-pinned restatement in
``vocalarc_oracle`` -- STFT / iSTFT (:1044-1136, with the frame step as a
parameter), RMSNorm (:419-424), Linear, RoPE (:692-744), softmax attention
(:753-800), head gates (:808-818), exact-erf GELU (:666-672), tanh and the GLU
mask scatter (:1316-1340) -- composed at the configuration's widths.  The one
operation the reference does not have is the GEGLU feed-forward: the first
Linear emits ``2 * ff_inner`` rows ``[value; gate]`` and ``h = value *
gelu(gate)`` (Shazeer, "GLU Variants Improve Transformer", 2020).

Pinning: with the bundled sizes (``stack.BUNDLED``) this oracle reproduces
``vocalarc_oracle.forward`` bit for bit (``tests/test_stack.py``), and that
module is pinned to the reference executable's dumps.  For other sizes
(config 3: dim 512, 62 bands, hop 441, GEGLU) there is no reference
implementation; the semantics are builder-defined, not reference-pinned.
"""

from __future__ import annotations

import numpy as np

from karaoke_platform_sidecar_native_b200.stack import StackConfig, split_weights
from oracle import vocalarc_oracle as O

F32 = np.float32


def band_rows(cfg: StackConfig, source: np.ndarray, band: int) -> np.ndarray:
    """Band ``band`` of ``source[1025][2][T][2]`` as ``[T][4 w_b]`` rows (frequency, channel, re/im)."""
    first, width = cfg.band_first[band], cfg.band_bins[band]
    block = source[first:first + width]
    return np.ascontiguousarray(block.transpose(2, 0, 1, 3)).reshape(source.shape[2], 4 * width)


def band_split(cfg: StackConfig, w: dict, source: np.ndarray) -> np.ndarray:
    """``source`` -> band-major ``x[bands][T][dim]``."""
    frames = source.shape[2]
    out = np.empty((cfg.bands, frames, cfg.dim), dtype=F32)
    for band in range(cfg.bands):
        p = f"bands.{band}."
        rows = O.rms_norm(band_rows(cfg, source, band), w[p + "gamma"])
        out[band] = O.linear(rows, w[p + "weight"], w[p + "bias"])
    return out


def transformer(cfg: StackConfig, w: dict, prefix: str, data: np.ndarray) -> np.ndarray:
    """One pre-norm axial block on ``data[S][L][dim]``."""
    seqs, length, _ = data.shape
    inner = cfg.heads * cfg.dim_head
    x = data.astype(F32)
    normed = O.rms_norm(x, w[prefix + "gamma"])
    qkv = O.linear(normed, w[prefix + "qkv"])
    gates = O.sigmoid(O.linear(normed, w[prefix + "gate_weight"], w[prefix + "gate_bias"]))
    cos, sin = O.rotary_tables(length)
    q = O.apply_rotary(qkv[..., :inner].reshape(seqs, length, cfg.heads, cfg.dim_head), cos, sin)
    k = O.apply_rotary(qkv[..., inner:2 * inner].reshape(seqs, length, cfg.heads, cfg.dim_head), cos, sin)
    v = qkv[..., 2 * inner:].reshape(seqs, length, cfg.heads, cfg.dim_head)
    att = O.attention(q, k, v) * gates[..., None]
    x = (x + O.linear(att.reshape(seqs, length, inner), w[prefix + "out_weight"])).astype(F32)
    normed = O.rms_norm(x, w[prefix + "ff_gamma"])
    pre = O.linear(normed, w[prefix + "ff1_weight"], w[prefix + "ff1_bias"])
    if cfg.geglu:
        hidden = (pre[..., :cfg.ff_inner] * O.gelu(pre[..., cfg.ff_inner:])).astype(F32)
    else:
        hidden = O.gelu(pre)
    return (x + O.linear(hidden, w[prefix + "ff2_weight"], w[prefix + "ff2_bias"])).astype(F32)


def block(cfg: StackConfig, w: dict, layer: int, axis: int, x: np.ndarray) -> np.ndarray:
    """Block (layer, axis) on band-major ``x[bands][T][dim]``, returned band-major."""
    prefix = f"layers.{layer}.{axis}."
    if axis == 0:
        return transformer(cfg, w, prefix, x)
    f = np.ascontiguousarray(x.transpose(1, 0, 2))
    return np.ascontiguousarray(transformer(cfg, w, prefix, f).transpose(1, 0, 2))


def mask_estimate(cfg: StackConfig, w: dict, x: np.ndarray) -> np.ndarray:
    """Final norm + per-band mask MLPs: band-major ``x`` -> ``mask[1025][2][T][2]``."""
    frames = x.shape[1]
    normed = O.rms_norm(x, w["final_gamma"])
    mask = np.zeros((O.FREQ_BINS, O.CHANNELS, frames, 2), dtype=F32)
    for band in range(cfg.bands):
        p = f"masks.{band}."
        d = cfg.band_dims[band]
        hidden = np.tanh(O.linear(normed[band], w[p + "first_weight"], w[p + "first_bias"]))
        proj = O.linear(hidden, w[p + "second_weight"], w[p + "second_bias"])
        values = (proj[:, :d] * O.sigmoid(proj[:, d:])).astype(F32)
        first = cfg.band_first[band]
        mask[first:first + d // 4] = values.reshape(frames, d // 4, O.CHANNELS, 2).transpose(1, 2, 0, 3)
    return mask


def forward(cfg: StackConfig, weights: np.ndarray, audio: np.ndarray, stages: dict | None = None) -> np.ndarray:
    """Whole-clip forward of one planar ``[2][len]`` clip -> vocals ``[2][len]``."""
    w = split_weights(cfg, weights)
    audio = np.asarray(audio, dtype=F32)
    length = audio.shape[1]
    source = O.stft(audio, cfg.hop)
    x = band_split(cfg, w, source)
    band = x.copy() if stages is not None else None
    for layer in range(cfg.depth):
        x = block(cfg, w, layer, 0, x)
        x = block(cfg, w, layer, 1, x)
    mask = mask_estimate(cfg, w, x)
    vocals = O.istft(source, mask, length, cfg.hop)
    if stages is not None:
        stages.update(source=source, band=band, features=x, mask=mask)
    return vocals


def frame_major(ref: np.ndarray) -> np.ndarray:
    """``[1025][2][T][2]`` -> the device's frame-major ``[T][1025][2][2]``."""
    return np.ascontiguousarray(ref.transpose(2, 0, 1, 3))
