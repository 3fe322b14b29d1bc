"""CPU oracle for the VocalArc BS-RoFormer separation forward (TEST INFRASTRUCTURE).

This module is the parity checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of ``bench.py`` may
import it.  It restates, in numpy float32 (FFT in float64 as the reference
does), the reference CPU path of ``native/vocalarc_separation.c``:

* STFT ``stft_channels`` :1044-1064 with ``reflect_index`` :1027-1034 and the
  periodic Hann window of :1052;
* band split ``band_split_one`` :887-915 / ``band_split`` :917-926;
* RMSNorm ``rms_norm_row_scalar`` :419-424;
* the axial transformer block ``transformer_forward`` :836-873, with RoPE
  ``apply_rotary`` :714-744 / ``rotary_rows`` :692-712 / ``fill_frequencies``
  :1312-1314, attention ``attention_heads`` :753-793 (non-causal softmax,
  scale 0.125), head gates ``apply_gates`` :808-818 and exact-erf GELU
  ``gelu_values`` :666-672;
* final norm ``inplace_norm`` :973-984 and the mask MLP ``mask_band``
  :1316-1340 (Linear, tanh, Linear, GLU, scatter);
* iSTFT ``istft_channels`` :1084-1127 (complex mask, Hermitian fill, inverse
  FFT / 2048, windowed overlap-add in frame order, divide by the channel-0
  window envelope or 0 when it is <= 1e-12; no DC zeroing);
* ``forward_model`` :1342-1445 (whole clip, frames = length / 512 + 1);
* chunked overlap-add ``Separator::demix`` onnx/native/onnx_sidecar.cpp:725-782
  with ``pad_chunk`` :366-383, applied around the native forward.

Parity of this restatement is pinned against the reference executable itself:
``tests/golden/make_golden.py`` runs the unchanged reference CPU build on the
seeded synthetic pack and stores its stage dumps (``VOCALARC_DEBUG_DUMP``) and
output WAV; ``tests/test_oracle.py`` compares this module against them.  The
chunk assembly (``demix``), ``bigshift`` and ``separate_tta`` follow the C++
ONNX sidecar, which cannot run here; ``tests/golden/make_demix_twin.py`` runs
the reference's Python twin of that loop (onnx/audio.py) and
``tests/test_demix_twin.py`` checks this module against it.

Known intentional differences: the reference exponentials use its own
polynomial ``fast_exp`` (:383-398) and its FFT is a radix-2 recurrence; both
are matched here only to float32 rounding, which the golden comparison
tolerances state.
"""

from __future__ import annotations

import math

import numpy as np

try:
    from scipy.special import erf as _erf
except ImportError:  # pragma: no cover - scipy is present in this image
    _erf = np.vectorize(math.erf)

from karaoke_platform_sidecar_native_b200.modelpack import (
    BAND_DIMS, BAND_FIRST, BAND_FREQS, BANDS, CHANNELS, DEPTH, DIM, DIM_HEAD, DIM_INNER,
    FREQ_BINS, HEADS, HOP, NFFT, WIN_LENGTH)

F32 = np.float32


def window() -> np.ndarray:
    """``0.5f - 0.5f * cosf((float)(2 pi i / 2048))`` (vocalarc_separation.c:1052)."""
    i = np.arange(NFFT, dtype=np.float64)
    arg = (2.0 * math.pi * i / WIN_LENGTH).astype(F32)
    c = np.cos(arg.astype(np.float64)).astype(F32)
    return (F32(0.5) - F32(0.5) * c).astype(F32)


def reflect_index(index: np.ndarray, length: int) -> np.ndarray:
    """Vectorised ``reflect_index`` (vocalarc_separation.c:1027-1034)."""
    index = np.asarray(index, dtype=np.int64)
    if length <= 1:
        return np.zeros_like(index)
    # Repeated reflection about 0 and length-1 is periodic with period 2*length-2.
    period = 2 * length - 2
    r = np.mod(index, period)
    return np.where(r >= length, period - r, r)


def frames_for(length: int, hop: int = HOP) -> int:
    return length // hop + 1


def stft(audio: np.ndarray, hop: int = HOP) -> np.ndarray:
    """Planar ``[2][len]`` audio -> ``source[1025][2][T][2]`` (reference layout).

    ``hop`` other than 512 is the same framing with another frame step (the
    configurable stack's STFT; the reference only has 512).
    """
    audio = np.asarray(audio, dtype=F32)
    length = audio.shape[1]
    frames = frames_for(length, hop)
    win = window()
    starts = np.arange(frames, dtype=np.int64) * hop - NFFT // 2
    idx = reflect_index(starts[:, None] + np.arange(NFFT)[None, :], length)
    out = np.empty((FREQ_BINS, CHANNELS, frames, 2), dtype=F32)
    for ch in range(CHANNELS):
        framed = (audio[ch][idx] * win[None, :]).astype(np.float64)
        spec = np.fft.fft(framed, axis=1)[:, :FREQ_BINS]
        out[:, ch, :, 0] = spec.real.T.astype(F32)
        out[:, ch, :, 1] = spec.imag.T.astype(F32)
    return out


def rms_norm(x: np.ndarray, gamma: np.ndarray) -> np.ndarray:
    """Row RMSNorm: ``x * (sqrtf(d) / sqrtf(sum x^2 + 1e-12)) * gamma``."""
    x = np.asarray(x, dtype=F32)
    d = x.shape[-1]
    sums = np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True).astype(F32)
    inverse = (F32(math.sqrt(d)) / np.sqrt(sums + F32(1e-12))).astype(F32)
    return ((x * inverse) * gamma).astype(F32)


def linear(x: np.ndarray, weight: np.ndarray, bias: np.ndarray | None = None) -> np.ndarray:
    y = np.matmul(x.astype(F32), weight.T.astype(F32))
    if bias is not None:
        y = y + bias
    return y.astype(F32)


def band_rows(source: np.ndarray, band: int) -> np.ndarray:
    """Gather band ``band`` of ``source[1025][2][T][2]`` as ``[T][d_b]`` rows.

    Row order is frequency, then channel, then (re, im) (vocalarc_separation.c:893-901).
    """
    first, width = BAND_FIRST[band], BAND_FREQS[band]
    block = source[first:first + width]                      # [w][2][T][2]
    return np.ascontiguousarray(block.transpose(2, 0, 1, 3)).reshape(source.shape[2], 4 * width)


def band_split(model, source: np.ndarray) -> np.ndarray:
    """``source`` -> ``time_sequences[90][T][256]``."""
    frames = source.shape[2]
    out = np.empty((BANDS, frames, DIM), dtype=F32)
    for band in range(BANDS):
        w = model.bands[band]
        rows = rms_norm(band_rows(source, band), w["gamma"])
        out[band] = linear(rows, w["weight"], w["bias"])
    return out


def rotary_frequencies() -> np.ndarray:
    """``1.0f / powf(10000.0f, (float)(2 i) / 64)`` (vocalarc_separation.c:1312-1314)."""
    i = np.arange(DIM_HEAD // 2)
    expo = (np.float32(2) * i.astype(F32) / F32(DIM_HEAD)).astype(F32)
    pw = np.power(10000.0, expo.astype(np.float64)).astype(F32)
    return (F32(1.0) / pw).astype(F32)


def rotary_tables(length: int):
    """cos/sin tables ``[length][32]`` as ``apply_rotary`` builds them (:726-731)."""
    freqs = rotary_frequencies()
    angle = (np.arange(length, dtype=F32)[:, None] * freqs[None, :]).astype(F32)
    a64 = angle.astype(np.float64)
    return np.cos(a64).astype(F32), np.sin(a64).astype(F32)


def apply_rotary(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Rotate contiguous pairs (2i, 2i+1) of ``x[..., L, heads, 64]``."""
    first = x[..., 0::2]
    second = x[..., 1::2]
    c = cos[:, None, :]
    s = sin[:, None, :]
    out = np.empty_like(x)
    out[..., 0::2] = first * c - second * s
    out[..., 1::2] = first * s + second * c
    return out


def sigmoid(x: np.ndarray) -> np.ndarray:
    return (F32(1.0) / (F32(1.0) + np.exp(-x.astype(F32)))).astype(F32)


def gelu(x: np.ndarray) -> np.ndarray:
    x = x.astype(F32)
    e = _erf((x * F32(0.7071067811865475)).astype(np.float64)).astype(F32)
    return (F32(0.5) * x * (F32(1.0) + e)).astype(F32)


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """Non-causal softmax attention, scale 0.125; inputs ``[S][L][H][64]``."""
    qh = q.transpose(0, 2, 1, 3)
    kh = k.transpose(0, 2, 1, 3)
    vh = v.transpose(0, 2, 1, 3)
    out = np.empty_like(qh)
    # Block over sequences to bound memory of the [S][H][L][L] score tensor.
    step = max(1, int(2e8 // max(1, qh.shape[1] * qh.shape[2] * qh.shape[2])))
    for s0 in range(0, qh.shape[0], step):
        scores = np.matmul(qh[s0:s0 + step], kh[s0:s0 + step].transpose(0, 1, 3, 2)) * F32(0.125)
        scores -= scores.max(axis=-1, keepdims=True)
        np.exp(scores, out=scores)
        scores /= scores.sum(axis=-1, keepdims=True)
        out[s0:s0 + step] = np.matmul(scores, vh[s0:s0 + step])
    return out.transpose(0, 2, 1, 3).astype(F32)


def transformer(w: dict, data: np.ndarray) -> np.ndarray:
    """One pre-norm axial block on ``data[S][L][256]`` (returns the new data)."""
    seqs, length, _ = data.shape
    x = data.astype(F32)
    normed = rms_norm(x, w["gamma"])
    qkv = linear(normed, w["qkv"])
    gates = sigmoid(linear(normed, w["gate_weight"], w["gate_bias"]))
    cos, sin = rotary_tables(length)
    q = apply_rotary(qkv[..., :DIM_INNER].reshape(seqs, length, HEADS, DIM_HEAD), cos, sin)
    k = apply_rotary(qkv[..., DIM_INNER:2 * DIM_INNER].reshape(seqs, length, HEADS, DIM_HEAD), cos, sin)
    v = qkv[..., 2 * DIM_INNER:].reshape(seqs, length, HEADS, DIM_HEAD)
    att = attention(q, k, v) * gates[..., None]
    x = (x + linear(att.reshape(seqs, length, DIM_INNER), w["out_weight"])).astype(F32)
    normed = rms_norm(x, w["ff_gamma"])
    hidden = gelu(linear(normed, w["ff1_weight"], w["ff1_bias"]))
    x = (x + linear(hidden, w["ff2_weight"], w["ff2_bias"])).astype(F32)
    return x


def transformer_stack(model, time_sequences: np.ndarray, keep: tuple = ()) -> tuple:
    """All 16 layers (time axis then band axis) from ``[90][T][256]``.

    Returns ``(features[T][90][256], dumps)`` where ``dumps`` maps layer index
    (after its band-axis block, as ``features1``/``features16`` in :1427) for
    every index listed in ``keep``.
    """
    x = time_sequences
    dumps = {}
    for layer in range(DEPTH):
        x = transformer(model.layers[layer][0], x)                  # [90][T][256]
        f = np.ascontiguousarray(x.transpose(1, 0, 2))              # [T][90][256]
        f = transformer(model.layers[layer][1], f)
        if layer + 1 in keep:
            dumps[layer + 1] = f.copy()
        x = np.ascontiguousarray(f.transpose(1, 0, 2))
    return np.ascontiguousarray(x.transpose(1, 0, 2)), dumps


def mask_estimate(model, features: np.ndarray) -> np.ndarray:
    """Final norm + 90 mask MLPs: ``features[T][90][256]`` -> ``mask[1025][2][T][2]``."""
    frames = features.shape[0]
    normed = rms_norm(features, model.final_gamma)
    mask = np.zeros((FREQ_BINS, CHANNELS, frames, 2), dtype=F32)
    for band in range(BANDS):
        w = model.masks[band]
        d = BAND_DIMS[band]
        hidden = np.tanh(linear(normed[:, band, :], w["first_weight"], w["first_bias"]))
        proj = linear(hidden, w["second_weight"], w["second_bias"])
        values = (proj[:, :d] * sigmoid(proj[:, d:])).astype(F32)    # [T][d]
        first = BAND_FIRST[band]
        block = values.reshape(frames, d // 4, CHANNELS, 2).transpose(1, 2, 0, 3)
        mask[first:first + d // 4] = block
    return mask


def istft(source: np.ndarray, mask: np.ndarray, length: int, hop: int = HOP) -> np.ndarray:
    """Masked inverse STFT with the native normalisation rule -> ``[2][length]``."""
    frames = source.shape[2]
    win = window()
    out = np.zeros((CHANNELS, length), dtype=F32)
    envelope = np.zeros(length, dtype=F32)
    for ch in range(CHANNELS):
        s = source[:, ch].astype(np.float32)                         # [1025][T][2]
        m = mask[:, ch].astype(np.float32)
        re = (s[..., 0] * m[..., 0] - s[..., 1] * m[..., 1]).astype(F32)
        im = (s[..., 0] * m[..., 1] + s[..., 1] * m[..., 0]).astype(F32)
        spec = re.astype(np.float64) + 1j * im.astype(np.float64)   # [1025][T]
        full = np.zeros((NFFT, frames), dtype=np.complex128)
        full[:FREQ_BINS] = spec
        full[NFFT - np.arange(1, FREQ_BINS - 1)] = np.conj(spec[1:FREQ_BINS - 1])
        time = np.fft.ifft(full, axis=0).real                        # includes / 2048
        contrib = (time * win.astype(np.float64)[:, None]).astype(F32)  # [2048][T]
        for frame in range(frames):
            start = frame * hop - NFFT // 2
            lo, hi = max(0, start), min(length, start + NFFT)
            if lo >= hi:
                continue
            out[ch, lo:hi] += contrib[lo - start:hi - start, frame]
            if ch == 0:
                envelope[lo:hi] += (win[lo - start:hi - start] * win[lo - start:hi - start]).astype(F32)
    safe = envelope > F32(1e-12)
    result = np.zeros_like(out)
    result[:, safe] = out[:, safe] / envelope[safe]
    return result


def forward(model, audio: np.ndarray, keep: tuple = (), stages: dict | None = None) -> np.ndarray:
    """Whole-clip native forward (``forward_model`` :1342): ``[2][len]`` -> vocals."""
    audio = np.asarray(audio, dtype=F32)
    length = audio.shape[1]
    source = stft(audio)
    band = band_split(model, source)
    features, dumps = transformer_stack(model, band, keep)
    mask = mask_estimate(model, features)
    vocals = istft(source, mask, length)
    if stages is not None:
        stages.update(source=source, band=band, features=features, mask=mask, dumps=dumps)
    return vocals


# --------------------------------------------------------------------------- chunked
CHUNK_SAMPLES = 881_559          # onnx/native/onnx_sidecar.cpp:53, onnx/config.py:23
STEP_SAMPLES = CHUNK_SAMPLES // 2


def pad_chunk(working: np.ndarray, start: int, chunk: int) -> np.ndarray:
    """``pad_chunk`` (onnx_sidecar.cpp:366-383): copy, reflect-fill if more than half."""
    total = working.shape[1]
    available = min(total - start, chunk) if start < total else 0
    out = np.zeros((CHANNELS, chunk), dtype=F32)
    out[:, :available] = working[:, start:start + available]
    if available > chunk // 2 and available > 1 and available < chunk:
        idx = reflect_index(np.arange(available, chunk), available)
        out[:, available:] = working[:, start + idx]
    return out


def chunk_plan(length: int, chunk: int = CHUNK_SAMPLES, step: int | None = None) -> tuple:
    """(border, padded_length, [(start, valid_length), ...]) of ``demix``."""
    step = chunk // 2 if step is None else step
    border = chunk - step
    padded = length + 2 * border if (length > 2 * border and border > 0) else length
    starts = []
    position = 0
    while position < padded:
        starts.append((position, min(chunk, padded - position)))
        position += step
    return border, padded, starts


def chunk_weights(count: int, chunk: int, batch: int = 1, fade_ramp: np.ndarray | None = None) -> np.ndarray:
    """Per-chunk OLA weights ``[count][chunk]``: linear fade over the last chunk/10
    samples, forced to 1 for chunks of the first and the final predict batch
    (onnx_sidecar.cpp:740-767; ``batch`` is the sidecar's model batch size).

    ``fade_ramp`` (chunk/10 values) replaces the sidecar's ramp 1 - i/fade
    (:741-742).  The reference's Python twin of this loop (onnx/audio.py:153-154)
    uses linspace(1, 0, fade) instead; the tests pass that ramp to compare the
    rest of the assembly with the twin's own output."""
    fade = chunk // 10
    base = np.ones(chunk, dtype=F32)
    if fade_ramp is None:
        base[chunk - fade:] = (F32(1.0) - np.arange(fade, dtype=F32) / F32(fade)).astype(F32)
    elif fade > 0:
        base[chunk - fade:] = np.asarray(fade_ramp, dtype=F32)
    weights = np.repeat(base[None, :], count, axis=0)
    step_batches = [list(range(i, min(i + batch, count))) for i in range(0, count, batch)]
    for b_index, members in enumerate(step_batches):
        first_batch = b_index == 0 and len(members) == 1
        final_batch = b_index == len(step_batches) - 1
        if first_batch or final_batch:
            weights[members] = 1.0
    return weights


def demix(predict, mix: np.ndarray, chunk: int = CHUNK_SAMPLES, batch: int = 1,
          fade_ramp: np.ndarray | None = None) -> np.ndarray:
    """Chunked overlap-add (``Separator::demix`` onnx_sidecar.cpp:725-782);
    ``fade_ramp`` as in ``chunk_weights``."""
    mix = np.asarray(mix, dtype=F32)
    length = mix.shape[1]
    border, padded, plan = chunk_plan(length, chunk)
    if padded != length:
        idx = reflect_index(np.arange(padded) - border, length)
        working = mix[:, idx]
    else:
        working = mix
    weights = chunk_weights(len(plan), chunk, batch, fade_ramp)
    result = np.zeros((CHANNELS, padded), dtype=F32)
    counter = np.zeros((CHANNELS, padded), dtype=F32)
    for index, (start, valid) in enumerate(plan):
        estimate = predict(pad_chunk(working, start, chunk))
        w = weights[index, :valid]
        result[:, start:start + valid] += estimate[:, :valid] * w
        counter[:, start:start + valid] += w
    output = (result / np.maximum(counter, F32(1e-12))).astype(F32)
    if padded != length:
        output = output[:, border:border + length]
    return output


# ---------------------------------------------------------------- bigshifts + TTA
def rotate_audio(audio: np.ndarray, shift: int) -> np.ndarray:
    """``rotate_audio`` (onnx_sidecar.cpp:385-396): out[i] = in[(n - shift + i) % n]."""
    n = audio.shape[1]
    if n == 0:
        return audio.copy()
    shift %= n
    return audio[:, (n - shift + np.arange(n)) % n].astype(F32)


def unrotate_audio(audio: np.ndarray, shift: int) -> np.ndarray:
    """``unrotate_audio`` (onnx_sidecar.cpp:398-408): out[i] = in[(i + shift) % n]."""
    n = audio.shape[1]
    if n == 0:
        return audio.copy()
    shift %= n
    return audio[:, (np.arange(n) + shift) % n].astype(F32)


def bigshift(separate, mix: np.ndarray, count: int) -> np.ndarray:
    """``bigshift`` (onnx_sidecar.cpp:784-790): the mean of ``count`` chunked
    separations of circularly rotated copies, each rotated back.  Float32
    arithmetic in the reference's order: result = 0; result += 1 * estimate_k
    (k ascending); result *= 1/count."""
    mix = np.asarray(mix, dtype=F32)
    result = np.zeros_like(mix)
    shift_size = mix.shape[1] // count
    for index in range(count):
        estimate = unrotate_audio(separate(rotate_audio(mix, index * shift_size)), index * shift_size)
        result = (result + F32(1.0) * estimate).astype(F32)
    return (result * F32(1.0 / count)).astype(F32)


def separate_tta(separate, mix: np.ndarray, bigshifts: int = 2, tta: bool = True) -> np.ndarray:
    """``Separator::separate`` (onnx_sidecar.cpp:556-575).  With TTA the estimate
    of the channel-swapped mix (swapped back) is added and the polarity-flipped
    estimate ``inverted = -bigshift(-mix)`` is combined with ``right_scale = -1``
    (:572-573), then scaled by 1/3 -- restated exactly as the reference computes
    it."""
    mix = np.asarray(mix, dtype=F32)
    bigshifts = max(1, int(bigshifts))
    vocals = bigshift(separate, mix, bigshifts)
    if not tta:
        return vocals
    restored = bigshift(separate, mix[::-1].copy(), bigshifts)[::-1].copy()
    inverted = (bigshift(separate, (mix * F32(-1.0)).astype(F32), bigshifts) * F32(-1.0)).astype(F32)
    total = (vocals + F32(1.0) * restored).astype(F32)
    total = (total + F32(-1.0) * inverted).astype(F32)
    return (total * F32(1.0 / 3.0)).astype(F32)


# --------------------------------------------------------------- host WAV input
def wav_decode(raw: bytes):
    """``wav_read`` (vocalarc_separation.c:1152-1187): (planar float32 [channels][n], rate).

    RIFF/WAVE chunks are walked in order (the last "fmt " of >= 16 bytes and
    the last "data" win; a chunk running past the end stops the walk); PCM
    16/24/32-bit (format 1) or float32 (format 3), 1 or 2 channels.
    """
    if len(raw) < 44 or raw[:4] != b"RIFF" or raw[8:12] != b"WAVE":
        raise ValueError("unsupported WAV input")
    fmt = None
    data = None
    offset = 12
    while offset + 8 <= len(raw):
        size = int.from_bytes(raw[offset + 4:offset + 8], "little")
        payload = offset + 8
        if payload > len(raw) or size > len(raw) - payload:
            break
        tag = raw[offset:offset + 4]
        if tag == b"fmt " and size >= 16:
            body = raw[payload:payload + 16]
            fmt = (int.from_bytes(body[0:2], "little"), int.from_bytes(body[2:4], "little"),
                   int.from_bytes(body[4:8], "little"), int.from_bytes(body[14:16], "little"))
        elif tag == b"data":
            data = raw[payload:payload + size]
        offset = payload + size + (size & 1)
    if fmt is None or data is None:
        raise ValueError("WAV without fmt or data")
    form, channels, rate, bits = fmt
    if not (1 <= channels <= 2 and rate >= 1 and (form == 3 and bits == 32 or form == 1 and bits in (16, 24, 32))):
        raise ValueError("WAV must be PCM16/24/32 or float32 mono/stereo")
    width = bits // 8
    n = len(data) // (channels * width)
    body = np.frombuffer(data[:n * channels * width], dtype=np.uint8).reshape(n, channels, width)
    if form == 3:
        values = body.copy().view("<f4")[..., 0]
    elif bits == 16:
        values = body.copy().view("<i2")[..., 0].astype(F32) / F32(32768.0)
    elif bits == 24:
        v = body[..., 0].astype(np.int32) | (body[..., 1].astype(np.int32) << 8) | (body[..., 2].astype(np.int32) << 16)
        v = np.where(v & 0x800000, v | ~0xFFFFFF, v).astype(np.int32)
        values = v.astype(F32) / F32(8388608.0)
    else:
        values = body.copy().view("<i4")[..., 0].astype(F32) / F32(2147483648.0)
    return np.ascontiguousarray(values.T.astype(F32)), rate


def to_stereo(planar: np.ndarray) -> np.ndarray:
    """``to_stereo`` (vocalarc_separation.c:1189-1196): mono is duplicated."""
    return planar if planar.shape[0] == 2 else np.concatenate([planar, planar], axis=0)


def resample_linear(audio: np.ndarray, input_rate: int, output_rate: int = 44100) -> np.ndarray:
    """``resample_linear`` (vocalarc_separation.c:1198-1222): align_corners=False
    linear interpolation, output length llround(n * out / in) (at least 1)."""
    n = audio.shape[1]
    length = max(1, int(np.floor(n * output_rate / input_rate + 0.5)))
    i = np.arange(length, dtype=np.float64)
    position = np.maximum((i + 0.5) * input_rate / output_rate - 0.5, 0.0)
    upper = np.minimum(position + 1.0, n - 1)
    lower_i = position.astype(np.int64)
    upper_i = upper.astype(np.int64)
    fraction = (position - lower_i).astype(F32)
    one = F32(1.0)
    return (audio[:, lower_i] * (one - fraction) + audio[:, upper_i] * fraction).astype(F32)


def read_track(raw: bytes) -> np.ndarray:
    """A host request's input as ``separate`` prepares it (:1568-1572): decoded,
    stereo, resampled to 44.1 kHz when needed."""
    planar, rate = wav_decode(raw)
    stereo = to_stereo(planar)
    return stereo if rate == 44100 else resample_linear(stereo, rate)
