"""Seeded synthetic stereo mixes and float32 WAV I/O.

No public dataset is involved: the workloads are seeded numpy (PCG64) signals
with the shapes and value ranges the benchmark configurations describe.

* ``tone_mix`` (configs 1 and 5): three harmonic tones, f0 ~ U(100, 800) Hz,
  six harmonics with 1/k amplitude and random phase, peak-normalised to 0.2,
  plus independent white noise N(0, 0.05^2) per channel.
* ``long_mix`` (config 2): the same tone recipe with f0 redrawn every 0.5 s,
  pink noise (white noise shaped by 1/sqrt(f) in the frequency domain, scaled
  to sigma 0.05) and a 120 BPM click track of 10 ms exponentially decaying
  noise bursts.

Audio is planar ``float32[2][length]`` like the reference host's buffers
(``wav_read`` native/vocalarc_separation.c:1152-1187 stores channel-major).
"""

from __future__ import annotations

import struct

import numpy as np

RATE = 44100


def _harmonic(f0: np.ndarray, phase: np.ndarray, t: np.ndarray) -> np.ndarray:
    out = np.zeros_like(t)
    for k in range(1, 7):
        out += np.sin(2.0 * np.pi * k * f0 * t + k * phase) / k
    return out


def tone_mix(seconds: float, seed: int = 0) -> np.ndarray:
    """Config-1 recipe: three harmonic tones (peak 0.2) + white noise sigma 0.05."""
    rng = np.random.default_rng(seed)
    n = max(1, int(round(seconds * RATE)))
    t = np.arange(n, dtype=np.float64) / RATE
    f0 = rng.uniform(100.0, 800.0, size=3)
    phase = rng.uniform(0.0, 2.0 * np.pi, size=3)
    tone = sum(_harmonic(f0[j], phase[j], t) for j in range(3))
    tone *= 0.2 / max(np.max(np.abs(tone)), 1e-12)
    noise = rng.standard_normal((2, n)) * 0.05
    return (tone[None, :] + noise).astype(np.float32)


def pink_noise(n: int, rng: np.random.Generator, sigma: float) -> np.ndarray:
    spectrum = rng.standard_normal(n // 2 + 1) + 1j * rng.standard_normal(n // 2 + 1)
    freqs = np.arange(n // 2 + 1, dtype=np.float64)
    freqs[0] = 1.0
    spectrum /= np.sqrt(freqs)
    spectrum[0] = 0.0
    noise = np.fft.irfft(spectrum, n)
    return noise * (sigma / max(noise.std(), 1e-12))


def long_mix(seconds: float, seed: int = 1) -> np.ndarray:
    """Config-2 recipe: tones redrawn every 0.5 s + pink noise + 120 BPM clicks."""
    rng = np.random.default_rng(seed)
    n = max(1, int(round(seconds * RATE)))
    t = np.arange(n, dtype=np.float64) / RATE
    segment = int(0.5 * RATE)
    tone = np.zeros(n)
    for start in range(0, n, segment):
        stop = min(n, start + segment)
        f0 = rng.uniform(100.0, 800.0, size=3)
        phase = rng.uniform(0.0, 2.0 * np.pi, size=3)
        tone[start:stop] = sum(_harmonic(f0[j], phase[j], t[start:stop]) for j in range(3))
    tone *= 0.2 / max(np.max(np.abs(tone)), 1e-12)
    out = np.stack([tone + pink_noise(n, rng, 0.05) for _ in range(2)])
    click_len = int(0.010 * RATE)
    envelope = np.exp(-np.arange(click_len) / (click_len / 5.0))
    for start in range(0, n, segment):          # 120 BPM = one click per 0.5 s
        stop = min(n, start + click_len)
        burst = rng.standard_normal(stop - start) * envelope[: stop - start] * 0.3
        out[:, start:stop] += burst[None, :]
    return out.astype(np.float32)


CHUNK_SAMPLES = 881_559          # the ONNX sidecar's chunk (onnx/native/onnx_sidecar.cpp:53)


def demix_chunk_count(length: int, chunk: int = CHUNK_SAMPLES) -> int:
    """Number of chunks the chunked demix cuts a ``length``-sample track into."""
    step = chunk // 2
    border = chunk - step
    padded = length + 2 * border if length > 2 * border else length
    return -(-padded // step)


def demix_chunk(mix: np.ndarray, index: int, chunk: int = CHUNK_SAMPLES) -> np.ndarray:
    """Input of chunk ``index`` of the chunked demix, as the device path forms it.

    The track is reflect-padded by ``border = chunk - chunk//2`` samples on both
    sides (``Separator::demix`` onnx_sidecar.cpp:725-737), chunk ``index``
    starts at ``index * (chunk//2)`` of the padded track and a short final chunk
    is reflect-filled when more than half of it is real (``pad_chunk`` :366-383)
    or zero-filled otherwise.  Used to feed single chunks to the whole-clip
    forward, e.g. to check one chunk of a chunked run at its full size.
    """
    mix = np.asarray(mix, dtype=np.float32)
    length = mix.shape[1]
    step = chunk // 2
    border = chunk - step

    def reflect(i, n):
        if n <= 1:
            return np.zeros_like(i)
        period = 2 * n - 2
        r = np.mod(i, period)
        return np.where(r >= n, period - r, r)

    padded = length + 2 * border if length > 2 * border else length
    start = index * step
    if start >= padded:
        raise ValueError(f"chunk {index} starts past the padded track ({padded} samples)")
    available = min(padded - start, chunk)
    pos = np.arange(start, start + available)
    src = reflect(pos - border, length) if padded != length else pos
    out = np.zeros((mix.shape[0], chunk), dtype=np.float32)
    out[:, :available] = mix[:, src]
    if chunk // 2 < available < chunk and available > 1:
        fill = reflect(np.arange(available, chunk), available)
        out[:, available:] = out[:, fill]
    return out


def batch_mixes(count: int = 64, seconds: float = 180.0, first_seed: int = 100) -> list:
    """Config-5 recipe: ``count`` tone mixes with seeds first_seed.. (lazy list)."""
    return [(first_seed + i, seconds) for i in range(count)]


def write_wav_f32(path: str, audio: np.ndarray, rate: int = RATE) -> None:
    """Write planar ``[channels][n]`` float32 audio as a format-3 WAV."""
    audio = np.asarray(audio, dtype=np.float32)
    channels, n = audio.shape
    data = np.ascontiguousarray(audio.T).astype("<f4").tobytes()
    header = b"RIFF" + struct.pack("<I", 36 + len(data)) + b"WAVEfmt "
    header += struct.pack("<IHHIIHH", 16, 3, channels, rate, rate * channels * 4, channels * 4, 32)
    header += b"data" + struct.pack("<I", len(data))
    with open(path, "wb") as handle:
        handle.write(header + data)


def wav_bytes(audio: np.ndarray, rate: int = RATE, bits: int = 32, pcm: bool = False,
              extra_chunk: bytes = b"") -> bytes:
    """WAV file bytes of planar ``[channels][n]`` audio: float32 (format 3) or
    PCM 16/24/32-bit (format 1, values clipped to [-1, 1) and rounded).
    ``extra_chunk`` is inserted before "fmt " (e.g. a LIST chunk) to exercise
    chunk walking; odd-sized chunks get their pad byte."""
    audio = np.asarray(audio, dtype=np.float32)
    channels, n = audio.shape
    frames = np.ascontiguousarray(audio.T)
    if not pcm:
        data = frames.astype("<f4").tobytes()
        fmt_code, bits = 3, 32
    else:
        fmt_code = 1
        scale = float(2 ** (bits - 1))
        ints = np.clip(np.round(frames.astype(np.float64) * scale), -scale, scale - 1).astype(np.int64)
        if bits == 16:
            data = ints.astype("<i2").tobytes()
        elif bits == 32:
            data = ints.astype("<i4").tobytes()
        else:
            u = (ints & 0xFFFFFF).astype(np.uint32)
            b = np.stack([u & 0xFF, (u >> 8) & 0xFF, (u >> 16) & 0xFF], axis=-1).astype(np.uint8)
            data = b.tobytes()
    width = bits // 8
    fmt = struct.pack("<HHIIHH", fmt_code, channels, rate, rate * channels * width, channels * width, bits)
    body = b"WAVE" + extra_chunk + b"fmt " + struct.pack("<I", 16) + fmt + b"data" + struct.pack("<I", len(data)) + data
    if len(data) & 1:
        body += b"\0"
    return b"RIFF" + struct.pack("<I", len(body)) + body


def read_wav_f32(path: str) -> np.ndarray:
    """Read a float32 (format 3) WAV into planar ``[channels][n]``."""
    raw = open(path, "rb").read()
    if raw[:4] != b"RIFF" or raw[8:12] != b"WAVE":
        raise ValueError("not a WAV file")
    offset = 12
    fmt = None
    data = None
    while offset + 8 <= len(raw):
        tag = raw[offset:offset + 4]
        size = struct.unpack_from("<I", raw, offset + 4)[0]
        body = raw[offset + 8: offset + 8 + size]
        if tag == b"fmt ":
            fmt = struct.unpack_from("<HHIIHH", body, 0)
        elif tag == b"data":
            data = body
        offset += 8 + size + (size & 1)
    if fmt is None or data is None or fmt[0] != 3 or fmt[5] != 32:
        raise ValueError("expected a float32 WAV")
    channels = fmt[1]
    return np.frombuffer(data, dtype="<f4").reshape(-1, channels).T.astype(np.float32)
