"""Generate golden fixtures from the UNCHANGED reference CPU executable.

Run where the reference sources are checked out (``make -C oracle ref REF=<reference>/native``):

    python tests/golden/make_golden.py            # the small cases (seconds)
    python tests/golden/make_golden.py --large    # the benchmarked sizes (about 20 min on 8 cores)
    python tests/golden/make_golden.py --wav      # host input conversion (PCM16 mono 22.05 kHz)

For each case it writes a seeded float32 WAV, runs ``oracle/_ref/vocalarc-separation``
(built from native/vocalarc_separation.c by oracle/Makefile) over the JSONL
``load``/``separate`` protocol with ``VOCALARC_DEBUG_DUMP`` set
(vocalarc_separation.c:67-74, dumps at :1348, :1352, :1427, :1441), and stores
the stage tensors and the vocals WAV in ``tests/golden/<case>.npz``.  The model
pack is the seeded synthetic pack ``modelpack.TEST_RECIPE``; its sha256 is
stored so a test can confirm that regeneration is bit-identical.
"""

from __future__ import annotations

import hashlib
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from karaoke_platform_sidecar_native_b200 import fixtures, modelpack  # noqa: E402

EXE = os.path.join(ROOT, "oracle", "_ref", "vocalarc-separation")

#: case name -> (samples, seed, frames kept from the feature dumps)
CASES = {
    "clip_a": (13230, 0, (0, 1, 13, 25)),     # 0.3 s, T = 26
    "clip_t1": (300, 3, (0,)),                 # T = 1, length < NFFT/2 (multi-reflect)
    "clip_t2": (1000, 4, (0, 1)),              # T = 2
}
BANDS_KEPT = (0, 24, 60, 88, 89)

#: The sizes the benchmark runs, with both synthetic packs (parity recipe and
#: benchmark recipe).  case -> (input, pack recipe, frames kept)
#:   cfg1_10s_*    config 1: the 10 s seed-0 tone mix, whole clip, T = 862
#:   cfg2_chunk13_*  config 2: chunk 13 of the 27 chunks of the 240 s seed-1
#:                   mix (reflect border pad, pad_chunk), 881,559 samples,
#:                   T = 1722 -- one unit of the chunked benchmark
#: The input audio is not stored (it is regenerated from the seed); its sha256
#: is, so a test can confirm it rebuilt the same samples.
LARGE_CASES = {
    "cfg1_10s_test": (("tone", 10.0, 0), "TEST", (0, 1, 430, 860, 861)),
    "cfg1_10s_bench": (("tone", 10.0, 0), "BENCH", (0, 1, 430, 860, 861)),
    "cfg2_chunk13_test": (("chunk", 240.0, 1, 13), "TEST", (0, 1, 861, 1720, 1721)),
    "cfg2_chunk13_bench": (("chunk", 240.0, 1, 13), "BENCH", (0, 1, 861, 1720, 1721)),
}


def large_input(spec) -> np.ndarray:
    if spec[0] == "tone":
        return fixtures.tone_mix(spec[1], spec[2])
    mix = fixtures.long_mix(spec[1], spec[2])
    return fixtures.demix_chunk(mix, spec[3])


def run_reference(pack: str, wav: str, vocals: str, dump: str, threads: int = 8) -> dict:
    requests = [
        {"id": 1, "type": "load"},
        {"id": 2, "type": "separate", "inputPath": wav, "vocalsPath": vocals},
        {"id": 3, "type": "shutdown"},
    ]
    env = dict(os.environ, VOCALARC_DEBUG_DUMP=dump)
    proc = subprocess.run([EXE, "--model", pack, "--threads", str(threads)],
                          input="".join(json.dumps(r) + "\n" for r in requests),
                          capture_output=True, text=True, env=env, check=True)
    lines = [json.loads(x) for x in proc.stdout.splitlines() if x.strip()]
    assert lines[1]["ok"], proc.stdout
    return lines[1]


def main_large(names) -> None:
    for name in names:
        spec, recipe, frames_kept = LARGE_CASES[name]
        pack = modelpack.pack_path(modelpack.TEST_RECIPE if recipe == "TEST" else modelpack.BENCH_RECIPE)
        digest = hashlib.sha256(open(pack, "rb").read()).hexdigest()
        audio = large_input(spec)
        with tempfile.TemporaryDirectory() as tmp:
            wav = os.path.join(tmp, "in.wav")
            fixtures.write_wav_f32(wav, audio)
            vocals_path = os.path.join(tmp, "vocals.wav")
            prefix = os.path.join(tmp, "d")
            reply = run_reference(pack, wav, vocals_path, prefix)
            frames = reply["frames"]

            def dump(stage, shape):
                return np.fromfile(f"{prefix}-{stage}.f32", dtype=np.float32).reshape(shape)

            fk = list(frames_kept)
            mask = dump("mask", (1025, 2, frames, 2))[:, :, fk, :]
            f16 = dump("features16", (frames, 90, 256))[fk]
            vocals = fixtures.read_wav_f32(vocals_path)
            np.savez_compressed(
                os.path.join(HERE, f"{name}.npz"),
                vocals=vocals, mask=np.ascontiguousarray(mask), features16=f16,
                frames_kept=np.array(frames_kept), frames=np.array(frames),
                audio_sha256=np.array(hashlib.sha256(np.ascontiguousarray(audio).tobytes()).hexdigest()),
                pack_sha256=np.array(digest), recipe=np.array(recipe),
                inference_ms=np.array(float(reply.get("inferenceMs", -1))))
            print(name, "frames", frames, "inferenceMs", reply.get("inferenceMs"),
                  "vocals rms", float(np.sqrt((vocals ** 2).mean())), flush=True)


#: Host input conversion (wav_read, to_stereo, resample_linear): a PCM16 mono
#: 22.05 kHz WAV through the reference executable; its "source" dump is the
#: STFT of the converted 44.1 kHz stereo input.
WAV_CASE = "wav_pcm16_mono_22k"


def main_wav() -> None:
    pack = modelpack.pack_path(modelpack.TEST_RECIPE)
    digest = hashlib.sha256(open(pack, "rb").read()).hexdigest()
    mono = fixtures.tone_mix(0.25, 21)[:1, ::2]                     # 5513 samples at 22.05 kHz
    raw = fixtures.wav_bytes(mono, rate=22050, bits=16, pcm=True, extra_chunk=b"LIST" + (3).to_bytes(4, "little") + b"abc\0")
    with tempfile.TemporaryDirectory() as tmp:
        wav = os.path.join(tmp, "in.wav")
        open(wav, "wb").write(raw)
        vocals_path = os.path.join(tmp, "vocals.wav")
        prefix = os.path.join(tmp, "d")
        reply = run_reference(pack, wav, vocals_path, prefix)
        frames = reply["frames"]
        source = np.fromfile(f"{prefix}-source.f32", dtype=np.float32).reshape(1025, 2, frames, 2)
        vocals = fixtures.read_wav_f32(vocals_path)
        np.savez_compressed(os.path.join(HERE, f"{WAV_CASE}.npz"), wav=np.frombuffer(raw, dtype=np.uint8),
                            source=source, vocals=vocals, frames=np.array(frames), pack_sha256=np.array(digest))
        print(WAV_CASE, "frames", frames, "length", vocals.shape[1])


def main() -> None:
    pack = modelpack.pack_path(modelpack.TEST_RECIPE)
    digest = hashlib.sha256(open(pack, "rb").read()).hexdigest()
    for name, (samples, seed, frames_kept) in CASES.items():
        with tempfile.TemporaryDirectory() as tmp:
            audio = fixtures.tone_mix(samples / fixtures.RATE, seed)
            assert audio.shape[1] == samples
            wav = os.path.join(tmp, "in.wav")
            fixtures.write_wav_f32(wav, audio)
            vocals_path = os.path.join(tmp, "vocals.wav")
            prefix = os.path.join(tmp, "d")
            reply = run_reference(pack, wav, vocals_path, prefix)
            frames = reply["frames"]

            def dump(stage, shape):
                return np.fromfile(f"{prefix}-{stage}.f32", dtype=np.float32).reshape(shape)

            source = dump("source", (1025, 2, frames, 2))
            band = dump("band", (90, frames, 256))
            f1 = dump("features1", (frames, 90, 256))
            f16 = dump("features16", (frames, 90, 256))
            mask = dump("mask", (1025, 2, frames, 2))
            vocals = fixtures.read_wav_f32(vocals_path)
            np.savez_compressed(
                os.path.join(HERE, f"{name}.npz"),
                audio=audio, source=source, mask=mask, vocals=vocals,
                band=band[list(BANDS_KEPT)], bands_kept=np.array(BANDS_KEPT),
                features1=f1[list(frames_kept)], features16=f16[list(frames_kept)],
                frames_kept=np.array(frames_kept), frames=np.array(frames),
                pack_sha256=np.array(digest), seed=np.array(seed))
            print(name, "frames", frames, "vocals rms", float(np.sqrt((vocals ** 2).mean())))


if __name__ == "__main__":
    if "--wav" in sys.argv:
        main_wav()
    elif "--large" in sys.argv:
        chosen = [a for a in sys.argv[1:] if a in LARGE_CASES]
        main_large(chosen or list(LARGE_CASES))
    else:
        main()
