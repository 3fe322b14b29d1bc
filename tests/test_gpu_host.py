"""The reference's own C host over this provider (fallback, non-resident path, full-device hook) and the WAV batch pipeline.

Both executables are the unchanged reference JSONL host
(native/vocalarc_separation.c) built by oracle/Makefile:
  * ``vocalarc-separation-b200``       linked to this provider (drop-in);
  * ``vocalarc-separation-b200-hook``  the same plus the guarded hook of
    oracle/hook_patch.py that runs the whole forward on the device.
The goldens are the reference CPU executable's own vocals (tests/golden).

Failure handling is tested the way the reference provider behaves
(native_gpu_cuda.cu:88-94: disable on the first error, message on stderr, the
host recomputes on the CPU, vocalarc_separation.c:1380-1382) without faulting a
GPU: the failure is injected on the host (VOCALARC_B200_FAIL_AT), and a
device-side wait is made to run out on a barrier that nothing completes.
"""

import json
import math
import os
import subprocess
import tempfile

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from karaoke_platform_sidecar_native_b200 import fixtures, modelpack, native  # noqa: E402
from tests.conftest import GOLDEN, ROOT  # noqa: E402

pytestmark = pytest.mark.gpu
SNR_BAR_DB = 50.0
MAX_ABS_BAR = 2e-3
DROPIN = os.path.join(ROOT, "oracle", "_ref", "vocalarc-separation-b200")
HOOK = os.path.join(ROOT, "oracle", "_ref", "vocalarc-separation-b200-hook")


def snr_db(ref, test):
    ref = np.asarray(ref, dtype=np.float64)
    err = ref - np.asarray(test, dtype=np.float64)
    return 10 * math.log10((ref ** 2).sum() / max((err ** 2).sum(), 1e-300))


def run_host(exe, pack, audio, env_extra=None, threads=8):
    """One load + separate over JSONL; returns (reply, vocals, stderr)."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not os.path.exists(exe):
        pytest.skip(f"{os.path.basename(exe)} not built (make -C oracle dropin hook REF=...)")
    env = dict(os.environ)
    env.update(env_extra or {})
    with tempfile.TemporaryDirectory() as tmp:
        wav = os.path.join(tmp, "in.wav")
        fixtures.write_wav_f32(wav, audio)
        out = os.path.join(tmp, "vocals.wav")
        requests = [{"id": 1, "type": "load"}, {"id": 2, "type": "separate", "inputPath": wav, "vocalsPath": out},
                    {"id": 3, "type": "shutdown"}]
        proc = subprocess.run([exe, "--model", pack, "--threads", str(threads)],
                              input="".join(json.dumps(r) + "\n" for r in requests), capture_output=True, text=True,
                              env=env, timeout=900)
        lines = [json.loads(x) for x in proc.stdout.splitlines() if x.strip()]
        assert lines[1]["ok"], proc.stdout + proc.stderr
        return lines[1], fixtures.read_wav_f32(out), proc.stderr


@pytest.fixture(scope="module")
def golden_a():
    return np.load(os.path.join(GOLDEN, "clip_a.npz"))


# ------------------------------------------------------------------ host-injected failure
@pytest.mark.parametrize("fail_at", [1, 5, 65])
def test_injected_failure_host_recomputes_on_cpu(test_pack_path, golden_a, fail_at):
    # Call 1 is resident_begin, 2..64 the 32 blocks and their transposes, 65 the
    # mask head.  The provider fails that call as a CUDA error would; the host
    # leaves its resident branch and runs the whole forward on the CPU.
    reply, vocals, err = run_host(DROPIN, test_pack_path, golden_a["audio"],
                                  {"VOCALARC_B200_FAIL_AT": str(fail_at)})
    assert "injected failure" in err
    assert reply["backend"] == "native-cpu"          # the provider disabled itself
    assert snr_db(golden_a["vocals"], vocals) > 100   # the reference CPU path's own result
    assert np.abs(golden_a["vocals"] - vocals).max() < 1e-5


def test_nonresident_transformer_path(test_pack_path, golden_a):
    # VOCALARC_GPU_FULL_BATCHES=0: can_use_full_batches returns 0, the host keeps
    # its CPU grouping and calls native_gpu_transformer once per group of
    # sequences (host buffers in and out; vocalarc_separation.c:846).
    reply, vocals, _ = run_host(DROPIN, test_pack_path, golden_a["audio"], {"VOCALARC_GPU_FULL_BATCHES": "0"})
    assert reply["backend"] == "native-cuda-sm100a"
    assert reply["timeBandGroup"] < 90                 # not the full-batch grouping
    assert snr_db(golden_a["vocals"], vocals) >= SNR_BAR_DB
    assert np.abs(golden_a["vocals"] - vocals).max() <= MAX_ABS_BAR


# ------------------------------------------------------------------ full-device hook
@pytest.mark.parametrize("case", ["clip_a", "cfg1_10s_test"])
def test_hooked_host_runs_whole_forward_on_device(test_pack_path, case):
    path = os.path.join(GOLDEN, f"{case}.npz")
    if not os.path.exists(path):
        pytest.skip(f"{case}.npz not generated")
    g = np.load(path)
    audio = g["audio"] if "audio" in g.files else fixtures.tone_mix(10.0, 0)
    reply, vocals, _ = run_host(HOOK, test_pack_path, audio)
    assert reply["backend"] == "native-cuda-sm100a"
    assert reply["frames"] == audio.shape[1] // 512 + 1
    snr = snr_db(g["vocals"], vocals)
    print(f"{case}: hooked host SNR {snr:.1f} dB, inferenceMs {reply['inferenceMs']}")
    assert snr >= SNR_BAR_DB
    assert np.abs(g["vocals"] - vocals).max() <= MAX_ABS_BAR


def test_hooked_host_falls_back_when_device_forward_fails(test_pack_path, golden_a):
    # Call 1 of the hooked host is vocalarc_b200_separate itself: with it
    # failing, the request runs through forward_model on the CPU.
    reply, vocals, err = run_host(HOOK, test_pack_path, golden_a["audio"], {"VOCALARC_B200_FAIL_AT": "1"})
    assert "injected failure" in err
    assert reply["backend"] == "native-cpu"
    assert snr_db(golden_a["vocals"], vocals) > 100


# ------------------------------------------------------------------ bounded device wait
def test_bounded_wait_runs_out_and_is_reported(capfd, test_pack_blob):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    p = native.Provider(0)
    try:
        assert p.stage_wait_check(0) == -1               # limit out of range
        assert p.stage_wait_check(2000) == 0              # 2 ms limit: the wait runs out
        err = capfd.readouterr().err
        assert "gave up waiting (code 1)" in err         # kErrWaitTma recorded by the kernel
        assert p.backend == "native-cpu"                  # disabled, like any CUDA error
        assert p.stage_wait_check(2000) == 0              # stays disabled
    finally:
        p.close()
    # The context is still usable: a new provider on the same device separates.
    q = native.Provider(0)
    try:
        q.load_model(test_pack_blob)
        g = np.load(os.path.join(GOLDEN, "clip_t2.npz"))
        vocals = q.separate(g["audio"])
        assert snr_db(g["vocals"], vocals) >= SNR_BAR_DB
    finally:
        q.close()


# ------------------------------------------------------------------ batch with WAV I/O off the critical path
def test_separate_files_pipeline(tmp_path, test_pack_blob):
    # Three inputs in three formats through the reader / device / writer
    # pipeline: every vocals file equals the provider's own separation of the
    # decoded input bit for bit, instrumental = mix - vocals, and the PCM16
    # mono 22.05 kHz input matches the reference executable's vocals.
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    g = np.load(os.path.join(GOLDEN, "wav_pcm16_mono_22k.npz"))
    rng = np.random.default_rng(5)
    inputs = [tmp_path / "a.wav", tmp_path / "b.wav", tmp_path / "c.wav"]
    inputs[0].write_bytes(g["wav"].tobytes())
    inputs[1].write_bytes(fixtures.wav_bytes(fixtures.tone_mix(0.7, 3)))
    inputs[2].write_bytes(fixtures.wav_bytes((rng.standard_normal((2, 30000)) * 0.1).astype(np.float32),
                                             rate=48000, bits=24, pcm=True))
    vocals = [tmp_path / f"v{i}.wav" for i in range(3)]
    inst = [tmp_path / f"i{i}.wav" for i in range(3)]
    p = native.Provider(0)
    try:
        p.load_model(test_pack_blob)
        assert p.separate_files([str(x) for x in inputs], [str(x) for x in vocals], [str(x) for x in inst]) == 3
        for i in range(3):
            mix = native.read_track(str(inputs[i]))
            v = fixtures.read_wav_f32(str(vocals[i]))
            assert np.array_equal(v, p.separate(mix))
            assert np.array_equal(fixtures.read_wav_f32(str(inst[i])), (mix - v).astype(np.float32))
        assert snr_db(g["vocals"], fixtures.read_wav_f32(str(vocals[0]))) >= SNR_BAR_DB
        # An unreadable input is skipped and reported; the others are written.
        (tmp_path / "bad.wav").write_bytes(b"not a wav")
        assert p.separate_files([str(tmp_path / "bad.wav"), str(inputs[1])],
                                [str(tmp_path / "vb.wav"), str(tmp_path / "v1b.wav")]) == 1
        assert np.array_equal(fixtures.read_wav_f32(str(tmp_path / "v1b.wav")),
                              fixtures.read_wav_f32(str(vocals[1])))
    finally:
        p.close()


def test_separate_files_chunked_mode(tmp_path, test_pack_blob):
    # chunked = 1: each track goes through the chunked demix, exactly as
    # vocalarc_b200_separate_chunked separates the decoded input.
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    mix = fixtures.long_mix(1.5, seed=12)
    src = tmp_path / "in.wav"
    src.write_bytes(fixtures.wav_bytes(mix, rate=22050, bits=16, pcm=True))
    out = tmp_path / "v.wav"
    p = native.Provider(0)
    try:
        p.load_model(test_pack_blob)
        assert p.separate_files([str(src)], [str(out)], chunked=True) == 1
        decoded = native.read_track(str(src))
        assert np.array_equal(fixtures.read_wav_f32(str(out)), p.separate_chunked(decoded))
    finally:
        p.close()
