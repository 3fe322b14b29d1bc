#!/usr/bin/env python3
"""Benchmark: audio-seconds separated per second on B200 (BS-RoFormer forward).

Workload (N=1): BASELINE config 2 -- the bundled-layout model (synthetic
weights, seed 0; the real pack is a missing Git-LFS object) on a 240 s stereo
44.1 kHz synthetic mix (seed 1: tones redrawn every 0.5 s, pink noise, 120 BPM
clicks), separated in chunked mode: 27 chunks of 881,559 samples (T = 1,722
frames), overlap 2, linear fade (Separator::demix semantics).  One step = one
full separation of that track.  With N GPUs each rank separates its own
240 s track (seed 1 + rank): weak scaling, no data-path collective.

* ``value``: audio-s/s with the input resident in HBM (device pointers),
  timed with CUDA events on the provider stream, max over ranks.
* ``e2e``: the same through the C-ABI call ``vocalarc_b200_separate_chunked``
  with pinned host buffers (H2D of the mix and D2H of the vocals inside).
* ``roofline``: the dominant kernel from the live launch trace of the timed
  steps; achieved = algorithmic FLOPs (or bytes) per launch / mean launch time.
* ``cpu_baseline``: the unchanged reference CPU executable (built by
  oracle/Makefile) on a bounded sample on this host's cores.

``--impl reference`` times the reference's own CPU implementation (the same
executable) on bounded samples of the workload and prints the same JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from karaoke_platform_sidecar_native_b200 import fixtures, modelpack  # noqa: E402

METRIC = "audio-seconds separated per second (BS-RoFormer vocal separation, 240 s mix, chunked)"
UNIT = "audio_s/s"
REF_EXE = os.path.join(ROOT, "oracle", "_ref", "vocalarc-separation")
CHUNK = 881_559
FRAMES = CHUNK // 512 + 1
BAND_DIMS_SUM = sum(modelpack.BAND_DIMS)


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        p = json.load(open(path))
        return {"hbm_gbs": p["hbm_gbs"], "tflops": p.get("bf16_tflops_sustained", p["bf16_tflops"]),
                "tflops_burst": p["bf16_tflops"],
                "source": "measured (MEASURED_PEAKS.json; sustained bf16 for kernels inside a long step)"}
    return {"hbm_gbs": 6650.0, "tflops": 1400.0, "tflops_burst": 1590.0,
            "source": "fallback (6.65 TB/s, 1.4 PFLOP/s sustained)"}


def chunk_count(length):
    step = CHUNK // 2
    border = CHUNK - step
    padded = length + 2 * border if length > 2 * border else length
    return (padded + step - 1) // step


def kernel_work(name, chunks_per_launch):
    """Algorithmic work of one launch: (kind, amount) with kind 'flop' or 'byte'."""
    c, t = chunks_per_launch, FRAMES
    tokens = c * 90 * t
    flops = {
        "qkv gemm": 2 * tokens * 256 * (1536 + 8),
        "out gemm": 2 * tokens * 512 * 256,

        "ff1 gemm": 2 * tokens * 256 * 1024,
        "ff2 gemm": 2 * tokens * 1024 * 256,
        "ffn": 2 * 2 * tokens * 256 * 1024,
        "attention (L>128)": 4 * 64 * 8 * (c * 90) * t * t,
        "attention (L<=128)": 4 * 64 * 8 * (c * t) * 90 * 90,
        "mask gemm 1": 2 * tokens * 256 * 1024,
        "mask gemm 2": 2 * c * t * 2 * BAND_DIMS_SUM * 1024,
    }
    bytes_ = {
        "row stats": tokens * (256 * 4 + 256 * 2 + 4),
        "stft": c * (2 * CHUNK * 4 + t * 1025 * 16),
        "band split": c * t * (1025 * 16 + 90 * 256 * 4),
        "istft": c * t * (2 * 1025 * 16 + 2 * 2048 * 4),
        "overlap-add": c * (t * 2 * 2048 * 4 + 2 * CHUNK * 4),
    }
    if name in flops:
        return "flop", float(flops[name])
    if name in bytes_:
        return "byte", float(bytes_[name])
    return None, 0.0


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_ids):
        self.bus_ids = {b.lower()[-12:] for b in bus_ids}
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10 or parts[1].lower()[-12:] not in self.bus_ids:
                continue
            try:
                sm.append(float(parts[2]))
                smax.append(float(parts[3]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[6:10]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def reference_cpu_run(pack_path, clips, threads, warmup=1, exe=REF_EXE, env=None, replies=None):
    """Run a reference executable over JSONL on the given clips.

    Returns [(audio_seconds, inference_ms, wall_s)] for the clips after warmup;
    the raw ``separated`` replies are appended to ``replies`` when given.
    """
    results = []
    with tempfile.TemporaryDirectory() as tmp:
        proc = subprocess.Popen([exe, "--model", pack_path, "--threads", str(threads)], stdin=subprocess.PIPE,
                                stdout=subprocess.PIPE, text=True, env=env)

        def request(obj):
            proc.stdin.write(json.dumps(obj) + "\n")
            proc.stdin.flush()
            return json.loads(proc.stdout.readline())

        assert request({"id": 0, "type": "load"})["ok"]
        for i, audio in enumerate(clips):
            wav = os.path.join(tmp, f"in{i}.wav")
            fixtures.write_wav_f32(wav, audio)
            t0 = time.perf_counter()
            reply = request({"id": i + 1, "type": "separate", "inputPath": wav,
                             "vocalsPath": os.path.join(tmp, "v.wav")})
            wall = time.perf_counter() - t0
            assert reply["ok"], reply
            if replies is not None:
                replies.append(reply)
            if i >= warmup:
                results.append((audio.shape[1] / 44100.0, reply["inferenceMs"], wall))
        request({"id": 99, "type": "shutdown"})
        proc.wait(timeout=60)
    return results


REF_TIMER = os.path.join(ROOT, "oracle", "_ref", "ref-stage-timer")
CFG2_CHUNKS = 27


def reference_stage_timing(audio, reps, time_bands, band_frames, threads):
    """The reference CPU forward's own stage functions on one clip, timed by
    oracle/_ref/ref-stage-timer (built from native/vocalarc_separation.c in
    place).  The front (STFT, band split) and back (final norm, mask, iSTFT) run
    in full once; each of `reps` repetitions runs one layer pair on
    `time_bands` bands (time axis) and `band_frames` frames (band axis).
    Returns (frames, fixed_s, [full layer pair seconds per repetition], raw)."""
    pack = modelpack.pack_path(modelpack.BENCH_RECIPE)
    with tempfile.TemporaryDirectory() as tmp:
        wav = os.path.join(tmp, "in.wav")
        fixtures.write_wav_f32(wav, audio)
        proc = subprocess.run([REF_TIMER, "--model", pack, "--wav", wav, "--threads", str(threads), "--reps", str(reps),
                               "--time-bands", str(time_bands), "--band-frames", str(band_frames)],
                              capture_output=True, text=True, check=True)
    lines = [json.loads(x) for x in proc.stdout.splitlines() if x.strip()]
    front, back, layers = lines[0], lines[-1], lines[1:-1]
    frames = front["frames"]
    pairs = [x["time_axis_s"] * 90.0 / x["time_bands"] + x["band_axis_s"] * frames / x["band_frames"] +
             x["transposes_s"] for x in layers]
    fixed = front["stft_s"] + front["band_split_s"] + back["mask_s"] + back["istft_s"]
    return frames, fixed, pairs, {"front": front, "back": back, "layers": layers}


def cfg2_reference_inputs():
    """Chunk 13 of the config-2 track (881,559 samples, T = 1722) and the 10 s config-1 clip."""
    return fixtures.demix_chunk(fixtures.long_mix(240.0, seed=1), 13), fixtures.tone_mix(10.0, seed=0)


def cpu_baseline():
    """The reference CPU forward on this host's cores, on the workload's own unit:
    one T = 1722 chunk of the config-2 mix, front and back end in full, one of
    the 16 layer pairs sampled (a third of its band sequences and frames) and
    scaled; x 27 chunks per 240 s track (extrapolated).  The config-1 10 s
    clip the same way for its latency."""
    if not os.path.exists(REF_TIMER):
        return {"value": None, "unit": UNIT, "cores": 0, "kind": "reference",
                "sample": "reference stage timer not built (make -C oracle timer REF=...)"}
    threads = os.cpu_count() or 1
    chunk, clip = cfg2_reference_inputs()
    frames, fixed, pairs, raw = reference_stage_timing(chunk, 2, 32, 576, threads)
    chunk_s = fixed + 16 * pairs[-1]
    c_frames, c_fixed, c_pairs, _ = reference_stage_timing(clip, 2, 32, 288, threads)
    clip_s = c_fixed + 16 * c_pairs[-1]
    return {"value": 240.0 / (CFG2_CHUNKS * chunk_s), "unit": UNIT, "cores": threads, "kind": "reference",
            "sample": (f"reference CPU forward (native/vocalarc_separation.c stage functions, {threads} threads) on "
                       f"chunk 13 of the cfg2 mix (T={frames}): STFT, band split, mask and iSTFT in full, one layer "
                       f"pair on {raw['layers'][-1]['time_bands']} of 90 bands and "
                       f"{raw['layers'][-1]['band_frames']} of {frames} frames scaled to the full pair, x16 layers, "
                       f"x{CFG2_CHUNKS} chunks per 240 s track (extrapolated)"),
            "chunk_t1722_s_extrapolated": round(chunk_s, 3), "fixed_stages_s": round(fixed, 3),
            "layer_pair_s": round(pairs[-1], 3),
            "clip_10s_ms_extrapolated": round(clip_s * 1000.0, 1)}


def run_reference_arm(args, rank, world):
    """The reference's own CPU implementation on this arm's config: each step
    runs one sampled layer pair of a T = 1722 chunk of the cfg2 mix (a band
    group on the time axis, six frame groups on the band axis), scaled to the
    full pair; the chunk's STFT, band split, mask and iSTFT run in full once.
    A step's time is the extrapolated separation of the 240 s track:
    27 x (fixed stages + 16 x layer pair)."""
    if rank != 0:
        return 0
    if not os.path.exists(REF_TIMER):
        print(json.dumps({"impl": "reference", "unavailable": "reference stage timer not built"}), flush=True)
        return 0
    threads = os.cpu_count() or 1
    chunk, _ = cfg2_reference_inputs()
    t0 = time.perf_counter()
    frames, fixed, pairs, raw = reference_stage_timing(chunk, args.warmup + args.steps, 32, 192, threads)
    wall = time.perf_counter() - t0
    timed = pairs[args.warmup:]
    track_s = [CFG2_CHUNKS * (fixed + 16 * p) for p in timed]
    value = 240.0 * len(track_s) / sum(track_s)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000.0 * sum(track_s) / len(track_s), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"cfg2: 240 s stereo 44.1 kHz mix (seed 1), chunked demix, {CFG2_CHUNKS} chunks x "
                               f"{CHUNK} samples (T={FRAMES}), bundled-layout model with synthetic N(0,0.02) weights",
                   "sample_per_step": (f"one layer pair of chunk 13 (T={frames}) on "
                                       f"{raw['layers'][-1]['time_bands']} of 90 bands and "
                                       f"{raw['layers'][-1]['band_frames']} of {frames} frames, scaled; "
                                       "x16 layers + fixed stages, x27 chunks (extrapolated)")},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference",
                         "sample": "reference CPU stage functions (oracle/_ref/ref-stage-timer), see config"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "fixed_stages_s": round(fixed, 3), "run_wall_s": round(wall, 1),
    }
    print(json.dumps(line), flush=True)
    return 0


REF_CUBLAS_EXE = os.path.join(ROOT, "oracle", "_ref", "vocalarc-separation-cublas")


def reference_gpu_baseline(device, reps=3):
    """The reference's optional GPU build (native_gpu_cuda.cu: cuBLAS SGEMM and
    its own SIMT kernels, compiled unchanged for sm_100a by oracle/Makefile) on
    this B200, with VOCALARC_GPU_TF32=1 and =0: the config-1 10 s clip
    (whole clip, T = 862; p50 of `reps` inferenceMs and wall) and one
    881,559-sample chunk of the config-2 mix (T = 1722).  Its host still runs
    the STFT, band split and iSTFT on the CPU, which inferenceMs includes."""
    if not os.path.exists(REF_CUBLAS_EXE):
        return {"unavailable": "reference cuBLAS build not built (make -C oracle cublas)"}
    threads = os.cpu_count() or 1
    pack = modelpack.pack_path(modelpack.BENCH_RECIPE)
    clip = fixtures.tone_mix(10.0, seed=0)
    chunk = fixtures.demix_chunk(fixtures.long_mix(240.0, seed=1), 13)
    out = {"exe": "native/vocalarc_separation.c + native/native_gpu_cuda.cu (cuBLAS), unchanged, sm_100a",
           "device": device, "threads": threads}
    # The reference build uses device 0 of what it sees: show it only this
    # process's GPU (an entry of an inherited CUDA_VISIBLE_DEVICES list, if any).
    visible = [v for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    own = visible[device] if device < len(visible) else str(device)
    for tf32 in ("1", "0"):
        env = dict(os.environ, VOCALARC_GPU_TF32=tf32, CUDA_VISIBLE_DEVICES=own)
        replies = []
        res = reference_cpu_run(pack, [clip] * (reps + 1) + [chunk], threads, warmup=1, exe=REF_CUBLAS_EXE, env=env,
                                replies=replies)
        clip_ms = [r[1] for r in res[:reps]]
        clip_wall = [r[2] * 1000.0 for r in res[:reps]]
        chunk_ms = res[reps][1]
        key = "tf32" if tf32 == "1" else "fp32"
        out[key] = {
            "backend": replies[-1].get("backend"),
            "clip_10s_inference_ms_p50": round(float(np.median(clip_ms)), 1),
            "clip_10s_wall_ms_p50": round(float(np.median(clip_wall)), 1),
            "clip_10s_realtime_x": round(10.0 / (float(np.median(clip_ms)) / 1000.0), 2),
            "chunk_t1722_inference_ms": round(chunk_ms, 1),
            "cfg2_audio_s_per_s_extrapolated": round(240.0 / (27 * chunk_ms / 1000.0), 3),
        }
    return out


def traffic_per_launch(kernel):
    """DRAM bytes per launch of `kernel` at the bench's shape, from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.startswith(kernel + "\t"):
            try:
                return float(line.split("\t")[1])
            except (IndexError, ValueError):
                return None
    return None


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=5)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", default="ours", choices=("ours", "reference"))
    parser.add_argument("--seconds", type=float, default=240.0)
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-latency", action="store_true", help="skip the 10 s clip latency measurement")
    parser.add_argument("--no-batch", action="store_true", help="skip the config-5 batch (64 x 180 s tracks)")
    parser.add_argument("--no-strong", action="store_true", help="skip one track sharded across the ranks")
    parser.add_argument("--no-gpu-baseline", action="store_true", help="skip the reference cuBLAS build (N=1)")
    parser.add_argument("--gpu-baseline-only", action="store_true",
                        help="print only the reference cuBLAS build's timings on GPU 0")
    parser.add_argument("--precision", default="fp16", choices=("fp16", "bf16"))
    parser.add_argument("--ops", action="store_true",
                        help="config-4 op-level lines: time/band attention, STFT, band split")
    parser.add_argument("--shard", action="store_true",
                        help="strong scaling: one track's chunks sharded across the ranks, seams by CUDA IPC")
    parser.add_argument("--stack", action="store_true",
                        help="config 3: dim-512 / 62-band / hop-441 / GEGLU stack, 16 x 8 s clips, bf16")
    parser.add_argument("--sp", action="store_true",
                        help="10 s clip latency with the clip split across every visible GPU (one process)")
    parser.add_argument("--clips", type=int, default=0, help="--stack: clips per forward (default 16)")
    parser.add_argument("--depth", type=int, default=0, help="--stack: layers (default 12; fewer for profiling)")
    args = parser.parse_args()
    args.warmup = max(3, args.warmup)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference_arm(args, rank, world)
    if args.gpu_baseline_only:
        print(json.dumps({"gpu_baseline": reference_gpu_baseline(0)}), flush=True)
        return 0
    if args.shard:
        return run_shard(args, rank, world, local_rank)
    if args.ops:
        return run_ops(args)
    if args.stack:
        return run_stack(args)
    if args.sp:
        return run_sp(args)

    import torch
    import torch.distributed as dist

    from karaoke_platform_sidecar_native_b200 import native

    torch.cuda.set_device(local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local_rank))
    # Host-side channel of the chunk scheduler (64-byte IPC handles, barriers).
    gloo = dist.new_group(backend="gloo") if world > 1 else None

    provider = native.Provider(local_rank)
    if args.precision == "bf16":
        provider.set_precision(True)
    pack = modelpack.synthetic_pack(**modelpack.BENCH_RECIPE)
    t_load = time.perf_counter()
    provider.load_model(pack)
    model_load = {"ms": round((time.perf_counter() - t_load) * 1000.0, 1), "from_cache": provider.model_from_cache,
                  "pack_bytes": len(pack)}
    length = int(args.seconds * 44100)
    audio = fixtures.long_mix(args.seconds, seed=1 + rank)
    d_audio = torch.from_numpy(audio).cuda()
    d_vocals = torch.empty_like(d_audio)
    stream = torch.cuda.ExternalStream(provider.stream)

    def step():
        provider.separate_device(d_audio, 1, length, d_vocals, chunked=True, chunk=CHUNK, model_batch=1)

    torch.cuda.synchronize()
    for _ in range(args.warmup):
        step()
    provider.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- device-resident timed region
    props = torch.cuda.get_device_properties(local_rank)
    bus = "%08X:%02X:%02X.0" % (getattr(props, "pci_domain_id", 0), getattr(props, "pci_bus_id", 0),
                                getattr(props, "pci_device_id", 0))
    sampler = ClockSampler([bus])
    barrier()
    torch.cuda.synchronize()
    provider.synchronize()
    sampler.start()
    launches0 = provider.launch_count
    provider.trace_begin()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        step()
    stop.record(stream)
    trace = provider.trace_end()
    provider.synchronize()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    launches = provider.launch_count - launches0
    elapsed_ms = start.elapsed_time(stop)
    t = torch.tensor([elapsed_ms], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms = float(t.item())
    value = world * args.seconds * args.steps / (elapsed_ms / 1000.0)

    # ---- end to end through the C-ABI with pinned host buffers
    host_in = torch.from_numpy(audio).pin_memory()
    host_out = torch.empty_like(host_in).pin_memory()
    in_np = host_in.numpy()
    out_np = host_out.numpy()
    lib = provider.lib
    e2e_steps = max(1, min(args.steps, 3))
    barrier()
    e_start = torch.cuda.Event(enable_timing=True)
    e_stop = torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for _ in range(e2e_steps):
        ok = lib.vocalarc_b200_separate_chunked(provider.handle, native.fptr(in_np), length, CHUNK, 1,
                                                native.fptr(out_np))
        if not ok:
            raise RuntimeError("vocalarc_b200_separate_chunked failed")
    e_stop.record(stream)
    torch.cuda.synchronize()
    e_ms = e_start.elapsed_time(e_stop)
    t = torch.tensor([e_ms], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e_ms = float(t.item())
    e2e_value = world * args.seconds * e2e_steps / (e_ms / 1000.0)
    if not np.isfinite(out_np).all():
        raise RuntimeError("non-finite vocals")
    latency = clip_latency(provider, stream) if rank == 0 and not args.no_latency else None
    parity = bench_parity(provider, audio) if rank == 0 and args.seconds == 240.0 else None
    batch = None if args.no_batch else cfg5_batch(provider, stream, rank, world)
    strong = None if args.no_strong else strong_one_track(provider, stream, rank, world, gloo)
    gpu_base = None
    if world == 1 and not args.no_gpu_baseline:
        gpu_base = reference_gpu_baseline(local_rank)

    if rank == 0:
        peaks = load_peaks()
        chunks = chunk_count(length)
        kernels = []
        for name, (count, ms) in sorted(trace.items(), key=lambda kv: -kv[1][1]):
            kind, work = kernel_work(name, chunks)
            per_launch_ms = ms / max(1, count)
            entry = {"kernel": name, "launches": count, "total_ms": round(ms, 3),
                     "share": round(ms / max(1e-9, sum(v[1] for v in trace.values())), 4)}
            if kind == "flop":
                ach = work / (per_launch_ms / 1000.0) / 1e12
                entry.update(achieved_tflops=round(ach, 1), frac=round(ach / peaks["tflops"], 3))
            elif kind == "byte":
                ach = work / (per_launch_ms / 1000.0) / 1e9
                entry.update(achieved_gbs=round(ach, 1), frac=round(ach / peaks["hbm_gbs"], 3))
            kernels.append(entry)
        dominant = next((k for k in kernels if "frac" in k), None)
        roofline = None
        if dominant is not None:
            kind, work = kernel_work(dominant["kernel"], chunks)
            per_launch_s = dominant["total_ms"] / dominant["launches"] / 1000.0
            if kind == "flop":
                ach = work / per_launch_s / 1e12
                roofline = {"kernel": dominant["kernel"], "bound": "tensor", "achieved": round(ach, 1),
                            "peak": peaks["tflops"], "unit": "TFLOP/s", "frac": round(ach / peaks["tflops"], 4),
                            "traffic": traffic_per_launch(dominant["kernel"]), "peak_source": peaks["source"],
                            "work_per_launch": work}
            else:
                ach = work / per_launch_s / 1e9
                roofline = {"kernel": dominant["kernel"], "bound": "hbm", "achieved": round(ach, 1),
                            "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(ach / peaks["hbm_gbs"], 4),
                            "traffic": traffic_per_launch(dominant["kernel"]), "peak_source": peaks["source"],
                            "work_per_launch": work}
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline()
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(elapsed_ms / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": args.precision, "data": "synthetic",
            "config": {"workload": "cfg2: 240 s stereo 44.1 kHz mix (seed 1 + rank), chunked demix, "
                                   f"{chunks} chunks x {CHUNK} samples (T={FRAMES}), bundled-layout model with "
                                   "synthetic N(0,0.02) weights",
                       "chunks_per_step": chunks, "audio_seconds_per_step_per_gpu": args.seconds,
                       "l2": "inputs and workspace (~1 GB per chunk) far larger than the 126 MB L2; no flush",
                       "parallelism": f"weak: one track per GPU x{world}"},
            "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": int(audio.nbytes),
                    "d2h_bytes_per_step": int(audio.nbytes), "steps": e2e_steps,
                    "api": "vocalarc_b200_separate_chunked (C-ABI, pinned host buffers)"},
            "gpu_launches": int(launches),
            "parity": parity,
            "model_load": model_load,
            "latency_10s_clip": latency,
            "batch_cfg5": batch,
            "strong_one_track": strong,
            "gpu_baseline": gpu_base,
            "roofline": roofline,
            "kernels": kernels,
            "cpu_baseline": cpu,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    provider.close()
    return 0


GOLDEN_CHUNK = os.path.join(ROOT, "tests", "golden", "cfg2_chunk13_bench.npz")


def bench_parity(provider, audio):
    """Parity of the benchmark's own forward batch at its own size: the 27
    padded chunks of this rank's track through the whole-clip forward in one
    device call (the chunked step without its overlap-add, same batch), chunk
    13 against the vocals the unchanged reference CPU executable wrote for the
    same chunk with the same pack (tests/golden/cfg2_chunk13_bench.npz)."""
    import torch

    if not os.path.exists(GOLDEN_CHUNK):
        return {"checked": False, "why": "golden cfg2_chunk13_bench.npz missing"}
    golden = np.load(GOLDEN_CHUNK)
    count = fixtures.demix_chunk_count(audio.shape[1], CHUNK)
    chunks = np.stack([fixtures.demix_chunk(audio, c, CHUNK) for c in range(count)])
    d_in = torch.from_numpy(chunks).cuda()
    d_out = torch.empty_like(d_in)
    provider.separate_device(d_in, count, CHUNK, d_out)
    provider.synchronize()
    out = d_out[13].cpu().numpy().astype(np.float64)
    ref = golden["vocals"].astype(np.float64)
    err = ref - out
    snr = 10 * np.log10((ref ** 2).sum() / max((err ** 2).sum(), 1e-300))
    del d_in, d_out
    return {"checked": True, "vs": "reference CPU executable, chunk 13 of the cfg2 track (T=1722), same pack",
            "batch": count, "snr_db": round(float(snr), 2), "max_abs": float(np.abs(err).max()),
            "bar": {"snr_db": 50.0, "max_abs": 2e-3}, "pass": bool(snr >= 50.0 and np.abs(err).max() <= 2e-3)}


def tone_mix_device(seconds, seed, device):
    """Config-5 recipe (the tone mix of config 1) generated on the device: f0
    and phases drawn from numpy PCG64(seed) exactly as fixtures.tone_mix draws
    them, the white noise from torch's CUDA generator seeded with `seed` (same
    distribution, different samples from the CPU fixture)."""
    import torch

    rng = np.random.default_rng(seed)
    n = int(round(seconds * 44100))
    f0 = rng.uniform(100.0, 800.0, size=3)
    phase = rng.uniform(0.0, 2.0 * np.pi, size=3)
    t = torch.arange(n, dtype=torch.float64, device=device) / 44100.0
    tone = torch.zeros(n, dtype=torch.float64, device=device)
    for j in range(3):
        for k in range(1, 7):
            tone += torch.sin(2.0 * np.pi * k * float(f0[j]) * t + k * float(phase[j])) / k
    tone *= 0.2 / max(float(tone.abs().max()), 1e-12)
    gen = torch.Generator(device=device).manual_seed(int(seed))
    noise = torch.randn(2, n, generator=gen, device=device, dtype=torch.float32) * 0.05
    return tone.float()[None, :] + noise


def cfg5_batch(provider, stream, rank, world, tracks=64, seconds=180.0, first_seed=100):
    """Config 5: `tracks` independent 180 s tone mixes (seeds 100..163), split
    in contiguous blocks over the ranks; each rank separates its block in one
    chunked device call (21 chunks per track).  One timed pass; the job time
    is the max over ranks."""
    import torch
    import torch.distributed as dist

    lo, hi = tracks * rank // world, tracks * (rank + 1) // world
    length = int(round(seconds * 44100))
    d_in = torch.empty(max(1, hi - lo), 2, length, device="cuda")
    for i in range(lo, hi):
        d_in[i - lo] = tone_mix_device(seconds, first_seed + i, d_in.device)
    d_out = torch.empty_like(d_in)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    if hi > lo:
        provider.separate_device(d_in, hi - lo, length, d_out, chunked=True, chunk=CHUNK, model_batch=1)
    b.record(stream)
    provider.synchronize()
    torch.cuda.synchronize()
    ms = torch.tensor([a.elapsed_time(b)], device="cuda")
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    finite = bool(torch.isfinite(d_out).all().item())
    del d_in, d_out
    return {"tracks": tracks, "seconds_per_track": seconds, "tracks_per_rank": f"{tracks // world}-{-(-tracks // world)}",
            "chunks_per_track": chunk_count(length), "value": round(tracks * seconds / (ms / 1000.0), 2),
            "unit": UNIT, "ms": round(ms, 1), "finite": finite,
            "data": "seeded tone mixes generated on the device (f0/phase from numpy PCG64(seed), noise from the "
                    "CUDA generator)"}


def strong_one_track(provider, stream, rank, world, gloo, reps=2):
    """One 240 s track (seed 1) with its 27 chunks sharded across the ranks:
    contiguous ranges of >= 2 chunks, the overlap-add seam of each range
    boundary pulled by the next rank over NVLink (CUDA IPC peer copy), every
    rank writing its own output samples.  Per rank the phases are timed on the
    host around the synchronous calls: forward of the range, seam exchange
    (handle all-gather + peer copy), finish; the max over ranks is reported.
    The limiter is chunk granularity: the busiest rank runs ceil-ish(27/N)
    chunks of the 27, a ceiling of 27 / max chunks per rank."""
    import torch
    import torch.distributed as dist

    from karaoke_platform_sidecar_native_b200 import native, shard

    audio = fixtures.long_mix(240.0, seed=1)
    length = audio.shape[1]
    d_audio = torch.from_numpy(audio).cuda()
    d_vocals = torch.zeros_like(d_audio)
    plan = native.chunk_plan(length, CHUNK)
    ranges = shard.chunk_ranges(plan["chunks"], world)
    c0, c1 = ranges[rank]
    phases = np.zeros(4)

    def one():
        if world == 1:
            t = time.perf_counter()
            provider.separate_device(d_audio, 1, length, d_vocals, chunked=True, chunk=CHUNK, model_batch=1)
            provider.synchronize()
            return np.array([time.perf_counter() - t, 0.0, 0.0, time.perf_counter() - t])
        t0 = time.perf_counter()
        if c1 > c0:
            provider.range_forward(d_audio, length, c0, c1, CHUNK, 1)
        t1 = time.perf_counter()
        handle = provider.range_seam_export() if c1 > c0 and c1 < plan["chunks"] else None
        handles = [None] * world
        dist.all_gather_object(handles, handle, group=gloo)
        if c1 > c0 and c0 > 0:
            provider.range_seam_import(handles[rank - 1])
        provider.synchronize()
        t2 = time.perf_counter()
        if c1 > c0:
            provider.range_finish(d_vocals)
            provider.synchronize()
        t3 = time.perf_counter()
        dist.barrier(group=gloo)
        return np.array([t1 - t0, t2 - t1, t3 - t2, time.perf_counter() - t0])

    one()                                   # warm-up (range workspace sizes)
    if world > 1:
        dist.barrier()
    for _ in range(reps):
        phases += one()
    phases /= reps
    t = torch.tensor(phases, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    phases = t.cpu().numpy()
    busiest = max(b - a for a, b in ranges)
    del d_audio, d_vocals
    return {"track_seconds": 240.0, "chunks": plan["chunks"], "ranges": ranges, "value": round(240.0 / phases[3], 2),
            "unit": UNIT, "ms_per_track": round(phases[3] * 1000.0, 1),
            "phase_ms_max_over_ranks": {"range_forward": round(phases[0] * 1000.0, 1),
                                        "seam_exchange": round(phases[1] * 1000.0, 1),
                                        "finish": round(phases[2] * 1000.0, 1)},
            "granularity_ceiling_x": round(plan["chunks"] / busiest, 3), "busiest_rank_chunks": busiest,
            "exchange": "CUDA IPC peer copy of one [3][seam] fp32 buffer per range boundary (NVLink), handles over gloo",
            "timing": "host wall clock around the synchronous calls, mean of 2 passes, max over ranks"}


def clip_latency(provider, stream, reps=20):
    """p50 / p90 latency of one 10 s clip (config 1: seed-0 tone mix), whole-clip
    forward (T = 862), 1 GPU: through the C-ABI call vocalarc_b200_separate
    with host buffers (wall clock around the synchronous call) and on device
    memory (CUDA events on the provider stream)."""
    import torch

    from karaoke_platform_sidecar_native_b200 import native

    clip = np.ascontiguousarray(fixtures.tone_mix(seconds=10.0, seed=0), dtype=np.float32)
    out = np.zeros_like(clip)
    length = clip.shape[1]
    d_clip = torch.from_numpy(clip).cuda()
    d_out = torch.empty_like(d_clip)
    for _ in range(3):
        provider.lib.vocalarc_b200_separate(provider.handle, native.fptr(clip), length, native.fptr(out))
    wall, dev = [], []
    for _ in range(reps):
        t = time.perf_counter()
        if not provider.lib.vocalarc_b200_separate(provider.handle, native.fptr(clip), length, native.fptr(out)):
            raise RuntimeError("vocalarc_b200_separate failed")
        wall.append((time.perf_counter() - t) * 1000.0)
    for _ in range(reps):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        provider.separate_device(d_clip, 1, length, d_out)
        b.record(stream)
        torch.cuda.synchronize()
        dev.append(a.elapsed_time(b))
    q = lambda v, p: round(float(np.percentile(v, p)), 3)
    return {"clip": "cfg1: 10 s stereo 44.1 kHz tone mix (seed 0), whole clip, T = 862", "reps": reps,
            "e2e_ms_p50": q(wall, 50), "e2e_ms_p90": q(wall, 90), "device_ms_p50": q(dev, 50),
            "device_ms_p90": q(dev, 90), "api": "vocalarc_b200_separate (host buffers, synchronous)"}


def run_ops(args):
    """Config 4 (op-level microbenchmarks, seeded N(0,1) inputs in bf16), one JSON
    line per op: time-axis attention 992 seq x 801 tokens x 8 x 64, band-axis
    attention 12816 seq x 62 tokens, STFT of 16 x 2 channels x 801 frames
    (2048-point real FFTs; the bundled hop of 512), band split of 16 x 801
    frames (the bundled 90-band layout).  Inputs are larger than L2."""
    import torch

    from karaoke_platform_sidecar_native_b200 import native

    peaks = load_peaks()
    p = native.Provider(0)
    p.set_precision(True)
    stream = torch.cuda.ExternalStream(p.stream)
    g = torch.Generator(device="cuda").manual_seed(4)

    def timed(fn, steps):
        for _ in range(max(3, args.warmup)):
            fn()
        p.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(steps):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / steps

    lines = []
    d1, d2, d3 = 801, 62, 16
    rows = d1 * d2 * d3
    qkv = torch.randn(rows, 1536, device="cuda", generator=g).bfloat16()
    gates = torch.rand(rows, 8, device="cuda", generator=g)
    out = torch.empty(rows, 512, device="cuda", dtype=torch.bfloat16)
    for name, pos, seqs, length in (("time-axis attention", 1, d2 * d3, d1), ("band-axis attention", 2, d1 * d3, d2)):
        ms = timed(lambda: p.stage_attention(qkv, gates, out, d1, d2, d3, pos), max(5, args.steps))
        flop = 4.0 * length * length * 64 * 8 * seqs
        byts = rows * (1536 + 512) * 2 + rows * 8 * 4
        line = {"op": f"{name}, {seqs} seq x {length} tokens x 8 heads x 64, bf16", "ms": round(ms, 4),
                "tflops": round(flop / ms / 1e9, 1), "gbs": round(byts / ms / 1e6, 1),
                "roofline": ({"bound": "tensor", "frac": round(flop / ms / 1e9 / peaks["tflops_burst"], 4),
                              "peak_tflops": peaks["tflops_burst"]} if pos == 1 else
                             {"bound": "hbm", "frac": round(byts / ms / 1e6 / peaks["hbm_gbs"], 4),
                              "peak_gbs": peaks["hbm_gbs"]})}
        lines.append(line)
    del qkv, out, gates
    frames = 801
    length = (frames - 1) * 512
    audio = torch.randn(16, 2, length, device="cuda", generator=g)
    spec = torch.empty(16, frames, 1025, 2, 2, device="cuda")
    ms = timed(lambda: p.stage_stft(audio, 16, length, spec), max(5, args.steps))
    byts = audio.numel() * 4 + spec.numel() * 4
    lines.append({"op": "STFT, 16 x 2 x 801 frames of 2048-point real FFT", "ms": round(ms, 4),
                  "gbs": round(byts / ms / 1e6, 1),
                  "roofline": {"bound": "hbm", "frac": round(byts / ms / 1e6 / peaks["hbm_gbs"], 4),
                               "peak_gbs": peaks["hbm_gbs"]}})
    x = torch.empty(16 * 90 * frames, 256, device="cuda")
    p.load_model(modelpack.synthetic_pack(**modelpack.BENCH_RECIPE))
    ms = timed(lambda: p.stage_band_split(spec, 16, frames, x), max(5, args.steps))
    byts = spec.numel() * 4 + x.numel() * 4
    lines.append({"op": "band split (RMSNorm + Linear per band), 16 x 801 frames, 90 bundled bands", "ms": round(ms, 4),
                  "gbs": round(byts / ms / 1e6, 1),
                  "roofline": {"bound": "hbm", "frac": round(byts / ms / 1e6 / peaks["hbm_gbs"], 4),
                               "peak_gbs": peaks["hbm_gbs"]}})
    for line in lines:
        line.update({"config": "cfg4 op-level", "data": "synthetic N(0,1)", "dtype": "bf16"})
        print(json.dumps(line), flush=True)
    p.close()
    return 0


def run_stack(args):
    """Config 3, the layer-level tensor-core benchmark: the configurable stack at
    dim 512, depth 12, 8 x 64 heads, GEGLU FFN (mult 4), 62 bands, hop 441, bf16
    operands (random N(0, 0.02) weights, seed 2) on 16 clips of 8 s seeded
    Gaussian stereo audio (sigma 0.1).  One step = the whole forward of the 16
    clips (STFT to iSTFT).  value: audio-s/s with the clips resident in HBM;
    e2e: vocalarc_b200_stack_separate from pinned host buffers."""
    import torch

    from karaoke_platform_sidecar_native_b200 import native, stack as st

    cfg = st.CONFIG3.replace(depth=args.depth) if args.depth > 0 else st.CONFIG3
    clips, length = (args.clips if args.clips > 0 else st.CONFIG3_CLIPS), st.CONFIG3_CLIP
    frames = cfg.frames(length)
    s = st.Stack(cfg, st.synthetic_weights(cfg, seed=2))
    rng = np.random.default_rng(2)
    audio = (rng.standard_normal((clips, 2, length), dtype=np.float32) * np.float32(0.1))
    d_audio = torch.from_numpy(audio).cuda()
    d_vocals = torch.empty_like(d_audio)
    stream = torch.cuda.ExternalStream(s.stream)

    def step():
        s.forward_device(d_audio, clips, length, d_vocals)

    torch.cuda.synchronize()
    for _ in range(args.warmup):
        step()
    s.synchronize()
    props = torch.cuda.get_device_properties(0)
    bus = "%08X:%02X:%02X.0" % (getattr(props, "pci_domain_id", 0), getattr(props, "pci_bus_id", 0),
                                getattr(props, "pci_device_id", 0))
    sampler = ClockSampler([bus])
    sampler.start()
    launches0 = s.launch_count
    s.trace_begin()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        step()
    b.record(stream)
    trace = s.trace_end()
    s.synchronize()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = a.elapsed_time(b) / args.steps
    launches = s.launch_count - launches0
    audio_s = clips * length / 44100.0
    flops = st.forward_flops(cfg, clips, frames)
    peaks = load_peaks()
    kernels = []
    total = sum(v[1] for v in trace.values())
    split_bytes = clips * frames * (1025 * 16 + cfg.bands * cfg.dim * 4)   # band split is fp32 SIMT: HBM-bound
    for name, (count, kms) in sorted(trace.items(), key=lambda kv: -kv[1][1]):
        entry = {"kernel": name, "launches": count, "total_ms": round(kms, 3), "share": round(kms / total, 4)}
        if name == "band split" and kms > 0:
            ach = split_bytes * args.steps / (kms / 1000.0) / 1e9
            entry.update(achieved_gbs=round(ach, 1), frac=round(ach / peaks["hbm_gbs"], 3))
        elif name in flops and kms > 0:
            ach = flops[name] * args.steps / (kms / 1000.0) / 1e12
            entry.update(achieved_tflops=round(ach, 1), frac=round(ach / peaks["tflops"], 3))
        kernels.append(entry)
    all_flop = sum(flops.values())
    dominant = next(k for k in kernels if "achieved_tflops" in k)
    # End to end from pinned host memory through the C-ABI.
    host_in = torch.from_numpy(audio).pin_memory()
    host_out = torch.empty_like(host_in).pin_memory()
    e_steps = max(1, min(args.steps, 3))
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(e_steps):
        ok = s.lib.vocalarc_b200_stack_separate(s.handle, native.fptr(host_in.numpy()), clips, length,
                                                native.fptr(host_out.numpy()))
        if not ok:
            raise RuntimeError("vocalarc_b200_stack_separate failed")
    t1.record(stream)
    torch.cuda.synchronize()
    e_ms = t0.elapsed_time(t1) / e_steps
    if not np.isfinite(host_out.numpy()).all():
        raise RuntimeError("non-finite vocals")
    line = {
        "metric": "audio-seconds separated per second (config 3 stack forward)", "value": round(audio_s / (ms / 1000), 2),
        "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"cfg3: dim 512, depth {cfg.depth}, 8x64 heads, GEGLU mult 4, 62 bands, n_fft 2048, "
                               f"hop 441, {clips} clips x 8 s (801 frames) Gaussian sigma 0.1, N(0,0.02) weights seed 2",
                   "tokens_per_axis": clips * cfg.bands * frames,
                   "l2": "activations (~7 GB) far larger than the 126 MB L2; no flush"},
        "forward_tflops": round(all_flop / (ms / 1000) / 1e12, 1),
        "roofline": {"kernel": dominant["kernel"], "bound": "tensor", "achieved": dominant["achieved_tflops"],
                     "peak": peaks["tflops"], "unit": "TFLOP/s", "frac": dominant["frac"],
                     "peak_source": peaks["source"], "traffic": None},
        "e2e": {"value": round(audio_s / (e_ms / 1000), 2), "unit": UNIT, "h2d_bytes_per_step": int(audio.nbytes),
                "d2h_bytes_per_step": int(audio.nbytes), "api": "vocalarc_b200_stack_separate (pinned host buffers)"},
        "gpu_launches": int(launches), "kernels": kernels, "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    s.close()
    return 0


def run_sp(args, reps=20):
    """Latency of one 10 s clip (config 1, seed 0, whole clip) with its forward
    split across all visible GPUs by vocalarc_b200_separate_sp (time-axis
    blocks on band ranges, band-axis blocks on frame ranges), against the same
    clip on GPU 0 alone.  One process drives every GPU; wall clock around the
    synchronous C-ABI calls, host buffers."""
    import torch

    from karaoke_platform_sidecar_native_b200 import native

    n = torch.cuda.device_count()
    pack = modelpack.synthetic_pack(**modelpack.BENCH_RECIPE)
    providers = []
    for d in range(n):
        p = native.Provider(d)
        p.load_model(pack)
        providers.append(p)
    clip = np.ascontiguousarray(fixtures.tone_mix(seconds=10.0, seed=0), dtype=np.float32)

    def timed(fn):
        for _ in range(max(3, args.warmup)):
            fn()
        out = []
        for _ in range(reps):
            t = time.perf_counter()
            fn()
            out.append((time.perf_counter() - t) * 1000.0)
        return round(float(np.percentile(out, 50)), 3), round(float(np.percentile(out, 90)), 3)

    one = timed(lambda: providers[0].separate(clip))
    split = timed(lambda: native.separate_sp(providers, clip))
    same = bool(np.array_equal(native.separate_sp(providers, clip), providers[0].separate(clip)))
    print(json.dumps({"metric": "p50 latency of one 10 s clip, whole-clip forward split across GPUs",
                      "unit": "ms", "n_gpus": n, "higher_is_better": False, "data": "synthetic",
                      "split_ms_p50": split[0], "split_ms_p90": split[1], "one_gpu_ms_p50": one[0],
                      "one_gpu_ms_p90": one[1], "bit_identical_to_one_gpu": same, "reps": reps,
                      "config": {"workload": "cfg1: 10 s stereo 44.1 kHz tone mix (seed 0), T = 862, bundled-layout "
                                             "model, synthetic N(0,0.02) weights",
                                 "api": "vocalarc_b200_separate_sp vs vocalarc_b200_separate (host buffers)"}}),
          flush=True)
    for p in providers:
        p.close()
    return 0


def run_shard(args, rank, world, local_rank):
    """One cfg2 track, its chunks split across the ranks (chunk scheduler).

    Each rank runs its chunk range, the overlap-add seams cross by CUDA IPC peer
    copy and every rank writes its own output samples.  The process group is
    gloo: it carries only the 64-byte IPC handles, barriers and the timing max.
    A step is the whole track; the timed region per rank is CUDA events on the
    provider stream bracketing the step (host waits for neighbours included).
    """
    import torch
    import torch.distributed as dist

    from karaoke_platform_sidecar_native_b200 import native, shard

    torch.cuda.set_device(local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("gloo", timeout=timedelta(seconds=300))
    provider = native.Provider(local_rank)
    if args.precision == "bf16":
        provider.set_precision(True)
    provider.load_model(modelpack.synthetic_pack(**modelpack.BENCH_RECIPE))
    length = int(args.seconds * 44100)
    audio = fixtures.long_mix(args.seconds, seed=1)
    d_audio = torch.from_numpy(audio).cuda()
    d_vocals = torch.zeros_like(d_audio)
    plan = native.chunk_plan(length, CHUNK)
    stream = torch.cuda.ExternalStream(provider.stream)

    def step():
        if world > 1:
            return shard.separate_range(provider, d_audio, length, rank, world, chunk=CHUNK, d_vocals=d_vocals,
                                        plan=plan)
        provider.separate_device(d_audio, 1, length, d_vocals, chunked=True, chunk=CHUNK, model_batch=1)
        provider.synchronize()
        return (0, length)

    torch.cuda.synchronize()
    for _ in range(args.warmup):
        step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    launches0 = provider.launch_count
    start.record(stream)
    for _ in range(args.steps):
        owned = step()
    stop.record(stream)
    torch.cuda.synchronize()
    launches = provider.launch_count - launches0
    elapsed_ms = start.elapsed_time(stop)
    t = torch.tensor([elapsed_ms])
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms = float(t.item())
    value = args.seconds * args.steps / (elapsed_ms / 1000.0)
    ranges = shard.chunk_ranges(plan["chunks"], world)
    if rank == 0:
        line = {
            "metric": METRIC + " [one track sharded]", "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(elapsed_ms / args.steps, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": args.precision,
            "data": "synthetic",
            "config": {"workload": f"cfg2: one {args.seconds:g} s track, {plan['chunks']} chunks sharded as {ranges}",
                       "seam_samples": plan["seam"], "exchange": "CUDA IPC peer copy of one 3 x seam fp32 buffer "
                                                               "per range boundary",
                       "parallelism": f"chunk ranges x{world}"},
            "gpu_launches": int(launches), "rank0_owned_samples": list(owned),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    provider.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
