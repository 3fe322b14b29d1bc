"""Golden vectors for the chunk assembly from the reference's Python twin.

The chunked overlap-add, bigshifts and TTA of the ONNX sidecar
(onnx/native/onnx_sidecar.cpp:725-790, :556-575) cannot run here: the sidecar
needs onnxruntime and an exported model.  The reference ships a Python twin of
the same loop, ``onnx/audio.py`` (``demix`` :133-186, ``bigshifts`` :189-210,
``apply_tta`` :213-232), which needs only numpy and torch.  This script imports
that module from the reference checkout, unchanged, and runs it with a
deterministic stand-in for the network (``stand_in_torch``, below), at small chunk
sizes so that many chunks, both padding modes and every batch rule occur in a
few thousand samples.  It writes ``tests/golden/demix_twin.npz``: per case
the twin's output (the input is regenerated from its seed and checked by its
sha256) and the twin's fade ramp per chunk size.

Run where the checkout is present (VOCALARC_REFERENCE, else BASELINE.json's
reference_path):

    python tests/golden/make_demix_twin.py

The twin and the C++ sidecar differ in three places, which the tests state:
the fade ramp (linspace(1, 0, fade) against 1 - i/fade), the first-batch rule
(the twin sets the first chunk/10 samples of the window to 1, which are 1
already, so the rule does nothing; the sidecar sets the whole chunk's weight
to 1), and the sign of the polarity-flipped TTA estimate (the twin subtracts
the estimate of -mix; the sidecar adds it, :572-573).
"""

from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "demix_twin.npz")

#: case -> (chunk, length, model batch, bigshift count (0: demix only), tta, seed)
CASES = {
    "short_b2": (1000, 900, 2, 0, False, 11),        # length <= 2 border: no border padding
    "b1": (1000, 5000, 1, 0, False, 12),             # first batch of one chunk
    "b2": (1000, 5000, 2, 0, False, 13),
    "b3": (1000, 5000, 3, 0, False, 14),
    "one_batch": (1000, 5000, 64, 0, False, 15),     # every chunk in the final batch
    "odd_b2": (999, 4321, 2, 0, False, 16),          # odd chunk (as the real 881,559): step 499, border 500
    "tail_reflect_b2": (1000, 5300, 2, 0, False, 17),  # last chunk longer than half: reflect fill
    "bigshift2_b2": (1000, 4999, 2, 2, False, 18),
    "bigshift3_b2": (999, 4000, 2, 3, False, 19),
    "tta_b2": (1000, 4500, 2, 2, True, 20),
}


def stand_in_numpy(chunk_audio: np.ndarray, ramp: np.ndarray) -> np.ndarray:
    """The stand-in network for one chunk ``[2][chunk]``: a channel mix, a square
    term and a position ramp, with constants exact in float32 so that numpy and
    torch give the same bits."""
    x = chunk_audio.astype(np.float32)
    swapped = x[::-1]
    return ((0.75 * x - 0.25 * swapped) + 0.0625 * (x * x)) + ramp[None, :]


def stand_in_torch(batch, ramp):
    """``stand_in_numpy`` for a torch batch ``[B][2][chunk]``."""
    import torch

    x = batch.to(torch.float32)
    swapped = torch.flip(x, dims=(1,))
    return ((0.75 * x - 0.25 * swapped) + 0.0625 * (x * x)) + torch.from_numpy(ramp)[None, None, :]


def ramp_for(chunk: int) -> np.ndarray:
    return (np.arange(chunk, dtype=np.float32) / np.float32(chunk) * np.float32(0.01)).astype(np.float32)


def mix_for(length: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((2, length)) * 0.3).astype(np.float32)


def reference_root() -> str:
    base = os.environ.get("VOCALARC_REFERENCE")
    if not base:
        with open(os.path.join(ROOT, "BASELINE.json")) as handle:
            base = json.load(handle).get("reference_path")
    if not base or not os.path.isfile(os.path.join(base, "onnx", "audio.py")):
        raise SystemExit("reference checkout with onnx/audio.py not found (set VOCALARC_REFERENCE)")
    return base


def import_twin(base: str):
    """Import onnx/ of the checkout as a package under a private name (its
    modules use relative imports; the name avoids the onnx wheel)."""
    name = "vocalarc_reference_onnx_twin"
    package_dir = os.path.join(base, "onnx")
    spec = importlib.util.spec_from_file_location(name, os.path.join(package_dir, "__init__.py"),
                                                  submodule_search_locations=[package_dir])
    package = importlib.util.module_from_spec(spec)
    sys.modules[name] = package
    spec.loader.exec_module(package)
    audio = importlib.import_module(name + ".audio")
    config = importlib.import_module(name + ".config")
    return audio, config


def main() -> None:
    import torch

    torch.set_num_threads(1)
    audio, config_mod = import_twin(reference_root())
    arrays = {}
    for case, (chunk, length, batch, shifts, tta, seed) in CASES.items():
        config = config_mod.SeparationConfig(chunk_size=chunk, inference_batch_size=batch)
        ramp = ramp_for(chunk)

        def predict(parts, ramp=ramp):
            return stand_in_torch(parts, ramp)

        mix = mix_for(length, seed)
        arrays[f"{case}/mix_sha256"] = np.array(hashlib.sha256(mix.tobytes()).hexdigest())
        # The twin's fade ramp, exactly as its demix builds it (audio.py:154).
        arrays[f"ramp/{chunk}"] = torch.linspace(1.0, 0.0, chunk // 10).numpy().astype(np.float32)
        if shifts == 0:
            arrays[f"{case}/out"] = np.asarray(audio.demix(predict, mix, config), dtype=np.float32)
        elif not tta:
            arrays[f"{case}/out"] = np.asarray(audio.bigshifts(predict, mix, config, shifts), dtype=np.float32)
        else:
            base = np.asarray(audio.bigshifts(predict, mix, config, shifts), dtype=np.float32)
            arrays[f"{case}/base"] = base
            arrays[f"{case}/out"] = np.asarray(audio.apply_tta(predict, mix, base, config, shifts), dtype=np.float32)
            arrays[f"{case}/negated"] = np.asarray(audio.bigshifts(predict, -1.0 * mix, config, shifts),
                                                   dtype=np.float32)
    arrays["cases"] = np.array(json.dumps(CASES))
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT}: {len(CASES)} cases")


if __name__ == "__main__":
    main()
