#!/usr/bin/env python3
"""Apply the guarded full-device hook to a COPY of the reference JSONL host.

    python3 hook_patch.py <checkout>/native/vocalarc_separation.c OUT.c

Used by ``make -C oracle hook`` (the checkout is read, never changed; OUT.c is
written to a temporary directory and deleted after the build).  The three
insertions are the maintainer's hook: with a provider present, the pack is
also loaded into the sm_100a provider's own weight layout, and each
``separate`` request runs the whole forward on the device (STFT, band split,
32 axial blocks, mask head, iSTFT) through ``vocalarc_b200_separate``.  Any 0
return leaves the request on the host's own ``forward_model``, so the JSONL
protocol and the fallback behaviour are unchanged.

Anchors (reference lines): the provider header include (vocalarc_separation.c:30),
the successful ``load`` branch (:1548) and the ``forward_model`` call of
``separate`` (:1585).  Each anchor must occur exactly once.
"""

import sys

INCLUDE_ANCHOR = '#include "native_gpu.h"\n'
LOAD_ANCHOR = "            if (model_load(&network, model_path, argv[0])) {\n"
FORWARD_ANCHOR = ("            if (ok) ok = forward_model(&network, pool, stereo, length, time_group, "
                  "frequency_group, &buffers, &frames);\n")

INCLUDE_HOOK = '#include "vocalarc_b200.h"\n'
LOAD_HOOK = "                if (g_gpu) vocalarc_b200_load_model(g_gpu, network.blob, network.blob_size);\n"
FORWARD_HOOK = (
    "            int on_device = ok && g_gpu && vocalarc_b200_separate(g_gpu, stereo, length, buffers.audio_output);\n"
    "            if (on_device) frames = length / HOP + 1;\n"
    "            else if (ok) ok = forward_model(&network, pool, stereo, length, time_group, frequency_group, "
    "&buffers, &frames);\n")


def patch(source: str) -> str:
    for anchor in (INCLUDE_ANCHOR, LOAD_ANCHOR, FORWARD_ANCHOR):
        if source.count(anchor) != 1:
            raise SystemExit(f"hook_patch: anchor not found exactly once: {anchor.strip()!r}")
    source = source.replace(INCLUDE_ANCHOR, INCLUDE_ANCHOR + INCLUDE_HOOK)
    source = source.replace(LOAD_ANCHOR, LOAD_ANCHOR + LOAD_HOOK)
    return source.replace(FORWARD_ANCHOR, FORWARD_HOOK)


def main() -> None:
    if len(sys.argv) != 3:
        raise SystemExit(__doc__)
    with open(sys.argv[1]) as handle:
        source = handle.read()
    with open(sys.argv[2], "w") as handle:
        handle.write(patch(source))


if __name__ == "__main__":
    main()
