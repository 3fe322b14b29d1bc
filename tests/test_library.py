"""The C-ABI library builds, loads and exports every declared entry point (no GPU)."""

import ctypes
import os
import subprocess

import pytest

from karaoke_platform_sidecar_native_b200 import native

REFERENCE_ABI = (
    "native_gpu_create", "native_gpu_destroy", "native_gpu_matmul", "native_gpu_backend",
    "native_gpu_device", "native_gpu_uses_full_batches", "native_gpu_can_use_full_batches",
    "native_gpu_transformer", "native_gpu_resident_begin", "native_gpu_resident_transformer",
    "native_gpu_resident_transpose", "native_gpu_resident_end", "native_gpu_resident_mask",
)


@pytest.fixture(scope="module")
def lib():
    from karaoke_platform_sidecar_native_b200 import build
    build.build()
    return native.load()


def test_reference_abi_declared():
    # native_gpu.h:14-73 of the reference declares exactly these 13 functions.
    declared = native.declared_functions()
    for name in REFERENCE_ABI:
        assert name in declared


def test_every_declared_symbol_exported(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", native.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [name for name in native.declared_functions() if name not in exported]
    assert not missing, missing
    from karaoke_platform_sidecar_native_b200 import stack
    for name in native.declared_functions():
        assert name in native._SIGNATURES or name in stack.STACK_SIGNATURES, f"{name} has no ctypes signature"


def test_library_is_sm100a_and_self_contained(lib):
    # Static CUDA runtime: the only CUDA dependency at load time is the driver.
    deps = subprocess.run(["ldd", native.LIB_PATH], capture_output=True, text=True).stdout
    assert "libcudart" not in deps and "libcublas" not in deps and "libtorch" not in deps
    assert os.path.getsize(native.LIB_PATH) > 100_000


def test_null_provider_strings(lib):
    # NULL-safe static strings like the reference (native_gpu_cuda.cu:847-853).
    assert lib.native_gpu_backend(None) == b"native-cpu"
    assert lib.native_gpu_device(None) == b"none"
    assert lib.native_gpu_uses_full_batches(None) == 0
    assert lib.native_gpu_can_use_full_batches(None, 100) == 0
    assert lib.native_gpu_resident_begin(None, 90, 10, None) == 0
    assert lib.native_gpu_matmul(None, 1, 1, 1, None, None, None, None) == 0


def test_provider_disabled_by_environment(lib):
    # VOCALARC_GPU=off|cpu returns NULL before touching CUDA (native_gpu_cuda.cu:555-556).
    code = ("import ctypes,os;os.environ['VOCALARC_GPU']='off';"
            f"l=ctypes.CDLL({native.LIB_PATH!r});l.native_gpu_create.restype=ctypes.c_void_p;"
            "print(l.native_gpu_create())")
    out = subprocess.run(["python", "-c", code], capture_output=True, text=True, check=True).stdout.strip()
    assert out == "None"
