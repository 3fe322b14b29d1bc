import hashlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from karaoke_platform_sidecar_native_b200 import modelpack  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    # Converted model images of this session go to a private directory, not ~/.cache.
    if "VOCALARC_B200_IMAGE_CACHE" not in os.environ:
        import tempfile
        os.environ["VOCALARC_B200_IMAGE_CACHE"] = tempfile.mkdtemp(prefix="vocalarc_b200_images_")


@pytest.fixture(scope="session")
def test_pack_path():
    return modelpack.pack_path(modelpack.TEST_RECIPE)


@pytest.fixture(scope="session")
def test_pack_blob(test_pack_path):
    with open(test_pack_path, "rb") as handle:
        return handle.read()


@pytest.fixture(scope="session")
def test_model(test_pack_blob):
    return modelpack.parse_pack(test_pack_blob)


@pytest.fixture(scope="session")
def test_pack_sha256(test_pack_blob):
    return hashlib.sha256(test_pack_blob).hexdigest()


GOLDEN = os.path.join(ROOT, "tests", "golden")
