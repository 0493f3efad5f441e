import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "alphafold2-webgpu_b200"))
sys.path.insert(0, str(ROOT / "oracle"))

GOLDEN = ROOT / "tests" / "golden"
GOLDEN_BUNDLES = ["openfold-triangle-small", "af2-short-9", "af2-single-59", "af2-a3m-59"]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and libaf2cuda.so")


@pytest.fixture(scope="session")
def device():
    import af2cuda
    dev = af2cuda.Device(int(os.environ.get("AF2_TEST_DEVICE", "0")))
    yield dev
    dev.close()


def bundle_path(name: str) -> Path:
    return GOLDEN / name / "manifest.json"
