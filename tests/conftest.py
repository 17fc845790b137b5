import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "tiny_kev"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def native_lib():
    """The in-tree library, built if stale (nvcc cross-compiles without a GPU)."""
    from huncho_b200 import build, _native
    build.build()
    return _native.load()


@pytest.fixture(scope="session")
def tiny_dir():
    return GOLDEN


@pytest.fixture(scope="session")
def synth_root(tmp_path_factory):
    return Path(os.environ.get("HK_SYNTH_DIR") or tmp_path_factory.mktemp("synth"))
