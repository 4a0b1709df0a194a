import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    def load(name):
        path = GOLDEN / f"{name}.npz"
        if not path.exists():
            pytest.skip(f"golden fixture {name} not generated")
        return dict(np.load(path))
    return load
