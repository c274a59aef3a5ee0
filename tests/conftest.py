import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

os.environ.setdefault("OMP_NUM_THREADS", str(min(16, os.cpu_count() or 1)))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "dist: multi-process torch.distributed test on CPU (gloo)")


@pytest.fixture(scope="session")
def pkg():
    """The sampler package (its directory name is not an identifier, so it is registered under an alias)."""
    import __graft_entry__

    return __graft_entry__.load_package()
