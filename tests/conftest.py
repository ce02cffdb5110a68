"""Shared pytest setup: repo root on sys.path, the ``gpu`` marker, fixtures."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (run on a B200 with -m gpu)")


@pytest.fixture(scope="session")
def built_lib():
    """The in-tree C-ABI library (built here if missing or stale; nvcc cross-compiles)."""
    from mtp_b200 import build as b
    if b.LIB.exists():
        try:
            return b.build(quiet=True)
        except Exception:
            return b.LIB
    return b.build(quiet=True)


@pytest.fixture(scope="session")
def cuda_device(built_lib):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    import mtp_b200
    mtp_b200.load_library()
    return torch.device("cuda:0")


_PARITY = []


def record_parity(**fields):
    """Parity figures of one check, with the test that made it; written to the
    JSON file named by MTP_PARITY_LOG (if set) when the session ends."""
    import os
    fields["test"] = os.environ.get("PYTEST_CURRENT_TEST", "").split(" ")[0]
    _PARITY.append(fields)


def pytest_sessionfinish(session, exitstatus):
    import json
    import os
    path = os.environ.get("MTP_PARITY_LOG")
    if path and _PARITY:
        with open(path, "w") as f:
            json.dump(_PARITY, f, indent=1)


def golden(name: str):
    import torch
    return torch.load(GOLDEN / name, weights_only=False)
