import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def load_golden(name: str) -> dict:
    return json.loads((GOLDEN / name).read_text())


@pytest.fixture(scope="session")
def golden():
    return load_golden


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda", 0)


def reference_root() -> Path | None:
    """The reference checkout (renderityai/NamiTorch): $NAMITORCH_REFERENCE, else a
    checkout named ``reference`` beside this repository; None when neither holds the
    ``namitorch`` package."""
    env = os.environ.get("NAMITORCH_REFERENCE")
    root = Path(env) if env else REPO.parent / "reference"
    return root if (root / "namitorch").is_dir() else None


def reference_available() -> bool:
    return reference_root() is not None
