import json
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden" / "packages"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def golden(name: str) -> Path:
    return GOLDEN / name


def golden_ir(name: str) -> Path:
    (path,) = sorted((GOLDEN / name).glob("*.ir.json"))
    return path


def golden_meta(name: str) -> dict:
    return json.loads((GOLDEN / name / "meta.json").read_text())


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a CUDA device is required for -m gpu tests")
    return torch.device("cuda:0")
