import pathlib
import sys

import pytest

REPO = pathlib.Path(__file__).resolve().parents[1]
for sub in ("oracle", "lightbridge-engine_b200"):
    p = str(REPO / sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden_dir() -> pathlib.Path:
    return REPO / "tests" / "golden"


def read_golden(name: str) -> bytes:
    return (REPO / "tests" / "golden" / name).read_bytes()
