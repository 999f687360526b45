import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_sessionstart(session):
    # compile the CPU checkers (the reference shim only where its sources exist)
    from oracle import oracle as O
    O.build(reference=None)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")
    config.addinivalue_line("markers", "reference: needs the OpenNeedle sources to build oracle/_ref")


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import oracle as O
    O.build(reference=None)
    return O
