"""Shared fixtures.  GPU tests carry @pytest.mark.gpu; everything else runs on CPU."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
for p in (str(REPO),):
    if p not in sys.path:
        sys.path.insert(0, p)

# qgraph fixtures made by tests/golden/make_fixtures.py from the reference
QGRAPH_FIXTURES = ["fx_v1", "fx_v2", "c1_v1", "c1_v2", "qwen2_tiny", "qwen3_tiny", "d128_tiny"]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN
