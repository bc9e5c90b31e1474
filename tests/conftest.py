"""Shared pytest setup: the ``gpu`` marker and helpers for the attention parity tests."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built libwfattn")


@pytest.fixture(scope="session")
def kats() -> dict:
    """The reference's three attention test cases (inputs + NumPy-oracle outputs)."""
    return json.loads((GOLDEN / "attention_kats.json").read_text())["cases"]


@pytest.fixture(scope="session")
def gpt2_head_golden() -> dict:
    with np.load(GOLDEN / "gpt2_head_call.npz") as z:
        return {k: z[k] for k in z.files}


def approx_list(values, rel):
    return [pytest.approx(v, rel=rel) for v in values]
