"""Shared test setup: the `gpu` marker, package loading, seeded workloads."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (str(ROOT), str(ROOT / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

from __graft_entry__ import load_package  # noqa: E402

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def gsv():
    return load_package()


@pytest.fixture(scope="session")
def kat():
    return dict(np.load(GOLDEN / "kat_ref.npz"))


@pytest.fixture(scope="session")
def tiny():
    return dict(np.load(GOLDEN / "decoder_tiny.npz"))


@pytest.fixture(scope="session")
def encp_golden():
    return dict(np.load(GOLDEN / "encp_tiny.npz"))


# enc_p layers of the golden fixtures (one per stack).
ENCP_GOLDEN_LAYERS = {"encoder_ssl": 1, "encoder_text": 1, "encoder2": 1}


@pytest.fixture(scope="session")
def flow_golden():
    return dict(np.load(GOLDEN / "flow_tiny.npz"))


def rel_max(a, b):
    """max |a - b| / max |b|."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def snr_db(a, ref):
    a = np.asarray(a, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(10 * np.log10((ref ** 2).sum() / max(((a - ref) ** 2).sum(), 1e-300)))
