"""Shared pytest configuration: the ``gpu`` marker and seeded model fixtures."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and the built library")
    from tests.host import limit_threads
    limit_threads()


@pytest.fixture(scope="session")
def ops_golden():
    return dict(np.load(GOLDEN / "ops.npz"))


@pytest.fixture(scope="session")
def tiny30_golden():
    return dict(np.load(GOLDEN / "model_tiny30.npz"))


@pytest.fixture(scope="session")
def smollm2_golden():
    return dict(np.load(GOLDEN / "model_smollm2.npz"))


@pytest.fixture(scope="session")
def tiny30_model():
    """The reference runtime tests' model: 30 x 576, vocab 128, seed 2701."""
    from oracle import hf_reference as hf
    return hf.build_model(hf.reference_runtime_config(), 2701)


@pytest.fixture(scope="session")
def smollm2_model():
    """Benchmark geometry: vocab 49152, tied embeddings, RoPE theta 1e5, seed 0."""
    from oracle import hf_reference as hf
    return hf.build_model(hf.smollm2_config(), 0)
