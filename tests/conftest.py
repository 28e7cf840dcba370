"""Shared pytest setup: marker registration, import paths and fixtures.

Tests marked `gpu` need a B200 and the built libphonon_cuda.so; the rest run
on CPU. The CPU oracle (oracle/) is only ever used here as the checker.
"""
import json
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "speech-mac_b200"))
sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libphonon_cuda.so")


@pytest.fixture(scope="session")
def pins():
    return json.loads((GOLDEN / "pins.json").read_text())


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import ORACLE_SO, Oracle, build
    if not ORACLE_SO.exists():
        build()
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import REF_SO, Reference
    if not REF_SO.exists():
        pytest.skip("oracle/_ref/libphonon_ref.so not built (needs the speech-mac tree once)")
    return Reference()


@pytest.fixture(scope="session")
def weights12():
    from phonon_b200 import synth
    return synth.flow_weights(12, seed=0)


@pytest.fixture(scope="session")
def cuda_ok():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return True
