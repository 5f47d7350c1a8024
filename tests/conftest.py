"""Shared fixtures.  GPU tests are marked `gpu` (they need a B200 and the built CUDA library);
everything else runs on the CPU in a few minutes."""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "carbon-ocr_b200"))

from carbon_rec import model, netdef  # noqa: E402
from oracle import oracle as O  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the CUDA library")


@pytest.fixture(scope="session")
def golden():
    return json.loads((ROOT / "tests" / "golden" / "golden.json").read_text())


@pytest.fixture(scope="session")
def orc():
    O.build()
    return O.Oracle()


@pytest.fixture(scope="session")
def ref():
    if not O.Reference.available():
        pytest.skip("the reference's compiled code (oracle/_ref) is not here")
    return O.Reference()


@pytest.fixture(scope="session")
def rec_latin():
    """(int8 RecNet, fp32 RecNet, int8 ONNX model, fp32 ONNX model) of rec-latin, seed 0."""
    _, _, fp, i8 = model.make_rec_latin(0)
    return netdef.compile_model(i8), netdef.compile_model(fp), i8, fp


@pytest.fixture(scope="session")
def mini():
    _, _, fp, i8 = model.make_mini(4)
    return netdef.compile_model(i8), netdef.compile_model(fp), i8, fp


def pytest_collection_modifyitems(config, items):
    # the GPU tests need the library; build it once here if it is missing (nvcc, no GPU needed)
    if any("gpu" in it.keywords for it in items):
        from carbon_rec import build
        build.build()
