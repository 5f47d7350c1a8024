"""The library's host-side parts that run without a GPU (tests/native/host_parts.cpp): the
fork-join pool a run's layout uses and the stager's streaming copy into pinned chunks, compiled
from the library's own headers with the host compiler and run here."""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CUDA_INCLUDE = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "include"


@pytest.mark.skipif(shutil.which("g++") is None or not (CUDA_INCLUDE / "cuda_runtime.h").exists(),
                    reason="needs g++ and the CUDA headers")
def test_pool_and_streaming_copy(tmp_path):
    exe = tmp_path / "host_parts"
    subprocess.run(["g++", "-std=c++17", "-O2", "-pthread", f"-I{ROOT / 'carbon-ocr_b200' / 'csrc'}", f"-I{CUDA_INCLUDE}",
                    str(ROOT / "tests" / "native" / "host_parts.cpp"), "-o", str(exe)], check=True, capture_output=True,
                   text=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stdout + r.stderr
