"""The streaming manager's flat row -> slot table (csrc/slot_map.h) against
std::unordered_map over two million random operations (CPU only)."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent
CSRC = HERE.parent / "cuda-kv-persistence_b200" / "csrc"


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_slot_map_matches_unordered_map(tmp_path):
    exe = tmp_path / "slot_map_fuzz"
    subprocess.run(["g++", "-O2", "-std=c++17", "-I", str(CSRC), str(HERE / "slot_map_fuzz.cpp"),
                    "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    assert "slotmap fuzz ok" in out
