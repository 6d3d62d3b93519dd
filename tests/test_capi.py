"""libkvp.so loads and exports every symbol include/*.h declares (no compute)."""

from __future__ import annotations

import re
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"^\s*[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", text, flags=re.M):
            name = m.group(1)
            if name not in ("if", "for", "while", "return", "sizeof", "defined"):
                names.add(name)
    return names


def test_library_loads_and_exports_declared_symbols():
    from kvp._lib import LIB_PATH, SIGNATURES, lib
    L = lib()
    declared = declared_functions()
    assert len(declared) >= 50, declared
    for name in declared:
        assert hasattr(L, name), f"{name} declared in include/ but not exported"
        assert name in SIGNATURES, f"{name} has no ctypes signature"
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert declared <= exported
    assert L.kvp_version().decode().startswith("kvp-b200")


def test_reference_facade_signatures_unchanged():
    """The kvtm_* facade keeps the reference's exact parameter lists
    (src/kv_tile_manager.cu:223-339)."""
    text = (ROOT / "include" / "kv_tile_manager.h").read_text()
    for sig in [
        "void* kvtm_create(long budget_bytes, long max_window_bytes);",
        "int kvtm_admit(void* m, long tile_id, void* ptr, long bytes);",
        "int kvtm_arena_init(void* m, long cap_bytes, long row_stride_floats);",
        "int kvtm_streaming_stage(void* m, long row_id, const void* k_dev, long k_bytes,",
        "long kvtm_layout_tiles_per_frame(int tokens_per_frame, int tile_tokens);",
    ]:
        assert sig in text, sig


def test_no_cpu_fallback_when_library_missing(tmp_path, monkeypatch):
    """The product fails loudly without its native library."""
    import importlib
    import kvp._lib as lb
    monkeypatch.setattr(lb, "LIB_PATH", tmp_path / "missing.so")
    monkeypatch.setattr(lb, "_LIB", None)
    try:
        lb.lib()
    except lb.KvpError as e:
        assert "no fallback" in str(e)
    else:
        raise AssertionError("loaded a library that does not exist")
    importlib.reload(lb)
