"""The C++ drop-in boundary: the reference's C++ interface served by
libkvp.so (no GPU needed).

The reference's driver (src/run_policy_experiment.cu:10-12,98-276) and any
other C++ caller use the classes and functions of src/kv_tile_manager.h,
src/tile_gating_policy.h and src/attn_kernel.h.  include/cxx/ restates those
headers and libkvp.so defines everything they declare, so such a caller
links against libkvp.so alone:

* the object layout a caller compiles in equals the reference's
  (tests/golden/cxx_layout_ref.json, made from the reference's own headers);
* the policies, called through TileGatingPolicy pointers, give the C
  oracle's ids;
* the reference's unmodified driver, linked against libkvp.so
  (oracle/_ref/policy_experiment_kvp), needs no symbol that libkvp.so does
  not define; with the reference checkout at hand ($KVP_REF_ROOT) it is
  also re-linked here, against the reference's headers and against
  include/cxx/.
"""

from __future__ import annotations

import json
import os
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
CXX_INC = ROOT / "include" / "cxx"
NATIVE = ROOT / "cuda-kv-persistence_b200" / "kvp" / "_native"
LIBKVP = NATIVE / "libkvp.so"
DRIVER_KVP = ROOT / "oracle" / "_ref" / "policy_experiment_kvp"
GOLDEN = ROOT / "tests" / "golden"
CUDA_INC = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "include"
CUDA_LIB = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "lib64"
REF = os.environ.get("KVP_REF_ROOT")

POLICIES = ("none", "uniform", "recency", "motion", "reuse_weighted")


def _gxx(*args, cwd=None):
    r = subprocess.run(["g++", "-std=c++17", "-O1", *map(str, args)], capture_output=True, text=True,
                       cwd=cwd)
    assert r.returncode == 0, r.stdout + r.stderr
    return r


@pytest.fixture(scope="module")
def check_exe(tmp_path_factory):
    from kvp._lib import lib
    lib()  # builds nothing; fails loudly when libkvp.so is missing
    exe = tmp_path_factory.mktemp("cxx") / "cxx_boundary_check"
    _gxx("-I", CXX_INC, ROOT / "tests" / "cxx_boundary_check.cpp", "-L", NATIVE, "-lkvp",
         f"-Wl,-rpath,{NATIVE}", "-o", exe)
    return exe


def test_layout_matches_reference_headers(tmp_path):
    want = json.loads((GOLDEN / "cxx_layout_ref.json").read_text())
    want.pop("generator")
    exe = tmp_path / "probe"
    _gxx("-I", CXX_INC, GOLDEN / "cxx_layout_probe.cpp", "-o", exe)
    got = json.loads(subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout)
    assert got == want


def _dyn_symbols(path, defined):
    flag = "--defined-only" if defined else "--undefined-only"
    out = subprocess.run(["nm", "-D", flag, str(path)], capture_output=True, text=True,
                         check=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if ln.strip()}


CXX_SYMBOLS = [
    "_ZN13KVTileManagerC1Emm", "_ZN13KVTileManagerD1Ev", "_ZN13KVTileManager4initEv",
    "_ZN13KVTileManager5admitElPvm", "_ZN13KVTileManager7releaseEl", "_ZN13KVTileManager5clearEv",
    "_ZNK13KVTileManager15persisted_tilesEv", "_ZNK13KVTileManager12is_persistedEl",
    "_ZNK13KVTileManager18query_device_limitEv",
    "_ZN13KVTileManager10arena_initEmm", "_ZN13KVTileManager16arena_begin_stepEv",
    "_ZN13KVTileManager11arena_stageEPKvmS1_mPl", "_ZN13KVTileManager18arena_apply_windowEv",
    "_ZN13KVTileManager14arena_end_stepEv", "_ZN13KVTileManager15streaming_beginEv",
    "_ZN13KVTileManager15streaming_stageElPKvmS1_mbPlPb",
    "_ZN13KVTileManager17streaming_releaseEl", "_ZN13KVTileManager22streaming_apply_windowEv",
    "_ZN13KVTileManager13streaming_endEv",
    "_ZTV19NoPersistencePolicy", "_ZTV19UniformWindowPolicy", "_ZTV19RecencyWindowPolicy",
    "_ZTV19ReuseWeightedPolicy", "_ZTV17MotionGatedPolicy", "_ZN19ReuseWeightedPolicyC1Eii",
    "_Z25attn_forward_single_framePKfS0_S0_S0_PKlPfiiiii",
    "_Z21attn_forward_launcherPKfS0_S0_S0_PKlPfiiiib",
]


def test_library_defines_the_reference_cxx_interface():
    """Every member function of src/kv_tile_manager.h:21-90 that is not inline
    in the header, the five policies' vtables and constructors
    (src/tile_gating_policy.h:8-68) and the C++-linkage attention entry points
    (src/attn_kernel.h:15-29), next to the C-linkage pair."""
    exported = _dyn_symbols(LIBKVP, defined=True)
    missing = [s for s in CXX_SYMBOLS if s not in exported]
    assert not missing, missing
    assert {"attn_forward_single_frame", "attn_forward_launcher"} <= exported


def test_reference_driver_binary_resolves_against_libkvp():
    """oracle/_ref/policy_experiment_kvp is the reference's unmodified driver
    linked against libkvp.so and no other reference translation unit: every
    KVTileManager / policy / attention symbol it needs is one that libkvp.so
    defines, and it defines none of them itself."""
    if not DRIVER_KVP.exists():
        pytest.skip("oracle/_ref/policy_experiment_kvp not built (needs the reference checkout)")
    needed = subprocess.run(["readelf", "-d", str(DRIVER_KVP)], capture_output=True, text=True,
                            check=True).stdout
    assert "[libkvp.so]" in needed
    undef = _dyn_symbols(DRIVER_KVP, defined=False)
    ours = [s for s in undef if any(k in s for k in ("KVTileManager", "Policy", "attn_forward"))]
    assert len(ours) >= 15, ours
    exported = _dyn_symbols(LIBKVP, defined=True)
    assert not [s for s in ours if s not in exported]
    defined = subprocess.run(["nm", "--defined-only", str(DRIVER_KVP)], capture_output=True,
                             text=True, check=True).stdout
    assert "attn_forward_kernel" not in defined and "_ZN13KVTileManager" not in defined


@pytest.mark.skipif(not (REF and Path(REF, "src", "run_policy_experiment.cu").exists()),
                    reason="set KVP_REF_ROOT to the reference checkout to re-link its driver")
@pytest.mark.parametrize("headers", ["reference", "include_cxx"])
def test_relink_reference_driver(tmp_path, headers):
    """The unmodified src/run_policy_experiment.cu compiles and links against
    libkvp.so alone, with its own headers (its quoted includes resolve next to
    it) and with include/cxx/ (compiled through a symlink, so that the quoted
    includes fall through to -I)."""
    src = Path(REF) / "src" / "run_policy_experiment.cu"
    inc = []
    if headers == "include_cxx":
        link = tmp_path / "run_policy_experiment.cu"
        link.symlink_to(src)
        src, inc = link, ["-I", CXX_INC]
    exe = tmp_path / "driver"
    _gxx("-w", *inc, "-I", CUDA_INC, "-x", "c++", src, "-x", "none", "-L", NATIVE, "-lkvp",
         "-L", CUDA_LIB, "-lcudart", f"-Wl,-rpath,{NATIVE}", "-o", exe)
    undef = _dyn_symbols(exe, defined=False)
    assert "_ZN13KVTileManagerC1Emm" in undef


def test_policies_through_cxx_classes_match_oracle(check_exe, oracle):
    rng = np.random.default_rng(3)
    for _ in range(25):
        n = int(rng.integers(1, 600))
        mx = int(rng.integers(0, 120))
        tf = int(rng.integers(1, 40))
        s = (rng.random(n) if rng.random() < 0.5 else rng.integers(0, 4, n) / 3).astype(np.float32)
        text = " ".join(f"{x:.9g}" for x in s)
        out = subprocess.run([str(check_exe), "policies", str(n), str(mx), "98", str(tf)],
                             input=text, capture_output=True, text=True, check=True).stdout
        lines = out.strip().splitlines()
        assert [ln.split()[0] for ln in lines] == list(POLICIES)
        for pol, ln in zip(POLICIES, lines):
            parts = [int(x) for x in ln.split()[1:]]
            got = np.array(parts[1:1 + parts[0]], dtype=np.int64)
            want = oracle.select(pol, s, mx, 98, tf)
            assert np.array_equal(got, want), (pol, n, mx, tf)


def test_manager_accessors_without_a_device(check_exe):
    """A caller's inline accessors read the members the library keeps; an
    admission before init() is invalid, as in src/kv_tile_manager.cu:49-53."""
    out = subprocess.run([str(check_exe), "manager"], capture_output=True, text=True,
                         check=True).stdout
    kv = dict(ln.split(" ", 1) for ln in out.strip().splitlines())
    assert kv["persisted_bytes"] == "0" and kv["persisted_tiles"] == "0"
    assert kv["arena_ptr_null"] == "1" and kv["arena_used"] == "0"
    assert kv["staged_bytes"] == "0"
    assert kv["admit_too_large"] == "-1" and kv["admit_bad_args"] == "-1"
    assert kv["release_unknown"] == "0" and kv["is_persisted"] == "0"
    assert kv["ktile"] == "64 warps 8"
