"""The reference's own driver program on the GPU, through libkvp.so.

oracle/_ref/policy_experiment_kvp is the reference's unmodified
src/run_policy_experiment.cu compiled against its own C++ headers and linked
against libkvp.so alone, so every KVTileManager, policy and attention call it
makes runs this library's code (the C++ boundary of include/cxx/).
oracle/_ref/policy_experiment_gpu is the reference's complete program,
kernel included, built for sm_100a; oracle/_ref/policy_experiment_ref is the
same driver built for the host with the reference's manager and policies.

On benchmark configs 1 (one 1560-token frame, MotionGated, 22 fp32 tiles) and
2 (8 frames, causal cross-frame, Recency, 22 tiles; arena and streaming):

* what the driver prints (slots, the frame-0 selection, the streamed
  staged bytes) equals the reference program's, line for line;
* the output is within the reference's gates of the fp32 golden
  (tests/test_correctness.py:26-27: max-abs < 1e-3, mean-abs < 1e-4;
  config 2 on two heads of every frame);
* the output is bitwise equal to the None policy's
  (tests/test_policy_variants.py:174-176);
* the output agrees with the reference kernel's on every row within 1e-4.
"""

from __future__ import annotations

import subprocess
from pathlib import Path

import numpy as np
import pytest

from kvp import traces
from oracle.attention import attention_frames

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
REFBIN = ROOT / "oracle" / "_ref"
DRV_KVP = REFBIN / "policy_experiment_kvp"
DRV_GPU = REFBIN / "policy_experiment_gpu"
DRV_HOST = REFBIN / "policy_experiment_ref"
GOLDEN = ROOT / "tests" / "golden"
T, H, D = 1560, 12, 1536
SET_ASIDE_22 = 22 * 16 * D * 4 * 2  # 22 fp32 tiles: 4,325,376 B


def _need(*exes):
    for e in exes:
        if not e.exists():
            pytest.skip(f"{e.name} not built (oracle/Makefile with the reference checkout)")


@pytest.fixture(scope="module")
def inputs(tmp_path_factory, cuda):
    d = traces.write_driver_inputs(tmp_path_factory.mktemp("drv"), 8, seed=0)
    q, k, v = (np.fromfile(d / f"{n}.bin", dtype=np.float32).reshape(8 * T, D) for n in "qkv")
    return d, q, k, v


def _run(exe, d, *, policy, mode, frames, streaming=False, csv, set_aside=SET_ASIDE_22, tag):
    out = d / "out" / f"{exe.name}_{tag}.bin"
    cmd = [str(exe), "--policy", policy, "--attn-mode", mode, "--q", str(d / "q.bin"),
           "--k", str(d / "k.bin"), "--v", str(d / "v.bin"), "--motion-csv", str(csv),
           "--out", str(out), "--frames", str(frames), "--tokens", str(T), "--hidden", str(D),
           "--heads", str(H), "--tile-tokens", "16", "--set-aside-bytes", str(set_aside)]
    if streaming:
        cmd.append("--streaming")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    o = np.fromfile(out, dtype=np.float32).reshape(frames * T, D)
    lines = [ln for ln in r.stdout.splitlines() if not ln.startswith("policy=") or "->" not in ln]
    return lines, o


def _stats(got, want):
    d = np.abs(got.astype(np.float64) - want.astype(np.float64))
    return float(d.max()), float(d.mean())


def test_config1_motion_gated(inputs):
    _need(DRV_KVP, DRV_GPU, DRV_HOST)
    d, q, k, v = inputs
    # the driver reads the first `frames` frames of the files
    csv = GOLDEN / "motion_config1.csv"
    lines, o = _run(DRV_KVP, d, policy="motion", mode="intra", frames=1, csv=csv, tag="c1")
    ref_lines, o_ref = _run(DRV_GPU, d, policy="motion", mode="intra", frames=1, csv=csv, tag="c1")
    host_lines = subprocess.run(
        [str(DRV_HOST), "--policy", "motion", "--attn-mode", "intra", "--q", str(d / "q.bin"),
         "--k", str(d / "k.bin"), "--v", str(d / "v.bin"), "--motion-csv", str(csv),
         "--out", str(d / "out" / "host_c1.bin"), "--frames", "1", "--tokens", str(T),
         "--hidden", str(D), "--heads", str(H), "--set-aside-bytes", str(SET_ASIDE_22)],
        capture_output=True, text=True, check=True, timeout=600).stdout.splitlines()
    assert lines == ref_lines
    assert lines == [ln for ln in host_lines if "->" not in ln]
    assert any("slots=22" in ln for ln in lines), lines
    _, o_none = _run(DRV_KVP, d, policy="none", mode="intra", frames=1, csv=csv, tag="c1none")
    assert np.array_equal(o, o_none)
    want = attention_frames(q[:T], k[:T], v[:T], frames=1, tokens=T, heads=H, head_dim=128,
                            mode="intra")
    mx, mean = _stats(o, want)
    assert mx < 1e-3 and mean < 1e-4, (mx, mean)
    mx_ref, _ = _stats(o, o_ref)
    assert mx_ref < 1e-4, mx_ref


@pytest.mark.parametrize("streaming", [False, True], ids=["arena", "streaming"])
def test_config2_cross_recency(inputs, streaming):
    _need(DRV_KVP, DRV_GPU)
    d, q, k, v = inputs
    csv = GOLDEN / "motion_config2.csv"
    tag = "c2s" if streaming else "c2a"
    lines, o = _run(DRV_KVP, d, policy="recency", mode="cross", frames=8, streaming=streaming,
                    csv=csv, tag=tag)
    ref_lines, o_ref = _run(DRV_GPU, d, policy="recency", mode="cross", frames=8,
                            streaming=streaming, csv=csv, tag=tag)
    assert lines == ref_lines
    if streaming:
        assert any(ln.startswith("streamed staged_bytes=") for ln in lines), lines
    _, o_none = _run(DRV_KVP, d, policy="none", mode="cross", frames=8, csv=csv, tag=tag + "none")
    assert np.array_equal(o, o_none)
    mx_ref, _ = _stats(o, o_ref)
    assert mx_ref < 1e-4, mx_ref
    heads = [0, 11]
    want = attention_frames(q, k, v, frames=8, tokens=T, heads=H, head_dim=128, mode="cross",
                            heads_subset=heads)
    cols = np.concatenate([np.arange(h * 128, (h + 1) * 128) for h in heads])
    mx, mean = _stats(o[:, cols], want[:, cols])
    assert mx < 1e-3 and mean < 1e-4, (mx, mean)
