"""benchmark configs 2, 3 and 5 at their own shapes on the GPU.

The reference gates its full configurations on bitwise equality of every
policy's output with the None policy's (tests/test_policy_variants.py:174-179)
and on the fp32 golden (tests/test_correctness.py:26-27).  Here every
config runs the reference driver's per-frame loop (kvp.frames.run_frames:
admission, staging, KVMap upload, window, one tcgen05 launch per frame) at
1560 tokens per frame and all 12 heads, in arena and streaming mode:

* config 2: 8 frames, causal cross-frame, Recency with 22 bf16 tiles
  (2,162,688 B), the AR(1) trace tests/golden/motion_config2.csv;
* config 3: 6 frames of the 50-frame blob trace under the 5-frame window
  (4 previous frames + the current one; frames 4 and 5 see a full window),
  ReuseWeighted with the device's whole persisting-L2 budget, one layer;
* config 5: the static and the high-motion cell at 100 % of the budget, all
  16 frames, every policy.

Each output is bitwise equal to None's and within the bf16 gates of the fp32
oracle (max-abs < 2e-2, rel-L2 < 1e-2) on every row of two heads.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from kvp.traces import qkv, read_motion_csv
from oracle.attention import attention_frames
from test_gpu_kernels import check_bf16

pytestmark = pytest.mark.gpu

T, H = 1560, 12
D = H * 128
TILES = 98
CHECK_HEADS = [0, 11]
GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"


def _max_persist():
    from kvp._lib import DeviceInfo, lib
    info = DeviceInfo()
    assert lib().kvp_query_device(-1, C.byref(info)) == 0
    return int(info.max_persisting_l2_bytes)


def _run_policies(q, k, v, scores, policies, *, set_aside, frames, streaming, window=0):
    from kvp.attention import read_status
    from kvp.frames import run_frames
    stream = int(torch.cuda.current_stream().cuda_stream)
    read_status()
    outs = {}
    for policy in policies:
        out = torch.full_like(q, float("nan"))
        run_frames(q, k, v, out, scores, policy=policy, set_aside=set_aside, frames=frames,
                   tokens=T, heads=H, stream=stream, streaming=streaming, window=window)
        outs[policy] = out.float().cpu().numpy()
    assert read_status() == 0
    return outs


def _oracle_heads(q, k, v, frames, window=0):
    return attention_frames(q.float().cpu().numpy(), k.float().cpu().numpy(),
                            v.float().cpu().numpy(), frames=frames, tokens=T, heads=H,
                            head_dim=128, mode="cross", window=window, heads_subset=CHECK_HEADS)


def _check(outs, want, what):
    cols = np.concatenate([np.arange(h * 128, (h + 1) * 128) for h in CHECK_HEADS])
    for p, o in outs.items():
        assert np.array_equal(o, outs["none"]), (what, p)
    check_bf16(outs["none"][:, cols], want[:, cols], what)


@pytest.fixture(scope="module")
def inputs16(cuda):
    q, k, v = (t.cuda() for t in qkv(16 * T, D, seed=0))
    return q, k, v


@pytest.mark.parametrize("streaming", [False, True], ids=["arena", "streaming"])
def test_config2_recency_22_tiles(inputs16, streaming):
    q, k, v = (t[:8 * T] for t in inputs16)
    scores = read_motion_csv(GOLDEN / "motion_config2.csv", 8, TILES)
    outs = _run_policies(q, k, v, scores, ("none", "recency"), set_aside=2162688, frames=8,
                         streaming=streaming)
    _check(outs, _oracle_heads(q, k, v, 8), ("config 2", streaming))


@pytest.mark.parametrize("streaming", [False, True], ids=["arena", "streaming"])
def test_config3_window_of_five(inputs16, streaming):
    F, W = 6, 5
    q, k, v = (t[:F * T] for t in inputs16)
    scores = read_motion_csv(GOLDEN / "motion_config3.csv", 50, TILES)[:F]
    outs = _run_policies(q, k, v, scores, ("none", "reuse_weighted"),
                         set_aside=_max_persist(), frames=F, streaming=streaming, window=W)
    _check(outs, _oracle_heads(q, k, v, F, window=W), ("config 3", streaming))


@pytest.fixture(scope="module")
def oracle16(inputs16):
    return _oracle_heads(*inputs16, 16)


@pytest.mark.parametrize("regime", ["static", "high"])
@pytest.mark.parametrize("streaming", [False, True], ids=["arena", "streaming"])
def test_config5_full_budget(inputs16, oracle16, regime, streaming):
    q, k, v = inputs16
    scores = read_motion_csv(GOLDEN / f"motion_config5_{regime}.csv", 16, TILES)
    outs = _run_policies(q, k, v, scores,
                         ("none", "uniform", "recency", "motion", "reuse_weighted"),
                         set_aside=_max_persist(), frames=16, streaming=streaming)
    _check(outs, oracle16, ("config 5", regime, streaming))


@pytest.mark.parametrize("config", ["2", "5-high"])
def test_batched_frames_match_the_per_frame_loop(inputs16, oracle16, monkeypatch, config):
    """Arena mode with every frame planned first, staged into an arena of its
    own and run in one grid (kvp.frames.run_frames_batched, step by step and
    as one kvp_session_run_frames_batched call): each policy's output is
    bitwise the per-frame loop's (key split off, which the batched grid never
    uses), bitwise None's, and within the bf16 gates."""
    from kvp.attention import read_status
    from kvp.frames import run_frames, run_frames_batched
    monkeypatch.setenv("KVP_ATTN_SPLITS", "1")
    if config == "2":
        F, policies, budget = 8, ("none", "recency"), 2162688
        scores = read_motion_csv(GOLDEN / "motion_config2.csv", 8, TILES)
    else:
        F, policies, budget = 16, ("none", "uniform", "recency", "motion", "reuse_weighted"), _max_persist()
        scores = read_motion_csv(GOLDEN / "motion_config5_high.csv", 16, TILES)
    q, k, v = (t[:F * T] for t in inputs16)
    stream = int(torch.cuda.current_stream().cuda_stream)
    read_status()
    outs = {}
    for policy in policies:
        a = torch.full_like(q, float("nan"))
        b = torch.full_like(q, float("nan"))
        c = torch.full_like(q, float("nan"))
        run_frames_batched(q, k, v, a, scores, policy=policy, set_aside=budget, frames=F, tokens=T,
                           heads=H, stream=stream)
        run_frames(q, k, v, b, scores, policy=policy, set_aside=budget, frames=F, tokens=T,
                   heads=H, stream=stream)
        run_frames_batched(q, k, v, c, scores, policy=policy, set_aside=budget, frames=F, tokens=T,
                           heads=H, stream=stream, native=True)
        assert torch.equal(a, b), policy
        assert torch.equal(c, b), policy
        outs[policy] = a.float().cpu().numpy()
    assert read_status() == 0
    want = oracle16 if F == 16 else _oracle_heads(q, k, v, F)
    _check(outs, want[:F * T], ("batched", config))


@pytest.mark.parametrize("streaming", [False, True], ids=["arena", "streaming"])
def test_native_loop_matches_the_python_loop(inputs16, streaming):
    """kvp_session_run_frames (the whole per-frame loop in one native call)
    gives the bytes of the step-by-step loop, config 5 high at 10 %."""
    from kvp.attention import read_status
    from kvp.frames import run_frames
    scores = read_motion_csv(GOLDEN / "motion_config5_high.csv", 16, TILES)
    q, k, v = inputs16
    stream = int(torch.cuda.current_stream().cuda_stream)
    read_status()
    for policy in ("none", "reuse_weighted", "recency"):
        a = torch.full_like(q, float("nan"))
        b = torch.full_like(q, float("nan"))
        kw = dict(policy=policy, set_aside=_max_persist() // 10, frames=16, tokens=T, heads=H,
                  stream=stream, streaming=streaming)
        run_frames(q, k, v, a, scores, native=True, **kw)
        run_frames(q, k, v, b, scores, **kw)
        assert torch.equal(a, b), policy
    assert read_status() == 0


@pytest.mark.parametrize("mode,window", [("cross", 5), ("intra", 0)], ids=["cross-window5", "intra"])
def test_native_batched_loop_window_and_intra(inputs16, monkeypatch, mode, window):
    """kvp_session_run_frames_batched with a 5-frame causal window (config 3's
    shape, 6 frames, ReuseWeighted at the full budget) and in intra mode
    (8 frames, Recency, 22 tiles): bitwise the per-frame loop (key split off,
    which the batched grid never uses), and None's."""
    from kvp.attention import read_status
    from kvp.frames import run_frames, run_frames_batched
    monkeypatch.setenv("KVP_ATTN_SPLITS", "1")
    if mode == "cross":
        F, budget, policies = 6, _max_persist(), ("none", "reuse_weighted")
        scores = read_motion_csv(GOLDEN / "motion_config3.csv", 50, TILES)[:F]
    else:
        F, budget, policies = 8, 2162688, ("none", "recency")
        scores = read_motion_csv(GOLDEN / "motion_config2.csv", 8, TILES)
    q, k, v = (t[:F * T] for t in inputs16)
    stream = int(torch.cuda.current_stream().cuda_stream)
    read_status()
    outs = {}
    for policy in policies:
        a = torch.full_like(q, float("nan"))
        b = torch.full_like(q, float("nan"))
        kw = dict(policy=policy, set_aside=budget, frames=F, tokens=T, heads=H, stream=stream,
                  mode=mode, window=window)
        run_frames_batched(q, k, v, a, scores, native=True, **kw)
        run_frames(q, k, v, b, scores, **kw)
        assert torch.equal(a, b), policy
        outs[policy] = a
    assert torch.equal(outs[policies[0]], outs[policies[1]])
    assert read_status() == 0
