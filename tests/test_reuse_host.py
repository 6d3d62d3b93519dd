"""Temporal-reuse streaming (slots keyed by token position, a tile re-copied
only when the trace's reuse column says it changed) on the host, CPU only.

The reference reads the reuse column (src/run_policy_experiment.cu:114-118)
and stages with changed = false (:211); kvmap_reuse_ref.json holds the same
loop with real flags run on the reference's own KVTileManager
(src/kv_tile_manager.cu:153-200, through oracle/ref_stub/ref_shims.cpp).
Bit-exact: the oracle against those fixtures, the product's Session against
the oracle (maps, copy lists, re-copies, sticky hits, staged bytes, window).
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from kvp.session import Session
from kvp.traces import motion_config2, read_motion_csv, reuse_flags

GOLDEN = Path(__file__).resolve().parent / "golden"
T = 1560
CSV = {"config2_reuse": "motion_config2_reuse.csv", "config5_high": "motion_config5_high.csv",
       "config3": "motion_config3.csv"}


def digest(a):
    return hashlib.sha256(np.ascontiguousarray(a, dtype="<i8").tobytes()).hexdigest()[:16]


def _cases():
    return json.loads((GOLDEN / "kvmap_reuse_ref.json").read_text())["cases"]


def _inputs(oracle, case):
    scores, col = oracle.read_motion_csv(GOLDEN / CSV[case["trace"]], case["frames"], 98,
                                         with_reuse=True)
    reuse = {"csv": col, "derived": reuse_flags(scores), "none": None}[case["flags"]]
    return scores, reuse


def _session_run(scores, reuse, *, policy, frames, set_aside, elem=4, tokens=T, hidden=1536):
    s = Session(mode="reuse", policy=policy, frames=frames, tokens=tokens, hidden=hidden,
                elem_bytes=elem, set_aside=set_aside, streaming=True)
    out = {k: [] for k in ("copies", "restaged", "hits", "staged_bytes", "window_bytes", "maps",
                           "pairs")}
    for f in range(frames):
        st = s.plan_frame(f, scores, reuse)
        assert (st.map_row0, st.map_rows) == (f * tokens, tokens)
        out["copies"].append(st.copies)
        out["restaged"].append(st.restaged)
        out["hits"].append(st.hits)
        out["staged_bytes"].append(st.staged_bytes)
        out["window_bytes"].append(st.window_bytes)
        out["maps"].append(s.host_map(f * tokens, tokens))
        out["pairs"].append(s.copies())
    s.finish()
    s.close()
    return out


@pytest.mark.parametrize("case", _cases(),
                         ids=lambda c: "{trace}-{policy}-{set_aside}-{flags}".format(**c))
def test_oracle_reuse_matches_reference(oracle, case):
    scores, reuse = _inputs(oracle, case)
    got = oracle.run_reuse(scores, reuse, policy=case["policy"], frames=case["frames"],
                           set_aside=case["set_aside"])
    for f, want in enumerate(case["per_frame"]):
        have = {"sha": digest(got["maps"][f]), "mapped": int((got["maps"][f] >= 0).sum()),
                "copies": int(got["copies"][f]), "restaged": int(got["restaged"][f]),
                "hits": int(got["hits"][f]), "staged_bytes": int(got["staged_bytes"][f]),
                "window_bytes": int(got["window_bytes"][f])}
        assert have == want, f"frame {f}"


def _assert_session_equals_oracle(ref, ses, frames):
    off = 0
    for f in range(frames):
        assert np.array_equal(ses["maps"][f], ref["maps"][f]), f
        n = int(ref["copies"][f])
        assert ses["copies"][f] == n
        assert np.array_equal(ses["pairs"][f][:, 0], ref["copy_rows"][off:off + n]), f
        assert np.array_equal(ses["pairs"][f][:, 1], ref["copy_slots"][off:off + n]), f
        off += n
        assert ses["restaged"][f] == int(ref["restaged"][f])
        assert ses["hits"][f] == int(ref["hits"][f])
        assert ses["staged_bytes"][f] == int(ref["staged_bytes"][f])
        assert ses["window_bytes"][f] == max(int(ref["window_bytes"][f]), 0)


@pytest.mark.parametrize("case", [c for c in _cases() if c["trace"] != "config3"],
                         ids=lambda c: "{trace}-{policy}-{set_aside}-{flags}".format(**c))
@pytest.mark.parametrize("elem", [4, 2])
def test_session_reuse_matches_oracle(oracle, case, elem):
    scores, reuse = _inputs(oracle, case)
    # bf16 rows are half as wide: half the budget admits the same rows
    sa = case["set_aside"] * elem // 4
    ref = oracle.run_reuse(scores, reuse, policy=case["policy"], frames=case["frames"],
                           set_aside=sa, elem_bytes=elem)
    ses = _session_run(scores, reuse, policy=case["policy"], frames=case["frames"],
                       set_aside=sa, elem=elem)
    _assert_session_equals_oracle(ref, ses, case["frames"])


def test_reuse_column_round_trip(oracle, tmp_path):
    sc = motion_config2()
    want = reuse_flags(sc)
    s1, r1 = read_motion_csv(GOLDEN / "motion_config2_reuse.csv", 8, 98, with_reuse=True)
    s2, r2 = oracle.read_motion_csv(GOLDEN / "motion_config2_reuse.csv", 8, 98, with_reuse=True)
    assert np.array_equal(r1, want) and np.array_equal(r2, want)
    assert np.array_equal(s1, s2)
    assert r1[0].sum() == 0                       # frame 0 is always written fresh
    frac = r1[1:].mean()
    assert 0.45 <= frac <= 0.55                   # the percentile-50 split
    # a trace without the column reads as "nothing reusable"
    _, r3 = read_motion_csv(GOLDEN / "motion_config2.csv", 8, 98, with_reuse=True)
    assert r3.sum() == 0


def test_reuse_edge_cases(oracle):
    rng = np.random.default_rng(5)
    frames, tokens, hidden = 6, 100, 64          # 7 tiles, the last one 4 rows
    nt = 7
    scores = rng.random((frames, nt)).astype(np.float32)
    tile_bytes = 16 * hidden * 4 * 2
    for reuse in (None, np.ones((frames, nt), np.int8), rng.integers(0, 2, (frames, nt)).astype(np.int8)):
        for policy in ("none", "uniform", "recency", "motion", "reuse_weighted"):
            for sa in (0, tile_bytes - 1, 3 * tile_bytes, 7 * tile_bytes, 20 * tile_bytes):
                ref = oracle.run_reuse(scores, reuse, policy=policy, frames=frames, tokens=tokens,
                                       hidden=hidden, set_aside=sa)
                ses = _session_run(scores, reuse, policy=policy, frames=frames, tokens=tokens,
                                   hidden=hidden, set_aside=sa)
                _assert_session_equals_oracle(ref, ses, frames)
    # every tile kept and nothing changed: after frame 0 nothing is copied
    ones = np.ones((frames, nt), np.int8)
    ref = oracle.run_reuse(scores, ones, policy="uniform", frames=frames, tokens=tokens,
                           hidden=hidden, set_aside=7 * tile_bytes)
    assert int(ref["copies"][0]) == tokens and ref["copies"][1:].sum() == 0
    assert (ref["hits"][1:] == tokens).all()
    # every tile changed: every kept row is re-copied into the slot it holds
    ref = oracle.run_reuse(scores, None, policy="uniform", frames=frames, tokens=tokens,
                           hidden=hidden, set_aside=7 * tile_bytes)
    assert (ref["copies"] == tokens).all() and (ref["restaged"][1:] == tokens).all()
    assert int(ref["staged_bytes"][-1]) == frames * tokens * hidden * 4 * 2


def test_reuse_mode_needs_streaming():
    # KvpError (a RuntimeError; other tests reload the module that defines it)
    with pytest.raises(RuntimeError, match="invalid configuration"):
        Session(mode="reuse", policy="recency", frames=4, streaming=False)
    s = Session(mode="reuse", policy="recency", frames=2, streaming=True)
    with pytest.raises(RuntimeError, match="not in stack mode"):
        s.plan_stack(np.zeros((2, 98), np.float32))
    with pytest.raises(RuntimeError, match="out of order"):
        s.plan_frame(1, np.zeros((2, 98), np.float32))


def _mixed_groups(m):
    g = m[:len(m) // 8 * 8].reshape(-1, 8)
    base = (g < 0).all(1)
    run = (g >= 0).all(1) & (np.diff(g, axis=1) == 1).all(1)
    return int((~base & ~run).sum())


@pytest.mark.parametrize("trace", ["ar1", "iid"])
def test_reuse_maps_keep_ascending_groups(oracle, trace):
    """Every 8-row group of a reuse-mode KVMap is all base rows or one
    ascending slot run (what the kernel stages with a TMA box), for every
    policy and budget: released tiles go back on the free stack last row
    first, so the next admitted tile gets ascending slots."""
    from kvp.traces import motion_config5
    sc = motion_config2(frames=16, seed=3) if trace == "ar1" else motion_config5("high", frames=16, seed=3)
    reuse = reuse_flags(sc)
    for policy in ("uniform", "recency", "motion", "reuse_weighted"):
        for frac in (0.05, 0.1, 0.25, 0.5, 1.0):
            r = oracle.run_reuse(sc, reuse, policy=policy, frames=16, hidden=1536, elem_bytes=2,
                                 set_aside=int(frac * 82_903_040))
            assert sum(_mixed_groups(r["maps"][f]) for f in range(16)) == 0, (policy, frac)
