"""Host logic of the product (libkvp.so, no GPU needed) against the oracle.

Bit-exact: policy selections (tgp_select), per-frame KVMaps, staging copy
lists, staged bytes and window spans of the session planner, and the
manager's admission accounting (kvtm_* in dry-run mode).
"""

from __future__ import annotations

import itertools
from pathlib import Path

import numpy as np
import pytest

from kvp import select
from kvp.manager import KVTileManager
from kvp.session import Session

GOLDEN = Path(__file__).resolve().parent / "golden"
T = 1560


def test_policy_select_matches_oracle(oracle):
    rng = np.random.default_rng(11)
    for _ in range(400):
        n = int(rng.integers(0, 700))
        mx = int(rng.integers(0, 300))
        tf = int(rng.integers(1, 60))
        s = (rng.random(n) if rng.random() < 0.5 else rng.integers(0, 4, n) / 3).astype(np.float32)
        for pol in ("none", "uniform", "recency", "motion", "reuse_weighted"):
            assert np.array_equal(select(pol, s, mx, 98, tf), oracle.select(pol, s, mx, 98, tf)), pol


def _compare(oracle, scores, *, policy, mode, streaming, frames, set_aside, elem, window=0,
             tokens=T, hidden=1536):
    ref = oracle.run_trace(scores, policy=policy, cross=mode == "cross", streaming=streaming,
                           frames=frames, tokens=tokens, hidden=hidden, elem_bytes=elem,
                           window=window, set_aside=set_aside)
    s = Session(mode=mode, policy=policy, frames=frames, tokens=tokens, hidden=hidden,
                elem_bytes=elem, set_aside=set_aside, streaming=streaming, window=window)
    off = 0
    for f in range(frames):
        st = s.plan_frame(f, scores)
        r0, want = ref.uploaded_slice(f, tokens, mode == "cross", window)
        assert (st.map_row0, st.map_rows) == (r0, len(want))
        assert np.array_equal(s.host_map(r0, len(want)), want), f
        n = int(ref.copy_count[f])
        cp = s.copies()
        assert len(cp) == n
        assert np.array_equal(cp[:, 0], ref.copy_rows[off:off + n])
        assert np.array_equal(cp[:, 1], ref.copy_slots[off:off + n])
        off += n
        assert st.staged_bytes == int(ref.staged_bytes[f])
        assert st.window_bytes == max(int(ref.window_bytes[f]), 0)
        if policy != "none":
            assert st.sel_count == int(ref.sel_count[f])
    s.finish()


@pytest.mark.parametrize("policy,mode,streaming,set_aside", [
    (p, m, st, sa) for p, m, st, sa in itertools.product(
        ["none", "uniform", "recency", "motion", "reuse_weighted"], ["intra", "cross"], [0, 1],
        [2162688, 4325376, 700000])])
def test_session_matches_oracle_ref8f(oracle, policy, mode, streaming, set_aside):
    scores = oracle.read_motion_csv(GOLDEN / "motion_ref8f.csv", 8, 98)
    _compare(oracle, scores, policy=policy, mode=mode, streaming=streaming, frames=8,
             set_aside=set_aside, elem=4)


@pytest.mark.parametrize("trace,frames,policy,window,streaming", [
    ("motion_config3.csv", 50, "reuse_weighted", 5, 1),
    ("motion_config3.csv", 50, "reuse_weighted", 5, 0),
    ("motion_config2.csv", 8, "recency", 0, 0),
    ("motion_config5_high.csv", 16, "motion", 3, 1),
    ("motion_config5_static.csv", 16, "uniform", 0, 0),
])
def test_session_matches_oracle_bf16_configs(oracle, trace, frames, policy, window, streaming):
    scores = oracle.read_motion_csv(GOLDEN / trace, frames, 98)
    _compare(oracle, scores, policy=policy, mode="cross", streaming=streaming, frames=frames,
             set_aside=82_903_040 // 4, elem=2, window=window)


def test_session_ragged_and_small_shapes(oracle):
    """Odd tails (tile_tokens not dividing T), tiny frames and hidden sizes."""
    rng = np.random.default_rng(3)
    for tokens, hidden, frames in [(40, 128, 3), (130, 256, 4), (1, 128, 2), (17, 128, 5)]:
        nt = (tokens + 15) // 16
        scores = rng.random((frames, nt)).astype(np.float32)
        for policy, mode, st in itertools.product(["recency", "motion", "reuse_weighted"],
                                                  ["intra", "cross"], [0, 1]):
            _compare(oracle, scores, policy=policy, mode=mode, streaming=st, frames=frames,
                     set_aside=3 * 16 * hidden * 2 * 2 + 7, elem=2, tokens=tokens, hidden=hidden)


def test_stack_plan_equals_last_cross_frame(oracle):
    """Stack mode = the dense cross admission of the last frame."""
    scores = oracle.read_motion_csv(GOLDEN / "motion_config4.csv", 21, 98)
    ref = oracle.run_trace(scores, policy="reuse_weighted", cross=True, streaming=False,
                           frames=21, elem_bytes=2, set_aside=82_903_040)
    s = Session(mode="stack", policy="reuse_weighted", frames=21, elem_bytes=2,
                set_aside=82_903_040)
    st = s.plan_stack(scores)
    assert np.array_equal(s.host_map(), ref.maps[20])
    assert st.copies == int(ref.copy_count[20])


def test_manager_capacity_scenario_dry_run(oracle):
    """The reference's capacity/admission contract S2-S8
    (tests/test_capacity_admission.py:97-148) on the dry-run manager."""
    budget, tile, win = 2162688, 98304, 134213632
    m = KVTileManager(budget, win, dry_run=True)
    o = oracle.manager(budget, win)
    assert m.init() and o.init() == 1
    assert m.query_device_limit() == budget == o.query_limit()
    base = 0x10000000
    admit = lambda t: (m.admit(t, base + t * tile, tile), o.admit(t, base + t * tile, tile))
    assert all(a == b == 1 for a, b in (admit(i) for i in range(22)))
    assert m.persisted_bytes() == budget and m.persisted_tiles() == 22
    assert admit(22) == (0, 0)                      # S3 refused
    assert admit(5) == (-1, -1)                     # S4 duplicate
    assert m.release(7) and not m.release(7)        # S5
    assert o.release(7) == 1 and o.release(7) == 0
    assert m.persisted_bytes() == budget - tile == o.persisted_bytes()
    assert admit(22) == (1, 1) and admit(23) == (0, 0)   # S6
    m.clear()
    assert m.persisted_tiles() == 0 and m.persisted_bytes() == 0   # S7
    assert m.admit(90, base, tile) == 1
    assert m.admit(-1, base, tile) == -1 and m.admit(1, 0, tile) == -1 and m.admit(2, base, 0) == -1
    assert m.admit(3, base, win + 1) == -1
    from kvp import TileLayout
    lay = TileLayout(1560, 16)                      # S8
    assert lay.tiles_per_frame == 98 and lay.tile_count(97) == 8 and lay.tile_start(97) == 1552
    assert sum(lay.tile_count(i) for i in range(98)) == 1560


def test_manager_random_sequences_match_oracle(oracle):
    """Arena and streaming accounting under random stage/release/window
    sequences, manager (dry run) vs oracle manager."""
    rng = np.random.default_rng(5)
    row_kb = 1536 * 4
    for trial in range(30):
        budget = int(rng.integers(1, 40)) * 2 * row_kb + int(rng.integers(0, 3)) * 100
        m = KVTileManager(budget, budget, dry_run=True)
        o = oracle.manager(budget, budget)
        m.init(); o.init()
        assert m.arena_init(budget, 2 * 1536) == (o.arena_init(budget, 2 * 1536) == 1)
        if trial % 2 == 0:
            for step in range(6):
                m.arena_begin_step(); o.arena_begin()
                for _ in range(int(rng.integers(0, 50))):
                    ok, row = m.arena_stage(1 << 20, row_kb, 2 << 20, row_kb)
                    import ctypes as C
                    r = C.c_int64(-1)
                    ok2 = o.arena_stage(row_kb, row_kb, C.byref(r))
                    assert ok == (ok2 == 1) and (not ok or row == r.value)
                assert m.arena_used_bytes() == o.arena_used()
                assert m.arena_apply_window() == (o.arena_window() == 1)
                m.arena_end_step(); o.arena_end()
        else:
            import ctypes as C
            assert m.streaming_begin() and o.streaming_begin() == 1
            live = set()
            for _ in range(300):
                rid = int(rng.integers(0, 80))
                if rng.random() < 0.35:
                    assert m.streaming_release(rid) == (o.streaming_release(rid) == 1)
                    live.discard(rid)
                else:
                    ch = bool(rng.random() < 0.2)
                    ok, slot, rs = m.streaming_stage(rid, 1 << 20, row_kb, 2 << 20, row_kb, ch)
                    s2, r2 = C.c_int64(-1), C.c_int(0)
                    ok2 = o.streaming_stage(rid, row_kb, row_kb, int(ch), C.byref(s2), C.byref(r2))
                    assert (ok, slot, rs) == (ok2 == 1, s2.value, bool(r2.value))
            assert m.streaming_staged_bytes() == o.streaming_staged_bytes()
            assert m.streaming_apply_window() == (o.streaming_window() == 1)
            m.streaming_end(); o.streaming_end()
