"""The motion-trace producer's host side, CPU only.

* oracle/motion.py (Farnebaeck restated from the paper + the reference's
  aggregation) against the reference's own traces/gen_motion_from_video.py,
  which ran OpenCV on the same seeded synthetic clip
  (tests/golden/motion_ref_clip.csv, make_golden.py --only motion):
  per-tile change rates within a few percent, the reuse threshold within 2%.
* The product's threshold (kvp_motion_threshold) bit-exact against
  numpy.percentile and the reference's comparisons.
"""

from __future__ import annotations

import csv
import json
from pathlib import Path

import numpy as np
import pytest

from kvp.motion import threshold
from kvp.traces import synthetic_video
from oracle import motion as M

GOLDEN = Path(__file__).resolve().parent / "golden"


def reference_clip_trace():
    meta = json.loads((GOLDEN / "motion_ref_clip.json").read_text())
    F, T = meta["frames"], meta["num_tiles"]
    change = np.zeros((F, T))
    reuse = np.zeros((F, T), np.int8)
    static = np.zeros((F, T), np.int8)
    with open(GOLDEN / "motion_ref_clip.csv") as fh:
        for row in csv.DictReader(fh):
            f, t = int(row["frame_id"]), int(row["tile_id"])
            change[f, t] = float(row["motion_score"])
            reuse[f, t] = int(row["reuse"])
            static[f, t] = int(row["is_static"])
    return meta, change, reuse, static


def compare_rates(got, want, what):
    """Per-tile rates of an independent implementation of the method against
    OpenCV's: median relative error < 1%, 90th percentile < 3%, max < 15%,
    correlation > 0.999."""
    rel = np.abs(got - want) / np.maximum(np.abs(want), 1e-3)
    assert np.median(rel) < 0.01, (what, np.median(rel))
    assert np.percentile(rel, 90) < 0.03, (what, np.percentile(rel, 90))
    assert rel.max() < 0.15, (what, rel.max())
    assert np.corrcoef(got.ravel(), want.ravel())[0, 1] > 0.999, what


def test_oracle_trace_matches_reference_tool():
    meta, want, want_reuse, _ = reference_clip_trace()
    clip = synthetic_video(meta["frames"], seed=5)
    change, tau, reuse, static = M.motion_trace(clip)
    compare_rates(change, np.round(want, 6), "oracle vs reference tool")
    assert abs(tau - meta["tau_reuse"]) / meta["tau_reuse"] < 0.02
    assert (reuse == want_reuse).mean() > 0.93
    assert reuse[0].sum() == 0 and abs(reuse[1:].mean() - 0.5) < 0.02


def _numpy_threshold(change, q):
    ch = np.asarray(change, np.float32).astype(np.float64)
    tau = float(np.percentile(ch[1:], q))
    reuse = (ch < tau).astype(np.int8)
    reuse[0] = 0
    return tau, reuse, (ch < tau).astype(np.int8)


@pytest.mark.parametrize("q", [50.0, 10.0, 33.3, 90.0, 0.0, 100.0])
def test_threshold_matches_numpy(q):
    rng = np.random.default_rng(int(q * 10))
    for F, T in ((2, 1), (5, 98), (50, 98), (7, 13)):
        ch = rng.random((F, T)).astype(np.float32)
        ch[2 % F, :T // 2] = 0.25                 # ties
        tau, reuse, static = threshold(ch, q)
        wtau, wreuse, wstatic = _numpy_threshold(ch, q)
        assert tau == wtau, (F, T, q)
        assert np.array_equal(reuse, wreuse) and np.array_equal(static, wstatic)


def test_threshold_on_reference_rates():
    """The reference's own rates through the product's threshold reproduce
    its reuse / is_static columns."""
    meta, want, want_reuse, want_static = reference_clip_trace()
    tau, reuse, static = threshold(np.round(want, 6).astype(np.float32))
    assert abs(tau - meta["tau_reuse"]) < 1e-5
    agree = (reuse == want_reuse).mean()
    assert agree > 0.995, agree                 # float32 rounding of the %.6f rates
    assert (static == want_static).mean() > 0.995
