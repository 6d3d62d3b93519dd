"""The GPU motion-trace producer (kvp_motion_*) on a device.

* Flow of one pair against oracle/motion.py (the same steps in numpy):
  median |difference| < 1e-3 px, 99th percentile < 2e-2 px.
* Per-tile change rates of the seeded clip against the oracle (relative
  2e-3) and against the reference's own tool run on the same clip
  (tests/golden/motion_ref_clip.csv, OpenCV): the tolerances of the
  oracle's own pin; reuse flags within the same agreement.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import motion as M
from test_motion_host import compare_rates, reference_clip_trace

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def clip():
    from kvp.traces import synthetic_video
    return synthetic_video(6, seed=5)


def test_gpu_flow_matches_oracle(cuda, clip):
    from kvp.motion import MotionProducer
    mp = MotionProducer()
    d = torch.from_numpy(clip).cuda()
    out = torch.empty(2, 480, 832, device="cuda")
    mp.flow(d[0], d[1], out, int(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    want = M.farneback(clip[0], clip[1])
    diff = np.abs(got - want)
    assert np.median(diff) < 1e-3, np.median(diff)
    assert np.percentile(diff, 99) < 2e-2, np.percentile(diff, 99)
    mp.close()


def test_gpu_trace_matches_oracle_and_reference(cuda, clip):
    from kvp.motion import MotionProducer, threshold
    meta, want, want_reuse, _ = reference_clip_trace()
    mp = MotionProducer()
    d = torch.from_numpy(clip).cuda()
    change = torch.full((len(clip), mp.tiles), -1.0, device="cuda")
    mp.change(d, change, int(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    got = change.cpu().numpy().astype(np.float64)
    oracle_change = M.motion_trace(clip)[0]
    rel = np.abs(got - oracle_change) / np.maximum(oracle_change, 1e-3)
    assert rel.max() < 2e-3, rel.max()
    assert np.array_equal(got[0], got[1])
    compare_rates(got, np.round(want, 6), "gpu vs reference tool")
    tau, reuse, static = threshold(got.astype(np.float32))
    assert abs(tau - meta["tau_reuse"]) / meta["tau_reuse"] < 0.02
    assert (reuse == want_reuse).mean() > 0.93
    mp.close()


def test_motion_rejects_bad_parameters(cuda):
    from kvp.motion import MotionProducer
    with pytest.raises(RuntimeError, match="kvp_motion_create"):
        MotionProducer(height=481)                  # not a multiple of the 30-row grid
    with pytest.raises(RuntimeError, match="kvp_motion_create"):
        MotionProducer(winsize=14)


@pytest.mark.parametrize("params", [
    dict(levels=1, winsize=9, iterations=2, poly_n=7, poly_sigma=1.5),
    dict(levels=0, winsize=5, iterations=1, poly_n=5, poly_sigma=1.1),
])
def test_gpu_flow_other_parameters_match_oracle(cuda, params):
    """Non-default flow parameters on a 240 x 416 clip (15 x 26 grid)."""
    from kvp.motion import MotionProducer
    from kvp.traces import synthetic_video
    clip = synthetic_video(3, seed=8, height=240, width=416)
    mp = MotionProducer(240, 416, grid=(15, 26), **params)
    d = torch.from_numpy(clip).cuda()
    out = torch.empty(2, 240, 416, device="cuda")
    mp.flow(d[1], d[2], out, int(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    want = M.farneback(clip[1], clip[2], pyr_scale=0.5, **params)
    diff = np.abs(out.cpu().numpy() - want)
    assert np.median(diff) < 1e-3 and np.percentile(diff, 99) < 2e-2, (params, np.median(diff))
    change = torch.empty(3, mp.tiles, device="cuda")
    mp.change(d, change, int(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    got = change.cpu().numpy()
    mags = [np.hypot(*M.farneback(clip[f - 1], clip[f], pyr_scale=0.5, **params)) for f in (1, 2)]
    want_change = np.zeros_like(got, dtype=np.float64)
    for f, m in enumerate(mags, start=1):
        want_change[f] = M.tile_means(M.cell_means(m, grid=(15, 26)))
    want_change[0] = want_change[1]
    rel = np.abs(got - want_change) / np.maximum(want_change, 1e-3)
    assert rel.max() < 2e-3, (params, rel.max())
    mp.close()
