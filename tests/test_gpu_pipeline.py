"""The extensions chained on a device: frames -> GPU motion producer (change
rates) -> reuse threshold -> reuse-mode Session (only changed tiles staged)
-> tcgen05 attention through the KVMap.  With K/V that really hold their
unchanged tiles, the output equals the None policy bitwise; the planner's
reuse flags equal the reference rule applied to the same rates."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_motion_to_reuse_to_attention(cuda):
    from kvp import frames as matrix
    from kvp.attention import read_status
    from kvp.motion import MotionProducer, threshold
    from kvp.traces import hold_reused_tiles, qkv, synthetic_video
    F, H = 5, 2
    D = H * 128
    clip = synthetic_video(F, seed=21)                       # 480 x 832, 30 x 52 grid
    mp = MotionProducer()
    change = torch.empty(F, mp.tiles, device="cuda")
    mp.change(torch.from_numpy(clip).cuda(), change, int(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    rates = change.cpu().numpy()
    tau, reuse, static = threshold(rates)
    assert reuse[0].sum() == 0 and 0.3 < reuse[1:].mean() < 0.7
    want = (rates.astype(np.float64) < tau).astype(np.int8)
    want[0] = 0
    assert np.array_equal(reuse, want)
    mp.close()

    T = 1560
    q, k, v = qkv(F * T, D, seed=4)
    hold_reused_tiles(k, v, reuse, tokens=T)
    q, k, v = q.cuda(), k.cuda(), v.cuda()
    stream = int(torch.cuda.current_stream().cuda_stream)
    budget = 40 * 16 * D * 2 * 2
    read_status()
    outs = {}
    for policy in ("none", "motion", "reuse_weighted"):
        out = torch.zeros_like(q)
        tot = matrix.run_reuse_frames(q, k, v, out, rates, reuse, policy=policy, set_aside=budget,
                                      frames=F, tokens=T, heads=H, stream=stream)
        outs[policy] = (out.cpu(), tot)
    assert read_status() == 0
    for policy in ("motion", "reuse_weighted"):
        out, tot = outs[policy]
        assert tot["hits"] > 0
        assert torch.equal(out, outs["none"][0]), policy
