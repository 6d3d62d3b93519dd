"""The per-frame cross-attention loop (kvp/frames.py) on a device: the
reference driver's loop for arena and streaming sessions produces outputs
bitwise identical to the None policy, within tolerance of the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.attention import attention_frames
from test_gpu_kernels import check_bf16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("streaming", [False, True])
def test_per_frame_loop_policies_bitwise(cuda, streaming):
    from kvp import frames as matrix
    from kvp.attention import read_status
    from kvp.traces import motion_config5, qkv
    F, T, H = 4, 300, 2
    D = H * 128
    q, k, v = (t.cuda() for t in qkv(F * T, D, seed=7))
    stream = int(torch.cuda.current_stream().cuda_stream)
    scores = motion_config5("high", frames=F, tiles=(T + 15) // 16, seed=3)
    read_status()
    outs = {}
    for policy in ("none", "recency", "motion", "reuse_weighted"):
        out = torch.empty_like(q)
        matrix.run_frames(q, k, v, out, scores, policy=policy, set_aside=40 * 16 * D * 2 * 2,
                          frames=F, tokens=T, heads=H, stream=stream, streaming=streaming)
        outs[policy] = out.float().cpu().numpy()
    assert read_status() == 0
    for p in outs:
        assert np.array_equal(outs[p], outs["none"]), p
    want = attention_frames(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                            frames=F, tokens=T, heads=H, head_dim=128, mode="cross")
    check_bf16(outs["none"], want, ("per-frame loop", streaming))
