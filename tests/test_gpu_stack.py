"""Full-size properties of the config-4 stack on the GPU.

One whole layer (12 heads) of the 21-frame x 1560-token block-causal stack
runs through the stack runner (admission, KVMap upload, arena gather,
persisting window, tcgen05 attention) with ReuseWeighted at the device's
max persisting budget and with None:

* outputs are bitwise identical (the reference's policy gate at full size);
* sampled query rows -- first, interior and last rows of frames 0, 10 and
  20, which cross the 128-row tile and frame edges -- match the fp32 oracle
  within the bf16 tolerance;
* the device status word stays clean.
"""

from __future__ import annotations

import ctypes as C
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def test_full_layer_policies_bitwise_and_oracle(cuda):
    from kvp import traces
    from kvp._lib import DeviceInfo, lib
    from kvp.attention import read_status
    from kvp.stack import StackRank
    from oracle.attention import attention_keys
    info = DeviceInfo()
    lib().kvp_query_device(-1, C.byref(info))
    sa = int(info.max_persisting_l2_bytes)
    scores = traces.read_motion_csv(GOLDEN / "motion_config4.csv", 21, 98)
    stream = int(torch.cuda.current_stream().cuda_stream)
    read_status()
    rw = StackRank(p0=0, p1=12, policy="reuse_weighted", set_aside=sa, device=cuda)
    rw.step(scores, stream)
    assert rw.sessions[0].info().staged_tiles > 0
    none = StackRank(p0=0, p1=12, policy="none", set_aside=sa, device=cuda)
    none.step(scores, stream)
    torch.cuda.synchronize()
    assert read_status() == 0
    a, b = rw.chunks[0].o, none.chunks[0].o
    assert torch.equal(a, b), "remapped stack output differs from the None policy"
    T = 1560
    c = rw.chunks[0]
    for h in (0, 7):
        cols = slice(h * 128, (h + 1) * 128)
        q = c.q[:, cols].float().cpu().numpy()
        k = c.k[:, cols].float().cpu().numpy()
        v = c.v[:, cols].float().cpu().numpy()
        got = a[:, cols].float().cpu().numpy()
        for f in (0, 10, 20):
            rows = np.r_[f * T: f * T + 16, f * T + 700: f * T + 716, (f + 1) * T - 16: (f + 1) * T]
            want = attention_keys(q[rows], k[: (f + 1) * T], v[: (f + 1) * T], 1, 128)
            err = float(np.abs(got[rows] - want).max())
            rel = float(np.linalg.norm(got[rows] - want) / np.linalg.norm(want))
            assert err < 2e-2 and rel < 1e-2, (h, f, err, rel)
