"""Temporal-reuse streaming on a device: the Session keeps the slots of tiles
it keeps selecting and stages only new or changed tiles, the tcgen05 kernel
reads frame f's keys through the KVMap.

* K/V that really hold unchanged tiles (each flagged tile repeats the
  previous frame's rows): every policy is bitwise equal to the None policy.
* K/V that do not: kept, unchanged tiles are read from the slot staged in an
  earlier frame; the output matches the oracle run on exactly those K/V rows
  (the arena replayed on the host from the oracle's copy lists) within the
  bf16 tolerance, and differs from the None policy.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.attention import attention_frames
from test_gpu_kernels import check_bf16

pytestmark = pytest.mark.gpu

F, T, H = 5, 300, 2
D = H * 128
NT = (T + 15) // 16


def _inputs(seed):
    from kvp.traces import motion_config2, qkv, reuse_flags
    scores = motion_config2(frames=F, seed=seed, tiles=NT)
    reuse = reuse_flags(scores)
    q, k, v = qkv(F * T, D, seed=seed)
    return scores, reuse, q, k, v


def _run(q, k, v, scores, reuse, policy, set_aside):
    from kvp import frames as matrix
    out = torch.zeros_like(q)
    stream = int(torch.cuda.current_stream().cuda_stream)
    tot = matrix.run_reuse_frames(q, k, v, out, scores, reuse, policy=policy, set_aside=set_aside,
                                  frames=F, tokens=T, heads=H, stream=stream)
    return out.float().cpu().numpy(), tot


BUDGETS = [6 * 16 * D * 2 * 2, NT * 16 * D * 2 * 2]   # 6 tiles, every tile


@pytest.mark.parametrize("set_aside", BUDGETS)
def test_reuse_loop_bitwise_on_held_tiles(cuda, set_aside):
    from kvp.attention import read_status
    from kvp.traces import hold_reused_tiles
    scores, reuse, q, k, v = _inputs(11)
    hold_reused_tiles(k, v, reuse, tokens=T)
    q, k, v = q.cuda(), k.cuda(), v.cuda()
    read_status()
    ref, _ = _run(q, k, v, scores, reuse, "none", set_aside)
    hits = 0
    for policy in ("uniform", "recency", "motion", "reuse_weighted"):
        got, tot = _run(q, k, v, scores, reuse, policy, set_aside)
        hits += tot["hits"]
        assert np.array_equal(got, ref), policy
    assert read_status() == 0
    assert hits > 0        # some frames read a slot staged in an earlier frame
    want = attention_frames(q.float().cpu().numpy(), k.float().cpu().numpy(),
                            v.float().cpu().numpy(), frames=F, tokens=T, heads=H, head_dim=128,
                            mode="intra")
    check_bf16(ref, want, "reuse loop, None")


def _replay_effective_kv(oracle, k, v, scores, reuse, policy, set_aside):
    """K/V rows the kernel reads per frame: the arena replayed from the
    oracle's copy lists (bf16 accounting), base rows where the map is -1."""
    r = oracle.run_reuse(scores, reuse, policy=policy, frames=F, tokens=T, hidden=D,
                         elem_bytes=2, set_aside=set_aside)
    cap = set_aside // (2 * D * 2)
    ak = np.zeros((max(cap, 1), D), np.float32)
    av = np.zeros_like(ak)
    ek, ev = k.copy(), v.copy()
    off = 0
    for f in range(F):
        n = int(r["copies"][f])
        rows, slots = r["copy_rows"][off:off + n], r["copy_slots"][off:off + n]
        off += n
        ak[slots], av[slots] = k[rows], v[rows]
        m = r["maps"][f]
        sel = np.nonzero(m >= 0)[0]
        ek[f * T + sel], ev[f * T + sel] = ak[m[sel]], av[m[sel]]
    return ek, ev, r


@pytest.mark.parametrize("policy", ["uniform", "recency", "reuse_weighted"])
def test_reuse_loop_stale_tiles_match_oracle(cuda, oracle, policy):
    from kvp.attention import read_status
    scores, reuse, q, k, v = _inputs(12)
    set_aside = BUDGETS[1]
    kf, vf = k.float().numpy(), v.float().numpy()
    ek, ev, r = _replay_effective_kv(oracle, kf, vf, scores, reuse, policy, set_aside)
    q, k, v = q.cuda(), k.cuda(), v.cuda()
    read_status()
    got, tot = _run(q, k, v, scores, reuse, policy, set_aside)
    assert read_status() == 0
    assert tot["copies"] == int(r["copies"].sum()) and tot["hits"] == int(r["hits"].sum())
    want = attention_frames(q.float().cpu().numpy(), ek, ev, frames=F, tokens=T, heads=H,
                            head_dim=128, mode="intra")
    check_bf16(got, want, ("reuse loop, stale rows", policy))
    ref, _ = _run(q, k, v, scores, reuse, "none", set_aside)
    assert tot["hits"] > 0 and not np.array_equal(got, ref)
