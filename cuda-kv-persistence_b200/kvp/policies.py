"""Tile gating policies (src/tile_gating_policy.h:8-68) through tgp_select."""

from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import check, lib

POLICIES = {"none": 0, "uniform": 1, "recency": 2, "motion": 3, "reuse_weighted": 4}


def select(policy, scores, max_tiles: int, tiles_per_frame: int = 98,
           total_frames: int = 1) -> np.ndarray:
    """ids chosen by ``policy`` among ``len(scores)`` candidates (int64 array).

    Same contract as TileGatingPolicy::select: at most max_tiles ids
    (Uniform returns exactly max_tiles, not clamped to the candidates)."""
    pid = POLICIES[policy] if isinstance(policy, str) else int(policy)
    s = np.ascontiguousarray(scores, dtype=np.float32)
    out = np.zeros(max(int(max_tiles), len(s), 1), dtype=np.int64)
    cnt = C.c_int(0)
    check(lib().tgp_select(pid, s.ctypes.data, len(s), int(max_tiles), int(tiles_per_frame),
                           int(total_frames), out.ctypes.data, C.byref(cnt)), "tgp_select")
    return out[:max(cnt.value, 0)].copy()
