"""Session: the per-frame KVMap / admission emitter over the C ABI.

Mirrors the host loop of src/run_policy_experiment.cu:156-274 (select ->
release -> stage -> KVMap) for intra, cross (optionally windowed) and
whole-stack modes.  With ``layers=0`` it only plans on the host (no GPU).
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._lib import KvpError, SessionConfig, StepInfo, check, lib
from .policies import POLICIES

MODES = {"intra": 0, "cross": 1, "stack": 2, "reuse": 3}


@dataclass
class Step:
    frame: int
    sel_count: int
    staged_tiles: int
    copies: int
    map_row0: int
    map_rows: int
    window_bytes: int
    staged_bytes: int
    restaged: int = 0
    hits: int = 0


class Session:
    def __init__(self, *, mode="cross", policy="recency", frames, tokens=1560, hidden=1536,
                 tile_tokens=16, elem_bytes=2, set_aside=2162688, streaming=False, window=0,
                 layers=0):
        cfg = SessionConfig(MODES[mode], window, int(streaming),
                            POLICIES[policy] if isinstance(policy, str) else int(policy), frames,
                            tokens, hidden, tile_tokens, elem_bytes, layers, set_aside)
        self._L = lib()
        self.h = self._L.kvp_session_create(C.byref(cfg))
        if not self.h:
            raise KvpError("kvp_session_create failed: " + self._L.kvp_last_error().decode())
        self.mode, self.frames, self.tokens, self.hidden = mode, frames, tokens, hidden
        self.layers = layers
        self.map_len = frames * tokens

    def close(self):
        if getattr(self, "h", None):
            self._L.kvp_session_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    @property
    def slots(self) -> int:
        return int(self._L.kvp_session_slots(self.h))

    @property
    def cap_rows(self) -> int:
        return int(self._L.kvp_session_cap_rows(self.h))

    def plan_frame(self, frame: int, scores_flat: np.ndarray, reuse=None) -> Step:
        """reuse ([frames][tiles] int8, 1 = tile unchanged) is read in reuse
        mode only; None = every tile changed."""
        s = np.ascontiguousarray(scores_flat, dtype=np.float32).reshape(-1)
        if self.mode == "reuse":
            r = None if reuse is None else np.ascontiguousarray(reuse, dtype=np.int8).reshape(-1)
            check(self._L.kvp_session_plan_frame_reuse(self.h, frame, s.ctypes.data,
                                                       None if r is None else r.ctypes.data),
                  "plan_frame")
        else:
            check(self._L.kvp_session_plan_frame(self.h, frame, s.ctypes.data), "plan_frame")
        return self.info()

    def plan_stack(self, scores_flat: np.ndarray) -> Step:
        s = np.ascontiguousarray(scores_flat, dtype=np.float32).reshape(-1)
        check(self._L.kvp_session_plan_stack(self.h, s.ctypes.data), "plan_stack")
        return self.info()

    def finish(self):
        check(self._L.kvp_session_finish(self.h), "finish")

    def info(self) -> Step:
        i = StepInfo()
        check(self._L.kvp_session_info(self.h, C.byref(i)), "info")
        return Step(i.frame, i.sel_count, i.staged_tiles, i.copies, i.map_row0, i.map_rows,
                    i.window_bytes, i.staged_bytes, i.restaged, i.hits)

    def host_map(self, row0: int = 0, n: int | None = None) -> np.ndarray:
        n = self.map_len - row0 if n is None else n
        out = np.empty(n, dtype=np.int64)
        check(self._L.kvp_session_map(self.h, row0, n, out.ctypes.data), "map")
        return out

    def copies(self) -> np.ndarray:
        n = self._L.kvp_session_copies(self.h, None, 0)
        out = np.empty((max(n, 1), 2), dtype=np.int32)
        self._L.kvp_session_copies(self.h, out.ctypes.data, n)
        return out[:n]

    def selected(self) -> np.ndarray:
        n = self._L.kvp_session_selected(self.h, None, 0)
        out = np.empty(max(n, 1), dtype=np.int64)
        self._L.kvp_session_selected(self.h, out.ctypes.data, n)
        return out[:n]

    # device side ------------------------------------------------------
    def device_map_ptr(self) -> int:
        return int(self._L.kvp_session_device_map(self.h) or 0)

    def arena_ptr(self, layer: int) -> int:
        return int(self._L.kvp_session_arena(self.h, layer) or 0)

    def upload(self, stream: int = 0):
        check(self._L.kvp_session_upload(self.h, C.c_void_p(stream)), "upload")

    def stage(self, k_ptrs, v_ptrs, stream: int = 0):
        n = len(k_ptrs)
        ka = (C.c_void_p * n)(*k_ptrs)
        va = (C.c_void_p * n)(*v_ptrs)
        check(self._L.kvp_session_stage(self.h, ka, va, C.c_void_p(stream)), "stage")

    def stage_layer(self, layer: int, k_ptr: int, v_ptr: int, stream: int = 0):
        check(self._L.kvp_session_stage_layer(self.h, layer, C.c_void_p(k_ptr), C.c_void_p(v_ptr),
                                              C.c_void_p(stream)), "stage_layer")

    def step(self, frame: int, scores_flat: np.ndarray, k_ptrs, v_ptrs, *, reuse=None,
             window_layer: int = 0, stream: int = 0):
        """plan_frame + upload + stage + window(window_layer) in one native
        call (only plan_frame for the None policy); window_layer < 0 skips
        the window.  Read info() for the step's counters."""
        s = np.ascontiguousarray(scores_flat, dtype=np.float32).reshape(-1)
        r = None
        if reuse is not None and self.mode == "reuse":
            r = np.ascontiguousarray(reuse, dtype=np.int8).reshape(-1)
        n = len(k_ptrs)
        ka = (C.c_void_p * max(n, 1))(*k_ptrs)
        va = (C.c_void_p * max(n, 1))(*v_ptrs)
        check(self._L.kvp_session_step(self.h, frame, s.ctypes.data,
                                       None if r is None else r.ctypes.data, ka, va, window_layer,
                                       C.c_void_p(stream)), "step")

    def run_frames(self, f0: int, nframes: int, scores_flat: np.ndarray, q, k, v, out, *,
                   heads: int, mode: str = "causal", window: int = 0, reuse=None,
                   stream: int = 0):
        """The per-frame loop of one layer in one native call
        (kvp_session_run_frames): step(f) then the attention of query frame f
        through this step's KVMap and arena 0, for f in [f0, f0 + nframes)."""
        from ._lib import AttnDesc, LayerIO
        sflat = np.ascontiguousarray(scores_flat, dtype=np.float32).reshape(-1)
        r = None
        if reuse is not None and self.mode == "reuse":
            r = np.ascontiguousarray(reuse, dtype=np.int8).reshape(-1)
        io = LayerIO(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), 0, 0, q.shape[0],
                     k.shape[0], 0)
        d = AttnDesc(self.tokens, 1, f0, {"intra": 0, "causal": 1}[mode], window, heads, 128, 0,
                     heads, 0)
        check(self._L.kvp_session_run_frames(self.h, f0, nframes, sflat.ctypes.data,
                                             None if r is None else r.ctypes.data, C.byref(io),
                                             C.byref(d), C.c_void_p(stream)), "run_frames")

    def run_frames_batched(self, f0: int, nframes: int, scores_flat: np.ndarray, q, k, v, out,
                           maps, *, heads: int, mode: str = "causal", window: int = 0,
                           stream: int = 0):
        """The dense-arena per-frame loop with all frames' attention in one
        grid, in one native call (kvp_session_run_frames_batched): frame
        f0 + i planned, its KVMap slice uploaded into maps[i] and its rows
        staged into arena i; then one kvp_attn_bf16_multi over the frames.
        maps: device int64 [nframes, frames * tokens] (None for the None
        policy)."""
        from ._lib import AttnDesc, LayerIO
        sflat = np.ascontiguousarray(scores_flat, dtype=np.float32).reshape(-1)
        io = LayerIO(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), 0, 0, q.shape[0],
                     k.shape[0], 0)
        d = AttnDesc(self.tokens, 1, f0, {"intra": 0, "causal": 1}[mode], window, heads, 128, 0,
                     heads, 0)
        mp = None if maps is None else C.c_void_p(maps.data_ptr())
        check(self._L.kvp_session_run_frames_batched(self.h, f0, nframes, sflat.ctypes.data,
                                                     C.byref(io), C.byref(d), mp,
                                                     C.c_void_p(stream)), "run_frames_batched")

    def stage_except(self, k_ptrs, v_ptrs, skip_row0: int, skip_rows: int, stream: int = 0):
        """stage() without the source rows [skip_row0, skip_row0 + skip_rows)."""
        n = len(k_ptrs)
        ka = (C.c_void_p * max(n, 1))(*k_ptrs)
        va = (C.c_void_p * max(n, 1))(*v_ptrs)
        check(self._L.kvp_session_stage_except(self.h, ka, va, skip_row0, skip_rows,
                                               C.c_void_p(stream)), "stage_except")

    def produce(self, layer: int, x, w, bias, q, k, v, *, row0: int, stream: int = 0):
        """Layer `layer`'s QKV projection of rows [row0, row0 + len(x)) with
        this step's KVMap: mapped rows land in the arena in the epilogue
        (call upload() first; skip these rows in stage_except)."""
        def p(t):
            return None if t is None else C.c_void_p(t.data_ptr())
        check(self._L.kvp_session_produce(self.h, layer, p(x), p(w), p(bias), p(q), p(k), p(v),
                                          row0, x.shape[0], C.c_void_p(stream)), "produce")

    def window(self, layer: int, stream: int = 0):
        check(self._L.kvp_session_window(self.h, layer, C.c_void_p(stream)), "window")

    def clear_window(self, stream: int = 0):
        check(self._L.kvp_session_clear_window(self.h, C.c_void_p(stream)), "clear_window")
