"""The reference driver's per-frame loop as a library call.

`run_frames` is the loop of src/run_policy_experiment.cu:156-274 for F
frames x T tokens, one layer of H heads, bf16: for every frame f one
Session.step call selects, releases and stages the admitted tiles' rows into
the arena, uploads the KVMap and sets the persisting window over the arena,
and the tcgen05 kernel runs query frame f over key frames 0..f (or over
frame f alone, intra).  Everything is issued on one stream; unlike the
reference there is no device synchronisation per frame.

`run_reuse_frames` is the same loop with temporal reuse: slots keyed by
token position, and only new or changed tiles re-staged.

`run_frames_batched` is the arena-mode loop with the frames' launches
merged: admission needs nothing from the GPU, so every frame is planned
first, each frame's admitted rows go to an arena of its own (with its own
KVMap snapshot), and one grid runs all frames (kvp_attn_bf16_multi).  Each
frame reads the same rows as in the per-frame loop, so outputs are the same.
"""

from __future__ import annotations

import torch

from .attention import attn_bf16, attn_bf16_multi
from .session import Session


def run_frames(q, k, v, out, scores, *, policy: str, set_aside: int, frames: int, tokens: int,
               heads: int, stream: int, streaming: bool = False, events=None,
               mode: str = "cross", window: int = 0, native: bool = False) -> dict:
    """One pass over all frames of a cell.  The Session (device buffers) is
    created before and destroyed after the optional (start, end) CUDA events,
    so a timed pass holds only the per-frame work.  mode "cross" (keys of
    frames 0..f, or of the last `window` frames up to f when window > 0:
    candidates and keys both) or "intra" (keys of frame f).  native: the
    whole loop in one kvp_session_run_frames call (no per-frame Python; the
    per-frame counters are then not collected and come back as None)."""
    hidden = heads * 128
    amode = "causal" if mode == "cross" else "intra"
    s = Session(mode=mode, policy=policy, frames=frames, tokens=tokens, hidden=hidden,
                elem_bytes=2, set_aside=set_aside, streaming=streaming, layers=1,
                window=window if mode == "cross" else 0)
    copies = staged = 0
    try:
        if events:
            events[0].record()
        kp, vp = [k.data_ptr()], [v.data_ptr()]
        if native:
            s.run_frames(0, frames, scores, q, k, v, out, heads=heads, mode=amode,
                         window=window if mode == "cross" else 0, stream=stream)
            copies = staged = None
        for f in range(0 if not native else frames, frames):
            s.step(f, scores, kp, vp, window_layer=0, stream=stream)
            st = s.info()
            copies += st.copies
            staged += st.staged_bytes
            win = window if mode == "cross" else 0
            if policy != "none":
                attn_bf16(q, k, v, out, tokens=tokens, frames=1, q_frame0=f, heads=heads,
                          mode=amode, window=win, kvmap_ptr=s.device_map_ptr(),
                          arena_ptr=s.arena_ptr(0), arena_rows=s.cap_rows, stream=stream)
            else:
                attn_bf16(q, k, v, out, tokens=tokens, frames=1, q_frame0=f, heads=heads,
                          mode=amode, window=win, stream=stream)
        if policy != "none":
            if not native:
                s.clear_window(stream)
        if events:
            events[1].record()
        torch.cuda.synchronize()   # the Session's buffers outlive every launch
        s.finish()
    finally:
        s.close()
    return {"copies": copies, "staged_bytes": staged}


def run_reuse_frames(q, k, v, out, scores, reuse, *, policy: str, set_aside: int, frames: int,
                     tokens: int, heads: int, stream: int, events=None) -> dict:
    """Temporal-reuse pass: per frame f the Session (mode "reuse") selects
    among frame f's tiles, keeps the slots of tiles it keeps selecting, and
    stages only new or changed tiles' rows; the kernel runs frame f's
    queries over frame f's keys through the KVMap (intra).  A kept,
    unchanged tile is read from the slot written in an earlier frame."""
    hidden = heads * 128
    s = Session(mode="reuse", policy=policy, frames=frames, tokens=tokens, hidden=hidden,
                elem_bytes=2, set_aside=set_aside, streaming=True, layers=1)
    tot = {"copies": 0, "restaged": 0, "hits": 0, "staged_bytes": 0}
    try:
        if events:
            events[0].record()
        kp, vp = [k.data_ptr()], [v.data_ptr()]
        for f in range(frames):
            s.step(f, scores, kp, vp, reuse=reuse, window_layer=0, stream=stream)
            st = s.info()
            tot["copies"] += st.copies
            tot["restaged"] += st.restaged
            tot["hits"] += st.hits
            tot["staged_bytes"] = st.staged_bytes
            if policy != "none":
                attn_bf16(q, k, v, out, tokens=tokens, frames=1, q_frame0=f, heads=heads,
                          mode="intra", kvmap_ptr=s.device_map_ptr(), arena_ptr=s.arena_ptr(0),
                          arena_rows=s.cap_rows, stream=stream)
            else:
                attn_bf16(q, k, v, out, tokens=tokens, frames=1, q_frame0=f, heads=heads,
                          mode="intra", stream=stream)
        if policy != "none":
            s.clear_window(stream)
        if events:
            events[1].record()
        torch.cuda.synchronize()
        s.finish()
    finally:
        s.close()
    return tot


def run_frames_batched(q, k, v, out, scores, *, policy: str, set_aside: int, frames: int,
                       tokens: int, heads: int, stream: int, events=None, mode: str = "cross",
                       window: int = 0, native: bool = False) -> dict:
    """Arena-mode per-frame admission (the reference driver's default,
    src/run_policy_experiment.cu:189-256) with one attention grid for all
    frames.  Frame f's admission is planned as in run_frames and staged into
    arena f; its KVMap slice is kept in a device buffer of its own.  One
    persisting window over frame F-1's arena covers the launch.  native: the
    whole pass in one kvp_session_run_frames_batched call (the per-frame
    counters then come back as None)."""
    hidden = heads * 128
    amode = "causal" if mode == "cross" else "intra"
    win = window if mode == "cross" else 0
    persist = policy != "none"
    s = Session(mode=mode, policy=policy, frames=frames, tokens=tokens, hidden=hidden,
                elem_bytes=2, set_aside=set_aside, streaming=False, layers=frames,
                window=win)
    maps = torch.full((frames, frames * tokens), -1, dtype=torch.int64, device=q.device)
    host_maps = torch.empty((frames, frames * tokens), dtype=torch.int64).pin_memory()
    hm = host_maps.numpy()
    ext = torch.cuda.ExternalStream(stream)
    copies = staged = 0
    try:
        if events:
            events[0].record()
        if native:
            s.run_frames_batched(0, frames, scores, q, k, v, out, maps if persist else None,
                                 heads=heads, mode=amode, window=win, stream=stream)
            if events:
                events[1].record()
            torch.cuda.synchronize()
            s.finish()
            return {"copies": None, "staged_bytes": None}
        for f in range(frames):
            st = s.plan_frame(f, scores)
            copies += st.copies
            staged += st.staged_bytes
            if persist:
                s.upload(stream)
                s.stage_layer(f, k.data_ptr(), v.data_ptr(), stream)
                # frame f's KVMap slice, pinned host row f -> device row f on the stream
                r0, n = st.map_row0, st.map_rows
                hm[f, r0:r0 + n] = s.host_map(r0, n)
                with torch.cuda.stream(ext):
                    maps[f, r0:r0 + n].copy_(host_maps[f, r0:r0 + n], non_blocking=True)
        layers = []
        for f in reversed(range(frames)):        # longest key span first
            L = dict(q=q, k=k, v=v, out=out, heads=heads, q_frame0=f)
            if persist:
                L.update(kvmap=maps[f], arena_ptr=s.arena_ptr(f), arena_rows=s.cap_rows)
            layers.append(L)
        if persist:
            s.window(frames - 1, stream)
        attn_bf16_multi(layers, tokens=tokens, frames=1, mode=amode, window=win, stream=stream)
        if persist:
            s.clear_window(stream)
        if events:
            events[1].record()
        torch.cuda.synchronize()
        s.finish()
    finally:
        s.close()
    return {"copies": copies, "staged_bytes": staged}
