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
"""

from __future__ import annotations

import torch

from .attention import attn_bf16
from .session import Session


def run_frames(q, k, v, out, scores, *, policy: str, set_aside: int, frames: int, tokens: int,
               heads: int, stream: int, streaming: bool = False, events=None,
               mode: str = "cross", window: int = 0) -> dict:
    """One pass over all frames of a cell.  The Session (device buffers) is
    created before and destroyed after the optional (start, end) CUDA events,
    so a timed pass holds only the per-frame work.  mode "cross" (keys of
    frames 0..f, or of the last `window` frames up to f when window > 0:
    candidates and keys both) or "intra" (keys of frame f)."""
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
        for f in range(frames):
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
