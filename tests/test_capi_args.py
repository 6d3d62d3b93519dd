"""Argument checks of the B200 entry points that refuse bad input before
any CUDA call (CPU only): the QKV producer, LayerNorm, the motion producer
and its threshold, the session's produce / reuse preconditions."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from kvp._lib import AttnDesc, LayerIO, MotionParams, QkvIO, lib

ERR_ARG = -1


def _qkv(**kw):
    base = dict(x=0x1000, w=0x2000, bias=0, q=0, k=0x3000, v=0x4000, arena=0, kvmap=0, rows=256,
                map_row0=0, arena_rows=0, D=256)
    base.update(kw)
    io = QkvIO(base["x"], base["w"], base["bias"], base["q"], base["k"], base["v"], base["arena"],
               base["kvmap"], base["rows"], base["map_row0"], base["arena_rows"], base["D"])
    return lib().kvp_qkv_project_bf16(C.byref(io), None)


@pytest.mark.parametrize("bad", [
    dict(rows=127),                    # fewer rows than one tile half
    dict(D=384),                       # not a multiple of 256
    dict(D=128),
    dict(x=0),                         # missing input
    dict(k=0),
    dict(x=0x1008),                    # not 16-byte aligned
    dict(v=0x4004),
    dict(kvmap=0x5000, arena=0),       # a map needs an arena
    dict(map_row0=-1),
])
def test_qkv_project_rejects(bad):
    assert _qkv(**bad) == ERR_ARG
    assert b"qkv_project" in lib().kvp_last_error()


@pytest.mark.parametrize("args", [
    (0x1000, 0x2000, 0x3000, 0x4000, 10, 12, 1e-5),     # D % 8
    (0x1000, 0x2000, 0x3000, 0x4000, 0, 16, 1e-5),      # no rows
    (0x1000, 0x2000, 0x3000, 0x4000, 10, 16, 0.0),      # eps
    (0x1004, 0x2000, 0x3000, 0x4000, 10, 16, 1e-5),     # misaligned x
    (0, 0x2000, 0x3000, 0x4000, 10, 16, 1e-5),
])
def test_layernorm_rejects(args):
    x, g, b, y, rows, D, eps = args
    rc = lib().kvp_layernorm_bf16(C.c_void_p(x), C.c_void_p(g), C.c_void_p(b), C.c_void_p(y), rows,
                                  D, C.c_float(eps), None)
    assert rc == ERR_ARG


@pytest.mark.parametrize("bad", [
    dict(height=481), dict(width=830), dict(winsize=14), dict(poly_n=4), dict(poly_n=17),
    dict(levels=-1), dict(pyr_scale=1.0), dict(iterations=0), dict(poly_sigma=0.0),
    dict(tile_cells=0), dict(height=16),
])
def test_motion_create_rejects(bad):
    p = dict(height=480, width=832, levels=3, winsize=15, iterations=3, poly_n=5, poly_sigma=1.2,
             pyr_scale=0.5, grid_rows=30, grid_cols=52, tile_cells=16)
    p.update(bad)
    mp = MotionParams(p["height"], p["width"], p["levels"], p["winsize"], p["iterations"],
                      p["poly_n"], p["poly_sigma"], p["pyr_scale"], p["grid_rows"], p["grid_cols"],
                      p["tile_cells"])
    assert not lib().kvp_motion_create(C.byref(mp))
    assert b"motion" in lib().kvp_last_error()


def test_motion_threshold_rejects_and_accepts_nulls():
    L = lib()
    ch = np.random.default_rng(0).random((4, 5)).astype(np.float32)
    assert L.kvp_motion_threshold(ch.ctypes.data, 1, 5, 50.0, None, None, None) == ERR_ARG
    assert L.kvp_motion_threshold(ch.ctypes.data, 4, 5, 101.0, None, None, None) == ERR_ARG
    assert L.kvp_motion_threshold(None, 4, 5, 50.0, None, None, None) == ERR_ARG
    tau = C.c_double(0.0)
    assert L.kvp_motion_threshold(ch.ctypes.data, 4, 5, 50.0, None, None, C.byref(tau)) == 0
    assert tau.value == float(np.percentile(ch[1:].astype(np.float64), 50.0))


def test_session_produce_preconditions_without_device_buffers():
    """A planning-only session (layers = 0) has no device map: produce refuses."""
    from kvp.session import Session
    s = Session(mode="stack", policy="recency", frames=2, tokens=256, hidden=256, elem_bytes=2,
                set_aside=1 << 20)
    s.plan_stack(np.ones((2, 16), np.float32))
    rc = lib().kvp_session_produce(s.h, 0, None, None, None, None, None, None, 0, 512, None)
    assert rc == ERR_ARG
    assert b"produce" in lib().kvp_last_error()
    s.close()


# ---------------------------------------------------------------- attention
ERR_CUDA = -2


def _attn(io_kw=None, **d_kw):
    """kvp_attn_bf16 on fake, aligned addresses: a 2-frame causal launch of
    2 heads over 300-token frames unless overridden."""
    io = dict(q=0x10000, k=0x20000, v=0x30000, out=0x40000, arena=0, kvmap=0, q_rows=600,
              kv_rows=600, arena_rows=0)
    io.update(io_kw or {})
    d = dict(tokens=300, frames=2, q_frame0=0, mode=1, window=0, heads=2, head_dim=128, head0=0,
             nheads=2, flat=0)
    d.update(d_kw)
    lio = LayerIO(*(io[k] for k in ("q", "k", "v", "out", "arena", "kvmap", "q_rows", "kv_rows",
                                    "arena_rows")))
    ld = AttnDesc(*(d[k] for k in ("tokens", "frames", "q_frame0", "mode", "window", "heads",
                                   "head_dim", "head0", "nheads", "flat")))
    return lib().kvp_attn_bf16(C.byref(lio), C.byref(ld), None)


@pytest.mark.parametrize("io_kw,d_kw", [
    (None, dict(head_dim=64)),                       # the kernel is built for 128
    (None, dict(heads=0, nheads=0)),
    (None, dict(tokens=0)),
    (None, dict(frames=0)),
    (None, dict(q_frame0=-1)),
    (None, dict(head0=1)),                           # heads [1, 3) of 2
    (None, dict(nheads=0)),
    (None, dict(window=-1)),
    (None, dict(mode=2)),
    (None, dict(flat=1, mode=0)),                    # flat tiles are causal only
    (None, dict(flat=1, window=2)),
    (None, dict(flat=1, tokens=100, frames=6)),      # flat needs >= 128 tokens per frame
    (None, dict(q_frame0=1)),                        # frames 1..2 need 900 rows
    (dict(kv_rows=599), {}),
    (dict(kvmap=0x50000, arena=0x60000, arena_rows=0), {}),   # a map into an empty arena
    (dict(q=0), {}),
    (dict(out=0), {}),
    (dict(k=0x20008), {}),                           # not 16-byte aligned
    (dict(arena=0x60004, arena_rows=64), {}),
])
def test_attn_bf16_rejects_before_touching_the_device(io_kw, d_kw):
    """Bad descriptors come back as KVP_ERR_ARG with a message, before the
    entry point flushes queued copies or fetches its device status word."""
    assert _attn(io_kw, **d_kw) == ERR_ARG
    assert b"attn_bf16" in lib().kvp_last_error()


@pytest.mark.parametrize("io_kw,d_kw", [
    (None, {}),
    (None, dict(mode=0)),
    (None, dict(flat=1)),
    (None, dict(head0=1, nheads=1, window=2)),
    (dict(kvmap=0x50000, arena=0x60000, arena_rows=64), {}),
])
def test_attn_bf16_valid_descriptors_pass_the_checks(io_kw, d_kw):
    """Descriptors of the shapes the GPU tests launch get past the argument
    checks: without a GPU the call then fails on its first CUDA call (the
    status word), never with KVP_ERR_ARG."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("would launch the kernel on fake addresses")
    assert _attn(io_kw, **d_kw) == ERR_CUDA


def test_attn_bf16_noalloc_rejects_before_touching_the_device():
    """The no-alloc entry point refuses a bad descriptor (and a map passed in
    device memory) before it looks up or writes its static scratch."""
    io = LayerIO(0x10000, 0x20000, 0x30000, 0x40000, 0, 0, 600, 600, 0)
    hmap = np.full(600, -1, dtype=np.int64)
    for d in (AttnDesc(300, 2, 0, 1, 0, 2, 64, 0, 2, 0),      # head_dim 64
              AttnDesc(300, 3, 0, 1, 0, 2, 128, 0, 2, 0)):    # 900 rows of 600
        rc = lib().kvp_attn_bf16_noalloc(C.byref(io), C.byref(d),
                                         hmap.ctypes.data_as(C.c_void_p), None, None)
        assert rc == ERR_ARG
        assert b"attn_bf16" in lib().kvp_last_error()
    # a bad descriptor with a host map is -1, not a capacity refusal
    for d in (AttnDesc(0, 2, 0, 1, 0, 2, 128, 0, 2, 0),        # tokens 0
              AttnDesc(300, 0, 0, 1, 0, 2, 128, 0, 2, 0),      # frames 0
              AttnDesc(300, 2, -5, 1, 0, 2, 128, 0, 2, 0),     # negative q_frame0
              AttnDesc(300, 2, 2**31 - 2, 1, 0, 2, 128, 0, 2, 0)):  # frame index overflows int
        rc = lib().kvp_attn_bf16_noalloc(C.byref(io), C.byref(d),
                                         hmap.ctypes.data_as(C.c_void_p), None, None)
        assert rc == ERR_ARG, (d.tokens, d.frames, d.q_frame0, rc)
    io_dev_map = LayerIO(0x10000, 0x20000, 0x30000, 0x40000, 0, 0x50000, 600, 600, 0)
    rc = lib().kvp_attn_bf16_noalloc(C.byref(io_dev_map), C.byref(AttnDesc(300, 2, 0, 1, 0, 2, 128,
                                                                          0, 2, 0)),
                                     None, None, None)
    assert rc == ERR_ARG


def test_attn_bf16_multi_rejects_before_touching_the_device():
    """kvp_attn_bf16_multi checks every layer's descriptor and that the
    layers share tokens, frames, mode, window and tiling, before any device
    work; q_frame0 and the head range may differ."""
    io = LayerIO(0x10000, 0x20000, 0x30000, 0x40000, 0, 0, 900, 900, 0)
    ios = (LayerIO * 2)(io, io)
    good = AttnDesc(300, 1, 0, 1, 0, 2, 128, 0, 2, 0)
    for other in (AttnDesc(301, 1, 0, 1, 0, 2, 128, 0, 2, 0),    # tokens
                  AttnDesc(300, 2, 0, 1, 0, 2, 128, 0, 2, 0),    # frames
                  AttnDesc(300, 1, 0, 0, 0, 2, 128, 0, 2, 0),    # mode
                  AttnDesc(300, 1, 0, 1, 2, 2, 128, 0, 2, 0)):   # window
        ds = (AttnDesc * 2)(good, other)
        assert lib().kvp_attn_bf16_multi(ios, ds, 2, None) == ERR_ARG
        assert b"differs from layer 0" in lib().kvp_last_error()
    bad = (AttnDesc * 2)(good, AttnDesc(300, 1, 0, 1, 0, 2, 64, 0, 2, 0))   # head_dim 64
    assert lib().kvp_attn_bf16_multi(ios, bad, 2, None) == ERR_ARG
    assert lib().kvp_attn_bf16_multi(ios, (AttnDesc * 2)(good, good), 0, None) == ERR_ARG


def test_session_run_frames_rejects_bad_arguments():
    """kvp_session_run_frames refuses a missing session, descriptor or frame
    range, and a bad descriptor, before any device work."""
    from kvp.session import Session
    s = Session(mode="cross", policy="none", frames=2, tokens=300, hidden=256, elem_bytes=2,
                set_aside=0, layers=0)
    try:
        io = LayerIO(0x10000, 0x20000, 0x30000, 0x40000, 0, 0, 600, 600, 0)
        d = AttnDesc(300, 1, 0, 1, 0, 2, 128, 0, 2, 0)
        scores = np.zeros(2 * 19, dtype=np.float32)
        f = lib().kvp_session_run_frames
        assert f(None, 0, 2, scores.ctypes.data, None, C.byref(io), C.byref(d), None) == ERR_ARG
        assert f(s.h, 0, 0, scores.ctypes.data, None, C.byref(io), C.byref(d), None) == ERR_ARG
        assert f(s.h, -1, 2, scores.ctypes.data, None, C.byref(io), C.byref(d), None) == ERR_ARG
        assert f(s.h, 0, 2, scores.ctypes.data, None, None, C.byref(d), None) == ERR_ARG
        # 3 frames of 300 rows do not fit the 600 rows the buffers hold
        assert f(s.h, 0, 3, scores.ctypes.data, None, C.byref(io), C.byref(d), None) == ERR_ARG
        d64 = AttnDesc(300, 1, 0, 1, 0, 2, 64, 0, 2, 0)
        assert f(s.h, 0, 2, scores.ctypes.data, None, C.byref(io), C.byref(d64), None) == ERR_ARG
    finally:
        s.close()


def test_session_run_frames_batched_rejects_bad_arguments():
    """kvp_session_run_frames_batched refuses a missing session, descriptor or
    frame range, a session it cannot batch (stack mode, streaming slots,
    fewer arenas than frames, no map buffer) and a bad descriptor, all before
    any device work."""
    from kvp.session import Session
    io = LayerIO(0x10000, 0x20000, 0x30000, 0x40000, 0, 0, 600, 600, 0)
    d = AttnDesc(300, 1, 0, 1, 0, 2, 128, 0, 2, 0)
    scores = np.zeros(3 * 19, dtype=np.float32)
    f = lib().kvp_session_run_frames_batched
    maps = C.c_void_p(0x50000)

    def call(s, f0, n, io_=C.byref(io), d_=C.byref(d), m=maps):
        return f(s, f0, n, scores.ctypes.data, io_, d_, m, None)

    s = Session(mode="cross", policy="none", frames=3, tokens=300, hidden=256, elem_bytes=2,
                set_aside=0, layers=0)
    try:
        assert call(None, 0, 2) == ERR_ARG
        assert call(s.h, 0, 0) == ERR_ARG
        assert call(s.h, -1, 2) == ERR_ARG
        assert call(s.h, 0, 2, io_=None) == ERR_ARG
        assert call(s.h, 0, 2, d_=None) == ERR_ARG
        assert call(s.h, 2, 2) == ERR_ARG                      # frames 2, 3 of a 3-frame session
        assert b"past the session" in lib().kvp_last_error()
        # 3 frames of 300 rows do not fit the 600 rows the buffers hold
        assert call(s.h, 0, 3) == ERR_ARG
        d64 = AttnDesc(300, 1, 0, 1, 0, 2, 64, 0, 2, 0)
        assert call(s.h, 0, 2, d_=C.byref(d64)) == ERR_ARG
    finally:
        s.close()
    for kw, what in ((dict(mode="cross", policy="recency", layers=0), b"one per frame"),
                     (dict(mode="cross", policy="recency", layers=0, streaming=True), b"streaming 0"),
                     (dict(mode="stack", policy="recency", layers=0), b"intra or cross")):
        s = Session(frames=3, tokens=300, hidden=256, elem_bytes=2, set_aside=1 << 20, **kw)
        try:
            assert call(s.h, 0, 2) == ERR_ARG, kw
            assert what in lib().kvp_last_error(), (kw, lib().kvp_last_error())
        finally:
            s.close()
