"""Argument checks of the B200 entry points that refuse bad input before
any CUDA call (CPU only): the QKV producer, LayerNorm, the motion producer
and its threshold, the session's produce / reuse preconditions."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from kvp._lib import MotionParams, QkvIO, lib

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
