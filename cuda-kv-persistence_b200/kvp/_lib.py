"""ctypes binding of libkvp.so (the C ABI declared in include/*.h).

The library is built in-tree by ``cuda-kv-persistence_b200/build.py`` (or
``__graft_entry__.build()``).  Loading fails loudly when it is missing:
there is no Python or CPU fallback for any kernel.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_native" / "libkvp.so"

c_long_p = C.POINTER(C.c_long)
c_int_p = C.POINTER(C.c_int)


class DeviceInfo(C.Structure):
    _fields_ = [("device", C.c_int), ("sm_count", C.c_int), ("cc_major", C.c_int),
                ("cc_minor", C.c_int), ("l2_bytes", C.c_longlong),
                ("max_persisting_l2_bytes", C.c_longlong),
                ("max_access_policy_window_bytes", C.c_longlong),
                ("persisting_limit_bytes", C.c_longlong), ("hbm_bytes", C.c_longlong)]


class LayerIO(C.Structure):
    _fields_ = [("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("out", C.c_void_p),
                ("arena", C.c_void_p), ("kvmap", C.c_void_p), ("q_rows", C.c_longlong),
                ("kv_rows", C.c_longlong), ("arena_rows", C.c_longlong)]


class AttnDesc(C.Structure):
    _fields_ = [("tokens", C.c_int), ("frames", C.c_int), ("q_frame0", C.c_int),
                ("mode", C.c_int), ("window", C.c_int), ("heads", C.c_int),
                ("head_dim", C.c_int), ("head0", C.c_int), ("nheads", C.c_int),
                ("flat", C.c_int)]


class SessionConfig(C.Structure):
    _fields_ = [("mode", C.c_int), ("window", C.c_int), ("streaming", C.c_int),
                ("policy", C.c_int), ("frames", C.c_int), ("tokens", C.c_int),
                ("hidden", C.c_int), ("tile_tokens", C.c_int), ("elem_bytes", C.c_int),
                ("layers", C.c_int), ("set_aside", C.c_longlong)]


class QkvIO(C.Structure):
    _fields_ = [("x", C.c_void_p), ("w", C.c_void_p), ("bias", C.c_void_p), ("q", C.c_void_p),
                ("k", C.c_void_p), ("v", C.c_void_p), ("arena", C.c_void_p), ("kvmap", C.c_void_p),
                ("rows", C.c_longlong), ("map_row0", C.c_longlong), ("arena_rows", C.c_longlong),
                ("D", C.c_int)]


class MotionParams(C.Structure):
    _fields_ = [("height", C.c_int), ("width", C.c_int), ("levels", C.c_int), ("winsize", C.c_int),
                ("iterations", C.c_int), ("poly_n", C.c_int), ("poly_sigma", C.c_float),
                ("pyr_scale", C.c_float), ("grid_rows", C.c_int), ("grid_cols", C.c_int),
                ("tile_cells", C.c_int)]


class StepInfo(C.Structure):
    _fields_ = [("frame", C.c_int), ("sel_count", C.c_int), ("staged_tiles", C.c_int),
                ("copies", C.c_int), ("map_row0", C.c_longlong), ("map_rows", C.c_longlong),
                ("window_bytes", C.c_longlong), ("staged_bytes", C.c_longlong),
                ("restaged", C.c_int), ("hits", C.c_int)]


# name -> (restype, argtypes); every symbol include/*.h declares.
SIGNATURES = {
    # include/kv_tile_manager.h
    "kvtm_create": (C.c_void_p, [C.c_long, C.c_long]),
    "kvtm_destroy": (None, [C.c_void_p]),
    "kvtm_init": (C.c_int, [C.c_void_p]),
    "kvtm_query_limit": (C.c_long, [C.c_void_p]),
    "kvtm_admit": (C.c_int, [C.c_void_p, C.c_long, C.c_void_p, C.c_long]),
    "kvtm_release": (C.c_int, [C.c_void_p, C.c_long]),
    "kvtm_clear": (None, [C.c_void_p]),
    "kvtm_persisted_bytes": (C.c_long, [C.c_void_p]),
    "kvtm_persisted_tiles": (C.c_int, [C.c_void_p]),
    "kvtm_dev_alloc": (C.c_void_p, [C.c_long]),
    "kvtm_dev_free": (None, [C.c_void_p]),
    "kvtm_arena_init": (C.c_int, [C.c_void_p, C.c_long, C.c_long]),
    "kvtm_arena_begin": (None, [C.c_void_p]),
    "kvtm_arena_stage": (C.c_int, [C.c_void_p, C.c_void_p, C.c_long, C.c_void_p, C.c_long,
                                   c_long_p]),
    "kvtm_arena_window": (C.c_int, [C.c_void_p]),
    "kvtm_arena_end": (None, [C.c_void_p]),
    "kvtm_arena_used": (C.c_long, [C.c_void_p]),
    "kvtm_arena_ptr": (C.c_void_p, [C.c_void_p]),
    "kvtm_streaming_begin": (C.c_int, [C.c_void_p]),
    "kvtm_streaming_stage": (C.c_int, [C.c_void_p, C.c_long, C.c_void_p, C.c_long, C.c_void_p,
                                       C.c_long, C.c_int, c_long_p, c_int_p]),
    "kvtm_streaming_release": (C.c_int, [C.c_void_p, C.c_long]),
    "kvtm_streaming_window": (C.c_int, [C.c_void_p]),
    "kvtm_streaming_end": (None, [C.c_void_p]),
    "kvtm_streaming_staged_bytes": (C.c_long, [C.c_void_p]),
    "kvtm_layout_tiles_per_frame": (C.c_long, [C.c_int, C.c_int]),
    "kvtm_layout_tile_start": (C.c_long, [C.c_int, C.c_int, C.c_long]),
    "kvtm_layout_tile_count": (C.c_int, [C.c_int, C.c_int, C.c_long]),
    "kvtm_create_ex": (C.c_void_p, [C.c_long, C.c_long, C.c_uint]),
    "kvtm_set_stream": (None, [C.c_void_p, C.c_void_p]),
    "kvtm_flush": (C.c_int, [C.c_void_p]),
    "kvtm_pending_copies": (C.c_long, [C.c_void_p]),
    "kvtm_window_log": (C.c_long, [C.c_void_p, c_long_p, c_int_p, C.c_long]),
    "kvtm_reset_calls": (C.c_long, [C.c_void_p]),
    # include/attn_kernel.h
    "attn_forward_launcher": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                     C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_bool]),
    "attn_forward_single_frame": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                         C.c_int, C.c_int]),
    # include/kvp.h
    "kvp_version": (C.c_char_p, []),
    "kvp_last_error": (C.c_char_p, []),
    "kvp_read_status": (C.c_int, [C.c_void_p]),
    "kvp_probe_bounded_wait": (C.c_int, [C.c_longlong, C.c_void_p]),
    "kvp_query_device": (C.c_int, [C.c_int, C.POINTER(DeviceInfo)]),
    "tgp_select": (C.c_int, [C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                             C.c_void_p, c_int_p]),
    "kvp_read_motion_csv": (C.c_int, [C.c_char_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "kvp_stage_rows": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                 C.c_longlong, C.c_void_p]),
    "kvp_attn_fp32": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_longlong,
                                C.c_longlong, C.c_longlong, C.c_void_p]),
    "kvp_attn_bf16": (C.c_int, [C.POINTER(LayerIO), C.POINTER(AttnDesc), C.c_void_p]),
    "kvp_attn_bf16_multi": (C.c_int, [C.POINTER(LayerIO), C.POINTER(AttnDesc), C.c_int, C.c_void_p]),
    "kvp_session_run_frames": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                         C.POINTER(LayerIO), C.POINTER(AttnDesc), C.c_void_p]),
    "kvp_session_run_frames_batched": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                                 C.POINTER(LayerIO), C.POINTER(AttnDesc),
                                                 C.c_void_p, C.c_void_p]),
    "kvp_attn_bf16_noalloc": (C.c_int, [C.POINTER(LayerIO), C.POINTER(AttnDesc), C.c_void_p,
                                        C.POINTER(C.c_int), C.c_void_p]),
    "kvp_session_create": (C.c_void_p, [C.POINTER(SessionConfig)]),
    "kvp_session_destroy": (None, [C.c_void_p]),
    "kvp_session_plan_frame": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p]),
    "kvp_session_plan_frame_reuse": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    "kvp_session_step": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                   C.c_void_p, C.c_int, C.c_void_p]),
    "kvp_session_stage_except": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_longlong,
                                           C.c_longlong, C.c_void_p]),
    "kvp_session_produce": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                      C.c_void_p, C.c_void_p, C.c_void_p, C.c_longlong,
                                      C.c_longlong, C.c_void_p]),
    "kvp_qkv_project_bf16": (C.c_int, [C.c_void_p, C.c_void_p]),
    "kvp_motion_create": (C.c_void_p, [C.c_void_p]),
    "kvp_motion_destroy": (None, [C.c_void_p]),
    "kvp_motion_tiles": (C.c_int, [C.c_void_p]),
    "kvp_motion_flow": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "kvp_motion_trace": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    "kvp_motion_threshold": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_double, C.c_void_p,
                                       C.c_void_p, C.c_void_p]),
    "kvp_layernorm_bf16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_longlong,
                                     C.c_int, C.c_float, C.c_void_p]),
    "kvp_session_plan_stack": (C.c_int, [C.c_void_p, C.c_void_p]),
    "kvp_session_finish": (C.c_int, [C.c_void_p]),
    "kvp_session_info": (C.c_int, [C.c_void_p, C.POINTER(StepInfo)]),
    "kvp_session_slots": (C.c_longlong, [C.c_void_p]),
    "kvp_session_cap_rows": (C.c_longlong, [C.c_void_p]),
    "kvp_session_map": (C.c_int, [C.c_void_p, C.c_longlong, C.c_longlong, C.c_void_p]),
    "kvp_session_copies": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int]),
    "kvp_session_selected": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int]),
    "kvp_session_device_map": (C.c_void_p, [C.c_void_p]),
    "kvp_session_arena": (C.c_void_p, [C.c_void_p, C.c_int]),
    "kvp_session_upload": (C.c_int, [C.c_void_p, C.c_void_p]),
    "kvp_session_stage": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "kvp_session_stage_layer": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                                          C.c_void_p]),
    "kvp_session_window": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p]),
    "kvp_session_clear_window": (C.c_int, [C.c_void_p, C.c_void_p]),
}

_LIB = None


class KvpError(RuntimeError):
    pass


def lib():
    """The loaded libkvp.so (raises if it was never built)."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise KvpError(f"{LIB_PATH} not found: build it with "
                           "`python cuda-kv-persistence_b200/build.py` (no fallback exists)")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def check(rc: int, what: str) -> int:
    if rc < 0:
        msg = lib().kvp_last_error().decode(errors="replace")
        raise KvpError(f"{what} failed (status {rc}): {msg}")
    return rc


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


def on_path_for_tests() -> str:
    return os.fspath(LIB_PATH)
