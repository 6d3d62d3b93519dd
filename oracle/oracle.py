"""CPU oracle for the remapped-attention admission path (ctypes front end).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline leg as the checker, never by the product package.

Three views of the same reference algorithm
(GauthamMK-0/cuda-kv-persistence, src/run_policy_experiment.cu:156-274 and
the classes it drives):

* ``Oracle``      our plain-C restatement (kvp_oracle.c -> _build/liboracle.so)
* ``RefLib``      the reference's own kvtm_* facade and policy classes, built
                  host-only from the reference sources (_ref/libkvpref.so)
* ``run_ref_driver`` the reference's unmodified driver main() built host-only
                  (_ref/policy_experiment_ref), parsed from its event log

The two _ref builds exist only where the reference sources were available at
build time; fixtures generated from them are committed under tests/golden/.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess
import tempfile
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
BUILD = HERE / "_build"
REF = HERE / "_ref"

POLICIES = {"none": 0, "uniform": 1, "recency": 2, "motion": 3, "reuse_weighted": 4}
POLICY_NAMES = {v: k for k, v in POLICIES.items()}

i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")


def build(ref: str | None = None) -> None:
    """Compile the oracle (and the reference host build when sources exist)."""
    cmd = ["make", "-s", "-C", str(HERE), "all"]
    if ref:
        cmd.append(f"REF={ref}")
    subprocess.run(cmd, check=True)


class _OrcParams(C.Structure):
    _fields_ = [("policy", C.c_int), ("cross", C.c_int), ("streaming", C.c_int),
                ("frames", C.c_int), ("tokens", C.c_int), ("hidden", C.c_int),
                ("tile_tokens", C.c_int), ("elem_bytes", C.c_int), ("window", C.c_int),
                ("set_aside", C.c_int64)]


@dataclass
class TraceResult:
    """Per-frame outputs of one admission loop (see kvp_oracle.h)."""
    maps: np.ndarray          # [F, F*T] int64, host KVMap after frame f staging
    sel_count: np.ndarray     # [F]
    sel_ids: np.ndarray       # [F, slots] raw policy ids
    copy_count: np.ndarray    # [F]
    copy_rows: np.ndarray     # concatenated source rows copied into the arena
    copy_slots: np.ndarray    # matching arena slots
    window_bytes: np.ndarray  # [F] persisting window span, -1 if refused
    staged_bytes: np.ndarray  # [F]
    staged_tiles: np.ndarray  # [F]

    def uploaded_slice(self, f: int, tokens: int, cross: bool, window: int = 0):
        """(row0, map values) the kernel of frame f reads."""
        if not cross:
            r0, r1 = f * tokens, (f + 1) * tokens
        else:
            base = max(0, f - window + 1) if window > 0 else 0
            r0, r1 = base * tokens, (f + 1) * tokens
        return r0, self.maps[f, r0:r1]


class Oracle:
    """ctypes binding of _build/liboracle.so (our C restatement)."""

    def __init__(self):
        path = BUILD / "liboracle.so"
        if not path.exists():
            build()
        L = C.CDLL(str(path))
        self.L = L
        L.orc_select.argtypes = [C.c_int, f32p, C.c_int, C.c_int, C.c_int, C.c_int, i64p,
                                 C.POINTER(C.c_int)]
        L.orc_run_trace.argtypes = [C.POINTER(_OrcParams), f32p, i64p, i32p, i64p, C.c_int,
                                    i32p, i64p, i64p, C.c_int64, i64p, i64p, i32p]
        L.orc_read_motion_csv.argtypes = [C.c_char_p, C.c_int, C.c_int, f32p, C.c_void_p]
        L.orc_run_reuse.argtypes = [C.POINTER(_OrcParams), f32p, C.c_void_p, i64p, i32p, i32p,
                                    i32p, i64p, i64p, C.c_int64, i64p, i64p, i32p]
        L.orc_tiles_per_frame.restype = C.c_int64
        L.orc_tile_start.restype = C.c_int64
        L.orc_tile_start.argtypes = [C.c_int, C.c_int, C.c_int64]
        L.orc_tile_count.argtypes = [C.c_int, C.c_int, C.c_int64]
        L.orc_mgr_create.restype = C.c_void_p
        L.orc_mgr_create.argtypes = [C.c_int64, C.c_int64]
        for n in ("orc_mgr_destroy", "orc_mgr_clear", "orc_mgr_arena_begin",
                  "orc_mgr_arena_end", "orc_mgr_streaming_end"):
            getattr(L, n).argtypes = [C.c_void_p]
            getattr(L, n).restype = None
        for n in ("orc_mgr_init", "orc_mgr_persisted_tiles", "orc_mgr_arena_window",
                  "orc_mgr_streaming_begin", "orc_mgr_streaming_window",
                  "orc_mgr_last_window_prop"):
            getattr(L, n).argtypes = [C.c_void_p]
        for n in ("orc_mgr_query_limit", "orc_mgr_persisted_bytes", "orc_mgr_arena_used",
                  "orc_mgr_streaming_staged_bytes", "orc_mgr_last_window_bytes",
                  "orc_mgr_window_calls", "orc_mgr_reset_calls"):
            getattr(L, n).argtypes = [C.c_void_p]
            getattr(L, n).restype = C.c_int64
        L.orc_mgr_admit.argtypes = [C.c_void_p, C.c_int64, C.c_uint64, C.c_int64]
        L.orc_mgr_release.argtypes = [C.c_void_p, C.c_int64]
        L.orc_mgr_arena_init.argtypes = [C.c_void_p, C.c_int64, C.c_int64]
        L.orc_mgr_arena_stage.argtypes = [C.c_void_p, C.c_int64, C.c_int64,
                                          C.POINTER(C.c_int64)]
        L.orc_mgr_streaming_stage.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int64,
                                              C.c_int, C.POINTER(C.c_int64),
                                              C.POINTER(C.c_int)]
        L.orc_mgr_streaming_release.argtypes = [C.c_void_p, C.c_int64]

    def select(self, policy, scores, max_tiles, tpf=98, total_frames=1):
        s = np.ascontiguousarray(scores, dtype=np.float32)
        out = np.zeros(max(max_tiles, len(s), 1), dtype=np.int64)
        cnt = C.c_int(0)
        pid = POLICIES[policy] if isinstance(policy, str) else int(policy)
        rc = self.L.orc_select(pid, s, len(s), max_tiles, tpf, total_frames, out, C.byref(cnt))
        assert rc == 0
        return out[:cnt.value].copy()

    def read_motion_csv(self, path, frames, num_tiles, with_reuse=False):
        s = np.zeros((frames, num_tiles), dtype=np.float32)
        r = np.zeros((frames, num_tiles), dtype=np.int8)
        n = self.L.orc_read_motion_csv(str(path).encode(), frames, num_tiles, s.reshape(-1),
                                       r.ctypes.data if with_reuse else None)
        assert n >= 0, f"cannot read {path}"
        return (s, r) if with_reuse else s

    def run_trace(self, scores_flat, *, policy, cross, streaming, frames, tokens=1560,
                  hidden=1536, tile_tokens=16, elem_bytes=4, window=0, set_aside=2162688):
        p = _OrcParams(POLICIES[policy], int(cross), int(streaming), frames, tokens, hidden,
                       tile_tokens, elem_bytes, window, set_aside)
        nt = (tokens + tile_tokens - 1) // tile_tokens
        slots = set_aside // (tile_tokens * hidden * elem_bytes * 2)
        sel_cap = max(slots, 1)
        cap_rows = set_aside // (2 * hidden * elem_bytes)
        copy_cap = max(frames * cap_rows, 1)
        scores = np.ascontiguousarray(scores_flat, dtype=np.float32).reshape(-1)
        assert scores.size >= frames * nt
        maps = np.empty((frames, frames * tokens), dtype=np.int64)
        sel_count = np.zeros(frames, np.int32)
        sel_ids = np.zeros((frames, sel_cap), np.int64)
        copy_count = np.zeros(frames, np.int32)
        copy_rows = np.zeros(copy_cap, np.int64)
        copy_slots = np.zeros(copy_cap, np.int64)
        window_bytes = np.zeros(frames, np.int64)
        staged_bytes = np.zeros(frames, np.int64)
        staged_tiles = np.zeros(frames, np.int32)
        rc = self.L.orc_run_trace(C.byref(p), scores, maps.reshape(-1), sel_count,
                                  sel_ids.reshape(-1), sel_cap, copy_count, copy_rows,
                                  copy_slots, copy_cap, window_bytes, staged_bytes,
                                  staged_tiles)
        assert rc == 0, f"orc_run_trace rc={rc}"
        n = int(copy_count.sum())
        return TraceResult(maps, sel_count, sel_ids, copy_count, copy_rows[:n].copy(),
                           copy_slots[:n].copy(), window_bytes, staged_bytes, staged_tiles)

    # manager (accounting restatement) -----------------------------------
    def run_reuse(self, scores_flat, reuse_flat, *, policy, frames, tokens=1560, hidden=1536,
                  tile_tokens=16, elem_bytes=4, set_aside=2162688) -> dict:
        """Temporal-reuse streaming loop (kvp_oracle.c orc_run_reuse)."""
        p = _OrcParams(POLICIES[policy], 0, 1, frames, tokens, hidden, tile_tokens, elem_bytes, 0,
                       set_aside)
        nt = (tokens + tile_tokens - 1) // tile_tokens
        cap_rows = set_aside // (2 * hidden * elem_bytes)
        copy_cap = max(frames * cap_rows, 1)
        scores = np.ascontiguousarray(scores_flat, dtype=np.float32).reshape(-1)
        assert scores.size >= frames * nt
        reuse = None
        if reuse_flat is not None:
            reuse = np.ascontiguousarray(reuse_flat, dtype=np.int8).reshape(-1)
            assert reuse.size >= frames * nt
        out = {k: np.zeros(frames, np.int32) for k in ("copies", "restaged", "hits", "staged_tiles")}
        out.update({k: np.zeros(frames, np.int64) for k in ("window_bytes", "staged_bytes")})
        maps = np.empty((frames, tokens), np.int64)
        copy_rows = np.zeros(copy_cap, np.int64)
        copy_slots = np.zeros(copy_cap, np.int64)
        rc = self.L.orc_run_reuse(C.byref(p), scores, None if reuse is None else reuse.ctypes.data,
                                  maps.reshape(-1), out["copies"], out["restaged"], out["hits"],
                                  copy_rows, copy_slots, copy_cap, out["window_bytes"],
                                  out["staged_bytes"], out["staged_tiles"])
        assert rc == 0, f"orc_run_reuse rc={rc}"
        n = int(out["copies"].sum())
        out.update(maps=maps, copy_rows=copy_rows[:n].copy(), copy_slots=copy_slots[:n].copy())
        return out

    def manager(self, budget, max_window):
        return _OrcMgr(self.L, budget, max_window)


class _OrcMgr:
    def __init__(self, L, budget, max_window):
        self.L = L
        self.h = L.orc_mgr_create(budget, max_window)

    def __del__(self):
        if getattr(self, "h", None):
            self.L.orc_mgr_destroy(self.h)
            self.h = None

    def __getattr__(self, name):
        fn = getattr(self.L, "orc_mgr_" + name)
        return lambda *a: fn(self.h, *a)


# ----------------------------------------------------------------- reference
class RefLib:
    """The reference's kvtm_* facade + policy classes, built host-only."""

    def __init__(self):
        path = REF / "libkvpref.so"
        if not path.exists():
            raise FileNotFoundError(f"{path} (reference host build) not built")
        L = C.CDLL(str(path))
        self.L = L
        L.kvpref_select.argtypes = [C.c_int, f32p, C.c_int, C.c_int, C.c_int, C.c_int, i64p,
                                    C.POINTER(C.c_int)]
        L.kvpref_run_window.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                        C.c_int, C.c_long, f32p, i64p, i64p]
        L.kvtm_create.restype = C.c_void_p
        L.kvtm_create.argtypes = [C.c_long, C.c_long]
        for n in ("kvtm_destroy", "kvtm_clear", "kvtm_arena_begin", "kvtm_arena_end",
                  "kvtm_streaming_end"):
            getattr(L, n).argtypes = [C.c_void_p]
            getattr(L, n).restype = None
        for n in ("kvtm_init", "kvtm_persisted_tiles", "kvtm_arena_window",
                  "kvtm_streaming_begin", "kvtm_streaming_window"):
            getattr(L, n).argtypes = [C.c_void_p]
        for n in ("kvtm_query_limit", "kvtm_persisted_bytes", "kvtm_arena_used",
                  "kvtm_streaming_staged_bytes"):
            getattr(L, n).argtypes = [C.c_void_p]
            getattr(L, n).restype = C.c_long
        L.kvtm_admit.argtypes = [C.c_void_p, C.c_long, C.c_void_p, C.c_long]
        L.kvtm_release.argtypes = [C.c_void_p, C.c_long]
        L.kvtm_dev_alloc.restype = C.c_void_p
        L.kvtm_dev_alloc.argtypes = [C.c_long]
        L.kvtm_dev_free.argtypes = [C.c_void_p]
        L.kvtm_arena_init.argtypes = [C.c_void_p, C.c_long, C.c_long]
        L.kvtm_arena_stage.argtypes = [C.c_void_p, C.c_void_p, C.c_long, C.c_void_p, C.c_long,
                                       C.POINTER(C.c_long)]
        L.kvtm_arena_ptr.restype = C.c_void_p
        L.kvtm_arena_ptr.argtypes = [C.c_void_p]
        L.kvtm_streaming_stage.argtypes = [C.c_void_p, C.c_long, C.c_void_p, C.c_long,
                                           C.c_void_p, C.c_long, C.c_int, C.POINTER(C.c_long),
                                           C.POINTER(C.c_int)]
        L.kvtm_streaming_release.argtypes = [C.c_void_p, C.c_long]
        L.kvpref_run_reuse.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_long,
                                       f32p, C.c_void_p, i64p, i32p, i32p, i32p, i64p, i64p]
        L.kvtm_layout_tiles_per_frame.restype = C.c_long
        L.kvtm_layout_tiles_per_frame.argtypes = [C.c_int, C.c_int]
        L.kvtm_layout_tile_start.restype = C.c_long
        L.kvtm_layout_tile_start.argtypes = [C.c_int, C.c_int, C.c_long]
        L.kvtm_layout_tile_count.argtypes = [C.c_int, C.c_int, C.c_long]

    def select(self, policy, scores, max_tiles, tpf=98, total_frames=1):
        s = np.ascontiguousarray(scores, dtype=np.float32)
        out = np.zeros(max(max_tiles, len(s), 1), dtype=np.int64)
        cnt = C.c_int(0)
        pid = POLICIES[policy] if isinstance(policy, str) else int(policy)
        assert self.L.kvpref_select(pid, s, len(s), max_tiles, tpf, total_frames, out,
                                    C.byref(cnt)) == 0
        return out[:cnt.value].copy()

    def run_window(self, scores_flat, *, policy, streaming, window, frames, tokens=1560,
                   hidden=1536, tile_tokens=16, set_aside=2162688):
        maps = np.empty((frames, frames * tokens), np.int64)
        staged = np.zeros(frames, np.int64)
        s = np.ascontiguousarray(scores_flat, dtype=np.float32).reshape(-1)
        rc = self.L.kvpref_run_window(POLICIES[policy], int(streaming), window, frames, tokens,
                                      hidden, tile_tokens, set_aside, s, maps.reshape(-1),
                                      staged)
        assert rc == 0, rc
        return maps, staged

    def run_reuse(self, scores_flat, reuse_flat, *, policy, frames, tokens=1560, hidden=1536,
                  tile_tokens=16, set_aside=2162688) -> dict:
        """The reference's KVTileManager driven by the temporal-reuse loop of
        ref_stub/ref_shims.cpp (kvpref_run_reuse); fp32 accounting."""
        s = np.ascontiguousarray(scores_flat, dtype=np.float32).reshape(-1)
        r = None if reuse_flat is None else np.ascontiguousarray(reuse_flat, dtype=np.int8).reshape(-1)
        maps = np.empty((frames, tokens), np.int64)
        out = {k: np.zeros(frames, np.int32) for k in ("copies", "restaged", "hits")}
        out.update({k: np.zeros(frames, np.int64) for k in ("staged_bytes", "window_bytes")})
        rc = self.L.kvpref_run_reuse(POLICIES[policy], frames, tokens, hidden, tile_tokens, set_aside,
                                     s, None if r is None else r.ctypes.data, maps.reshape(-1),
                                     out["copies"], out["restaged"], out["hits"], out["staged_bytes"],
                                     out["window_bytes"])
        assert rc == 0, rc
        out["maps"] = maps
        return out


@dataclass
class RefDriverRun:
    """What the reference driver's kernel launches saw, frame by frame."""
    launches: list            # [(frame, row0, n, {abs_row: value})]
    copies: list              # D2D row copies: (frame_at_copy, src_row, dst_slot)
    windows: list             # (frame_at_call, bytes, hitProp)
    stdout: str


def run_ref_driver(csv_path, *, policy, attn_mode, streaming, frames, tokens=1560,
                   hidden=1536, heads=12, tile_tokens=16, set_aside=2162688,
                   workdir=None) -> RefDriverRun:
    """Run the reference's unmodified driver main() (host build) on a motion CSV.

    Q/K/V inputs are sparse zero files of the right size: admission and the
    KVMap never depend on their values.
    """
    exe = REF / "policy_experiment_ref"
    if not exe.exists():
        raise FileNotFoundError(f"{exe} (reference host build) not built")
    elems = frames * tokens * hidden
    with tempfile.TemporaryDirectory(dir=workdir) as td:
        td = Path(td)
        for n in ("q", "k", "v"):
            with open(td / f"{n}.bin", "wb") as fh:
                fh.truncate(elems * 4)
        log = td / "events.log"
        cmd = [str(exe), "--policy", policy, "--attn-mode", attn_mode,
               "--q", str(td / "q.bin"), "--k", str(td / "k.bin"), "--v", str(td / "v.bin"),
               "--motion-csv", str(csv_path), "--out", str(td / "out" / "o.bin"),
               "--frames", str(frames), "--tokens", str(tokens), "--hidden", str(hidden),
               "--heads", str(heads), "--tile-tokens", str(tile_tokens),
               "--set-aside-bytes", str(set_aside)]
        if streaming:
            cmd.append("--streaming")
        env = dict(os.environ, KVP_REF_LOG=str(log))
        proc = subprocess.run(cmd, env=env, capture_output=True, text=True, check=True)
        return _parse_ref_log(log.read_text(), hidden, tokens, proc.stdout)


def _parse_ref_log(text, hidden, tokens, stdout) -> RefDriverRun:
    allocs = []  # (idx, base, size)
    launches, copies, windows = [], [], []
    frame = 0
    row_bytes = hidden * 4

    def locate(ptr):
        for idx, base, size in allocs:
            if base <= ptr < base + size:
                return idx, ptr - base
        return None, None

    for line in text.splitlines():
        parts = line.split()
        tag = parts[0]
        if tag == "A":
            allocs.append((int(parts[1]), int(parts[2]), int(parts[3])))
        elif tag == "c" and int(parts[1]) == 3:
            dst, src, nbytes = int(parts[2]), int(parts[3]), int(parts[4])
            si, so = locate(src)
            di, do = locate(dst)
            # driver allocation order: q, k, v, out, arena, kvmap (run_policy_experiment.cu:127-149)
            if si == 1 and do % (2 * row_bytes) == 0:
                copies.append((frame, so // row_bytes, do // (2 * row_bytes)))
        elif tag == "W":
            windows.append((frame, int(parts[2]), int(parts[3])))
        elif tag == "K":
            f, cross, T = int(parts[1]), int(parts[2]), int(parts[3])
            n = int(parts[11])
            row0 = 0 if cross else f * T
            vals = {}
            for kv in parts[12:]:
                i, v = kv.split(":")
                vals[row0 + int(i)] = int(v)
            launches.append((f, row0, n, vals))
            frame = f + 1
    return RefDriverRun(launches, copies, windows, stdout)
