"""Attention entry points over the C ABI (torch tensors are device memory only).

* ``attn_bf16``   -- tcgen05 remapped attention, one layer (kvp_attn_bf16)
* ``attn_bf16_multi`` -- several layers / head chunks in one launch
  (kvp_attn_bf16_multi)
* ``attn_fp32``   -- FP32 remapped attention over a key span (kvp_attn_fp32)
* ``attn_forward_single_frame`` / ``attn_forward_launcher`` -- the
  reference's entry points (src/attn_kernel.h:15-29), fp32
"""

from __future__ import annotations

import ctypes as C

from ._lib import AttnDesc, KvpError, LayerIO, check, lib


def _ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


def _stream(stream) -> int:
    if stream is None:
        import torch
        return int(torch.cuda.current_stream().cuda_stream)
    return int(stream)


def attn_bf16(q, k, v, out, *, tokens: int, frames: int, heads: int, q_frame0: int = 0,
              mode: str = "causal", window: int = 0, head0: int = 0, nheads: int | None = None,
              flat: bool = False, arena=None, arena_rows: int = 0, kvmap=None, kvmap_ptr: int = 0,
              arena_ptr: int = 0, stream=None) -> None:
    """Remapped bf16 attention for query frames [q_frame0, q_frame0+frames).

    q/k/v/out: bf16 [rows, heads*128] CUDA tensors; arena bf16 [rows, 2*D];
    kvmap int64 [kv_rows] indexed by absolute key row (or raw pointers via
    kvmap_ptr / arena_ptr, e.g. a Session's device buffers)."""
    io = LayerIO(_ptr(q), _ptr(k), _ptr(v), _ptr(out), arena_ptr or _ptr(arena),
                 kvmap_ptr or _ptr(kvmap), q.shape[0], k.shape[0],
                 arena_rows if (arena is not None or arena_ptr) else 0)
    d = AttnDesc(tokens, frames, q_frame0, {"intra": 0, "causal": 1, "cross": 1}[mode], window,
                 heads, 128, head0, heads - head0 if nheads is None else nheads, int(flat))
    check(lib().kvp_attn_bf16(C.byref(io), C.byref(d), C.c_void_p(_stream(stream))), "kvp_attn_bf16")


def attn_bf16_multi(layers, *, tokens: int, frames: int, q_frame0: int = 0, mode: str = "causal",
                    window: int = 0, flat: bool = False, stream=None) -> None:
    """attn_bf16 over several layers or head chunks of one shape in a single
    launch.  `layers`: dicts with q, k, v, out (bf16 [rows, h*128] tensors),
    heads, and optionally head0, nheads, q_frame0, arena / arena_ptr,
    arena_rows, kvmap / kvmap_ptr (as in attn_bf16)."""
    n = len(layers)
    ios = (LayerIO * n)()
    ds = (AttnDesc * n)()
    m = {"intra": 0, "causal": 1, "cross": 1}[mode]
    for i, L in enumerate(layers):
        arena, kvmap = L.get("arena"), L.get("kvmap")
        arena_ptr, kvmap_ptr = L.get("arena_ptr", 0), L.get("kvmap_ptr", 0)
        ios[i] = LayerIO(_ptr(L["q"]), _ptr(L["k"]), _ptr(L["v"]), _ptr(L["out"]),
                         arena_ptr or _ptr(arena), kvmap_ptr or _ptr(kvmap), L["q"].shape[0],
                         L["k"].shape[0],
                         L.get("arena_rows", 0) if (arena is not None or arena_ptr) else 0)
        heads = L["heads"]
        head0 = L.get("head0", 0)
        ds[i] = AttnDesc(tokens, frames, L.get("q_frame0", q_frame0), m, window, heads, 128, head0,
                         L.get("nheads") or heads - head0, int(flat))
    check(lib().kvp_attn_bf16_multi(ios, ds, n, C.c_void_p(_stream(stream))), "kvp_attn_bf16_multi")


def attn_fp32(q, k, v, out, *, T: int, heads: int, k_lo: int, k_hi: int, arena=None,
              kvmap=None, arena_rows: int = -1, stream=None) -> None:
    D = heads * 128
    check(lib().kvp_attn_fp32(_ptr(q), _ptr(k), _ptr(v), _ptr(arena), _ptr(kvmap), _ptr(out), T,
                              D, heads, k_lo, k_hi, arena_rows, C.c_void_p(_stream(stream))),
          "kvp_attn_fp32")


def attn_forward_single_frame(q_f, k, v, arena, kvmap_f, out_f, T, D, heads, cross, frame_idx):
    """src/attn_kernel.h:25-29 (legacy default stream)."""
    lib().attn_forward_single_frame(_ptr(q_f), _ptr(k), _ptr(v), _ptr(arena), _ptr(kvmap_f),
                                    _ptr(out_f), T, D, heads, int(cross), frame_idx)


def attn_forward_launcher(q, k, v, arena, kvmap, out, frames, T, D, heads, remap):
    """src/attn_kernel.h:15-19 (legacy default stream)."""
    lib().attn_forward_launcher(_ptr(q), _ptr(k), _ptr(v), _ptr(arena), _ptr(kvmap), _ptr(out),
                                frames, T, D, heads, bool(remap))


def read_status(stream=None) -> int:
    """Device status word (bit0 map out of range, bit1 timeout); clears it."""
    rc = lib().kvp_read_status(C.c_void_p(_stream(stream)))
    if rc < 0:
        raise KvpError("kvp_read_status failed")
    return rc
