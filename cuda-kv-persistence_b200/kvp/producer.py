"""The block's LayerNorm and QKV projection on the tcgen05 producer
(kvp_layernorm_bf16, kvp_qkv_project_bf16), with the arena written in the
epilogue.  Mirrors src/backbone.py:13-33 (nn.LayerNorm(D), nn.Linear(D, 3D),
qkv.view(b, t, 3, heads, head_dim)) in bf16 with fp32 accumulation; fails
loudly without libkvp.so."""

from __future__ import annotations

import ctypes as C

from ._lib import QkvIO, check, lib
from .attention import _ptr, _stream


def layernorm(x, gamma, beta, y, *, eps: float = 1e-5, stream=None) -> None:
    """y = LayerNorm(x) * gamma + beta; x, y bf16 [rows, D], gamma/beta fp32 [D]."""
    check(lib().kvp_layernorm_bf16(C.c_void_p(_ptr(x)), C.c_void_p(_ptr(gamma)),
                                   C.c_void_p(_ptr(beta)), C.c_void_p(_ptr(y)), x.shape[0],
                                   x.shape[1], C.c_float(eps), C.c_void_p(_stream(stream))),
          "kvp_layernorm_bf16")


def qkv_project(x, w, bias, q, k, v, *, arena=None, arena_ptr: int = 0, arena_rows: int = 0,
                kvmap=None, kvmap_ptr: int = 0, map_row0: int = 0, stream=None) -> None:
    """q | k | v = x . w^T + bias, split by columns (bf16 [rows, D] each; q
    may be None).  With a KVMap (int64, indexed by map_row0 + row), row r's
    K and V also land in arena row kvmap[map_row0 + r] when that entry is in
    [0, arena_rows)."""
    io = QkvIO(_ptr(x), _ptr(w), _ptr(bias), _ptr(q), _ptr(k), _ptr(v),
               arena_ptr or _ptr(arena), kvmap_ptr or _ptr(kvmap), x.shape[0], map_row0,
               arena_rows, x.shape[1])
    check(lib().kvp_qkv_project_bf16(C.byref(io), C.c_void_p(_stream(stream))),
          "kvp_qkv_project_bf16")
