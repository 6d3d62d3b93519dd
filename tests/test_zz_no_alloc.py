"""kvp_attn_bf16_noalloc against kvp_attn_bf16, through the C ABI.

The no-alloc entry point exists for callers that may not allocate device
memory (under an allocator that owns all device memory and forbids stray
cudaMalloc calls, or in a serving loop that cannot take the device-wide
synchronisation of a first-call cudaMalloc).  Its
scratch -- the status word and a device copy of the host-side KVMap -- is a
static device array shared by every call.  This file runs last so that a
failure here never hides the other GPU tests; it must pass both alone in a
fresh process and after the rest of the suite.

Two calls in a row with different inputs and maps: each output must match
the allocating entry point's within the bf16 tolerance of the other tests
(max-abs < 2e-2, rel-L2 < 1e-2; in practice the two are bitwise equal), and
the status word must come back clean both times.  Also: the call without a
map against kvp_attn_bf16 without one; a call without host_status whose map
sits in pinned memory that is refilled only after the stream has passed it;
and the device's free memory, unchanged across calls once the first call
has set the entry point up.
"""

from __future__ import annotations

import ctypes as C
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

BF16_MAX, BF16_REL_L2 = 2e-2, 1e-2


def _case(seed, F=3, T=300, H=2, arena_rows=512):
    rng = np.random.default_rng(seed)
    D = H * 128
    s = 1.0 / math.sqrt(128)
    q, k, v = ((torch.from_numpy(rng.standard_normal((F * T, D)).astype(np.float32)) * s)
               .to(torch.bfloat16).cuda() for _ in range(3))
    kvmap = np.full(F * T, -1, dtype=np.int64)
    rows = rng.choice(F * T, size=arena_rows // 2, replace=False)
    kvmap[rows] = rng.permutation(arena_rows)[: len(rows)]
    arena = torch.zeros(arena_rows, 2 * D, dtype=torch.bfloat16, device="cuda")
    idx = torch.from_numpy(rows).cuda()
    slots = torch.from_numpy(kvmap[rows]).cuda()
    arena[slots, :D] = k[idx]
    arena[slots, D:] = v[idx]
    return q, k, v, arena, kvmap, dict(F=F, T=T, H=H)


def _io_desc(q, k, v, out, arena, kvmap_dev, meta):
    from kvp._lib import AttnDesc, LayerIO
    io = LayerIO(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), arena.data_ptr(),
                 0 if kvmap_dev is None else kvmap_dev.data_ptr(), q.shape[0], k.shape[0],
                 arena.shape[0])
    d = AttnDesc(meta["T"], meta["F"], 0, 1, 0, meta["H"], 128, 0, meta["H"], 0)
    return io, d


def test_noalloc_matches_allocating_entry_point_twice(cuda):
    from kvp._lib import lib
    L = lib()
    stream = torch.cuda.current_stream().cuda_stream
    for seed in (101, 202):   # two calls in a row, different inputs and maps
        q, k, v, arena, kvmap, meta = _case(seed)
        ref = torch.zeros_like(q)
        io, d = _io_desc(q, k, v, ref, arena, torch.from_numpy(kvmap).cuda(), meta)
        assert L.kvp_attn_bf16(C.byref(io), C.byref(d), C.c_void_p(stream)) == 0
        out = torch.full_like(q, float("nan"))
        io2, d2 = _io_desc(q, k, v, out, arena, None, meta)
        status = C.c_int(-1)
        rc = L.kvp_attn_bf16_noalloc(C.byref(io2), C.byref(d2),
                                     kvmap.ctypes.data_as(C.c_void_p), C.byref(status),
                                     C.c_void_p(stream))
        assert rc == 0, L.kvp_last_error().decode()
        assert status.value == 0
        torch.cuda.synchronize()
        a, b = out.float().cpu().numpy(), ref.float().cpu().numpy()
        err = float(np.abs(a - b).max())
        rel = float(np.linalg.norm(a - b) / np.linalg.norm(b))
        assert err < BF16_MAX and rel < BF16_REL_L2, (seed, err, rel)


def test_noalloc_rejects_oversized_map(cuda):
    from kvp._lib import AttnDesc, LayerIO, lib
    L = lib()
    T, F = 1560, 43          # 67,080 rows > 65,536
    x = torch.zeros(8, 128, dtype=torch.bfloat16, device="cuda")
    io = LayerIO(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), 0, 0, F * T, F * T, 0)
    d = AttnDesc(T, F, 0, 1, 0, 1, 128, 0, 1, 0)
    hmap = np.full(F * T, -1, dtype=np.int64)
    rc = L.kvp_attn_bf16_noalloc(C.byref(io), C.byref(d), hmap.ctypes.data_as(C.c_void_p), None,
                                 C.c_void_p(0))
    assert rc == -3
    assert "exceeds" in L.kvp_last_error().decode()


def _compare(out, ref, what):
    a, b = out.float().cpu().numpy(), ref.float().cpu().numpy()
    err = float(np.abs(a - b).max())
    rel = float(np.linalg.norm(a - b) / np.linalg.norm(b))
    assert err < BF16_MAX and rel < BF16_REL_L2, (what, err, rel)


def test_noalloc_without_map_matches_allocating_entry_point(cuda):
    from kvp._lib import lib
    L = lib()
    stream = torch.cuda.current_stream().cuda_stream
    q, k, v, arena, _, meta = _case(303)
    ref = torch.zeros_like(q)
    io, d = _io_desc(q, k, v, ref, arena, None, meta)
    assert L.kvp_attn_bf16(C.byref(io), C.byref(d), C.c_void_p(stream)) == 0
    out = torch.full_like(q, float("nan"))
    io2, d2 = _io_desc(q, k, v, out, arena, None, meta)
    status = C.c_int(-1)
    assert L.kvp_attn_bf16_noalloc(C.byref(io2), C.byref(d2), None, C.byref(status),
                                   C.c_void_p(stream)) == 0, L.kvp_last_error().decode()
    assert status.value == 0
    torch.cuda.synchronize()
    _compare(out, ref, "no map")


def test_noalloc_pinned_map_without_status_then_no_new_device_memory(cuda):
    """host_status = NULL: the call does not synchronise, so the pinned map
    is refilled only after a stream synchronisation.  Once set up, further
    calls take no device memory (cudaMemGetInfo through torch, with no torch
    allocation between the readings)."""
    from kvp._lib import lib
    L = lib()
    stream = torch.cuda.current_stream().cuda_stream
    cases = [_case(seed) for seed in (404, 505)]
    refs, outs = [], []
    for q, k, v, arena, kvmap, meta in cases:
        ref = torch.zeros_like(q)
        io, d = _io_desc(q, k, v, ref, arena, torch.from_numpy(kvmap).cuda(), meta)
        assert L.kvp_attn_bf16(C.byref(io), C.byref(d), C.c_void_p(stream)) == 0
        refs.append(ref)
        outs.append(torch.full_like(q, float("nan")))
    pinned = torch.empty(cases[0][4].size, dtype=torch.int64).pin_memory()
    descs = [_io_desc(c[0], c[1], c[2], o, c[3], None, c[5]) for c, o in zip(cases, outs)]
    torch.cuda.synchronize()

    def call(i):
        pinned.numpy()[:] = cases[i][4]
        io, d = descs[i]
        rc = L.kvp_attn_bf16_noalloc(C.byref(io), C.byref(d),
                                     C.c_void_p(pinned.data_ptr()), None, C.c_void_p(stream))
        assert rc == 0, L.kvp_last_error().decode()
        torch.cuda.current_stream().synchronize()   # the stream has passed the map copy

    call(0)                       # sets up (the entry point has run before in this process or not)
    free_before, _ = torch.cuda.mem_get_info()
    call(1)
    call(0)
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before, (free_before, free_after)
    _compare(outs[0], refs[0], "pinned map, case 0")
    _compare(outs[1], refs[1], "pinned map, case 1")
