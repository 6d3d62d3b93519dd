"""The tcgen05 QKV producer and LayerNorm (kvp_qkv_project_bf16,
kvp_layernorm_bf16) on a device, and sessions that produce K/V straight into
the arena.

* Numerics: against the CPU restatement (oracle/qkv.py) on the same
  bf16-rounded inputs, bf16 tolerance (max-abs 2e-2, relative L2 1e-2); the
  reference block's own outputs (tests/golden/qkv_ref.npz) within 3e-2.
* Arena: every mapped row's arena K/V halves are bitwise the base rows,
  unmapped arena rows are untouched, an entry past the arena sets status
  bit 0 and writes nothing.
* Sessions: attention over an arena the producer wrote is bitwise equal to
  the None policy and to the gather path (stack and per-frame cross).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.qkv import layernorm as ln_ref
from oracle.qkv import qkv_params, qkv_split
from test_gpu_kernels import check_bf16

pytestmark = pytest.mark.gpu


def _bf(a, dev="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev).to(torch.bfloat16)


def _f(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("rows,D", [(128, 256), (300, 256), (1560, 1536), (4100, 512), (777, 768)])
def test_qkv_project_matches_oracle(cuda, rows, D):
    from kvp.attention import read_status
    from kvp.producer import qkv_project
    rng = np.random.default_rng(rows + D)
    x = _bf(rng.standard_normal((rows, D)))
    w = _bf(0.02 * rng.standard_normal((3 * D, D)))
    b = torch.from_numpy((0.1 * rng.standard_normal(3 * D)).astype(np.float32)).cuda()
    q, k, v = (torch.empty(rows, D, dtype=torch.bfloat16, device="cuda") for _ in range(3))
    read_status()
    qkv_project(x, w, b, q, k, v)
    torch.cuda.synchronize()
    assert read_status() == 0
    wq, wk, wv = qkv_split(_f(x), _f(w), _f(b))
    for got, want, name in ((q, wq, "q"), (k, wk, "k"), (v, wv, "v")):
        check_bf16(_f(got), want, (name, rows, D))
    # no bias, no Q output
    k2, v2 = torch.empty_like(k), torch.empty_like(v)
    qkv_project(x, w, None, None, k2, v2)
    _, wk0, wv0 = qkv_split(_f(x), _f(w), None)
    check_bf16(_f(k2), wk0, "k no bias")
    check_bf16(_f(v2), wv0, "v no bias")


def test_qkv_project_writes_mapped_rows_to_arena(cuda):
    from kvp.attention import read_status
    from kvp.producer import qkv_project
    rows, D, cap = 700, 512, 400
    rng = np.random.default_rng(3)
    x = _bf(rng.standard_normal((rows, D)))
    w = _bf(0.02 * rng.standard_normal((3 * D, D)))
    b = torch.from_numpy((0.1 * rng.standard_normal(3 * D)).astype(np.float32)).cuda()
    q, k, v = (torch.empty(rows, D, dtype=torch.bfloat16, device="cuda") for _ in range(3))
    map_row0 = 1000                       # x's row r is absolute row map_row0 + r
    kvmap = np.full(map_row0 + rows + 50, -1, np.int64)
    mapped = rng.choice(rows, size=cap, replace=False)
    slots = rng.permutation(cap)
    kvmap[map_row0 + mapped] = slots
    kvmap[map_row0 + 5] = cap + 7         # past the arena: reported, not written
    mapped_ok = mapped[mapped != 5]
    sentinel = torch.full((cap + 8, 2 * D), 3.0, dtype=torch.bfloat16, device="cuda")
    arena = sentinel.clone()
    read_status()
    qkv_project(x, w, b, q, k, v, arena=arena, arena_rows=cap,
                kvmap=torch.from_numpy(kvmap).cuda(), map_row0=map_row0)
    torch.cuda.synchronize()
    assert read_status() == 1
    a = arena.cpu()
    sl = torch.from_numpy(kvmap[map_row0 + mapped_ok])
    rows_t = torch.from_numpy(mapped_ok)
    assert torch.equal(a[sl, :D], k.cpu()[rows_t])
    assert torch.equal(a[sl, D:], v.cpu()[rows_t])
    untouched = np.setdiff1d(np.arange(cap + 8), kvmap[map_row0 + mapped_ok])
    assert torch.equal(a[torch.from_numpy(untouched)], sentinel.cpu()[torch.from_numpy(untouched)])
    # the base rows are the unmapped run's
    q2, k2, v2 = (torch.empty_like(q) for _ in range(3))
    qkv_project(x, w, b, q2, k2, v2)
    assert torch.equal(q, q2) and torch.equal(k, k2) and torch.equal(v, v2)


@pytest.mark.parametrize("rows,D", [(333, 256), (1560, 1536), (77, 2048), (100, 200)])
def test_layernorm_matches_oracle(cuda, rows, D):
    """Register-resident rows for D a multiple of 256 (up to 2048), the
    three-pass kernel otherwise (D = 200)."""
    from kvp.producer import layernorm
    rng = np.random.default_rng(rows)
    x = _bf(3.0 + 2.0 * rng.standard_normal((rows, D)))
    gamma = torch.from_numpy((1 + 0.1 * rng.standard_normal(D)).astype(np.float32)).cuda()
    beta = torch.from_numpy((0.1 * rng.standard_normal(D)).astype(np.float32)).cuda()
    y = torch.empty_like(x)
    layernorm(x, gamma, beta, y)
    check_bf16(_f(y), ln_ref(_f(x), _f(gamma), _f(beta)), ("layernorm", rows, D))


def test_producer_matches_reference_block(cuda):
    """LayerNorm + QKV producer against the reference DiTSelfAttentionBlock's
    outputs on the golden's seeded inputs (fp32 in the reference, bf16 here)."""
    from pathlib import Path
    from kvp.producer import layernorm, qkv_project
    g = np.load(Path(__file__).resolve().parent / "golden" / "qkv_ref.npz")
    x, gamma, beta, w, b = qkv_params(int(g["seed"]), int(g["rows"]), int(g["D"]))
    rows, D = x.shape
    xt = _bf(x)
    h = torch.empty_like(xt)
    layernorm(xt, torch.from_numpy(gamma).cuda(), torch.from_numpy(beta).cuda(), h)
    q, k, v = (torch.empty(rows, D, dtype=torch.bfloat16, device="cuda") for _ in range(3))
    qkv_project(h, _bf(w), torch.from_numpy(b).cuda(), q, k, v)
    r = g["sample_rows"]
    assert np.abs(_f(h)[r] - g["h"]).max() < 3e-2
    for t, name in ((q, "q"), (k, "k"), (v, "v")):
        got = _f(t)
        assert np.abs(got[r] - g[name]).max() < 3e-2, name
        assert np.abs(got.sum(0) - g[f"{name}_colsum"]).max() < 0.25, name


def _session_attention(policy, *, produce, mode, F, T, H, seed, set_aside):
    """Per frame (cross) or once (stack): plan, upload, then either the
    producer (rows of the step's own frames land in the arena) plus a gather
    of the rest, or the projection without a map plus the full gather; then
    attention through the session's map.  Returns the output (CPU)."""
    from kvp.attention import attn_bf16
    from kvp.producer import qkv_project
    from kvp.session import Session
    from kvp.traces import motion_config4
    D = H * 128
    rng = np.random.default_rng(seed)
    x = _bf(rng.standard_normal((F * T, D)))
    w = _bf(0.02 * rng.standard_normal((3 * D, D)))
    b = torch.from_numpy((0.1 * rng.standard_normal(3 * D)).astype(np.float32)).cuda()
    q, k, v = (torch.zeros(F * T, D, dtype=torch.bfloat16, device="cuda") for _ in range(3))
    out = torch.zeros_like(q)
    scores = motion_config4(frames=F, seed=seed, tiles=(T + 15) // 16)
    stream = int(torch.cuda.current_stream().cuda_stream)
    s = Session(mode=mode, policy=policy, frames=F, tokens=T, hidden=D, elem_bytes=2,
                set_aside=set_aside, layers=1)
    try:
        steps = [None] if mode == "stack" else list(range(F))
        for f in steps:
            st = s.plan_stack(scores) if f is None else s.plan_frame(f, scores)
            r0, n = (0, F * T) if f is None else (f * T, T)      # rows this step produces
            s.upload(stream)
            if produce:
                s.produce(0, x[r0:r0 + n], w, b, q[r0:r0 + n], k[r0:r0 + n], v[r0:r0 + n],
                          row0=r0, stream=stream)
                s.stage_except([k.data_ptr()], [v.data_ptr()], r0, n, stream)
            else:
                qkv_project(x[r0:r0 + n], w, b, q[r0:r0 + n], k[r0:r0 + n], v[r0:r0 + n])
                s.stage([k.data_ptr()], [v.data_ptr()], stream)
            s.window(0, stream)
            kw = dict(kvmap_ptr=s.device_map_ptr(), arena_ptr=s.arena_ptr(0),
                      arena_rows=s.cap_rows) if policy != "none" else {}
            if f is None:
                attn_bf16(q, k, v, out, tokens=T, frames=F, heads=H, mode="causal", flat=True,
                          stream=stream, **kw)
            else:
                attn_bf16(q, k, v, out, tokens=T, frames=1, q_frame0=f, heads=H, mode="causal",
                          stream=stream, **kw)
        s.clear_window(stream)
        torch.cuda.synchronize()
        s.finish()
    finally:
        s.close()
    return out.cpu(), st


@pytest.mark.parametrize("mode", ["stack", "cross"])
def test_session_produce_is_bitwise_equal_to_gather_and_none(cuda, mode):
    from kvp.attention import read_status
    F, T, H = 3, 300, 2
    D = H * 128
    set_aside = 30 * 16 * D * 2 * 2            # 30 of 57 tiles
    read_status()
    ref, _ = _session_attention("none", produce=False, mode=mode, F=F, T=T, H=H, seed=9,
                                set_aside=set_aside)
    for policy in ("recency", "reuse_weighted"):
        got, st = _session_attention(policy, produce=True, mode=mode, F=F, T=T, H=H, seed=9,
                                     set_aside=set_aside)
        assert st.copies > 0
        assert torch.equal(got, ref), (mode, policy)
        gat, _ = _session_attention(policy, produce=False, mode=mode, F=F, T=T, H=H, seed=9,
                                    set_aside=set_aside)
        assert torch.equal(gat, ref), (mode, policy, "gather")
    assert read_status() == 0


def test_session_produce_refuses_reuse_mode(cuda):
    from kvp.session import Session
    s = Session(mode="reuse", policy="recency", frames=2, tokens=256, hidden=256, elem_bytes=2,
                set_aside=1 << 20, layers=1, streaming=True)
    s.plan_frame(0, np.ones((2, 16), np.float32))
    s.upload(int(torch.cuda.current_stream().cuda_stream))
    x = torch.zeros(256, 256, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(768, 256, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="reuse"):
        s.produce(0, x, w, None, x, x, x, row0=0)
    torch.cuda.synchronize()
    s.close()
