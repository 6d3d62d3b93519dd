"""GPU parity of the remapped attention kernels, through the C ABI.

Every case compares the CUDA output with the CPU oracle (oracle/attention.py,
a restatement of the reference golden traces/gen_golden.py) and checks the
reference's gate that outputs are bitwise identical whatever the policy /
KVMap (tests/test_policy_variants.py:174-176 of the reference).

Tolerances: FP32 path max-abs < 1e-3 and mean-abs < 1e-4
(tests/test_correctness.py:26-27); BF16 tcgen05 path max-abs < 2e-2 against
the fp32 oracle on the same bf16-rounded inputs (the bf16 path's stated
tolerance).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import bf16_round, build_arena, errors, rand_qkv
from oracle.attention import attention_frames, attention_intra

pytestmark = pytest.mark.gpu

FP32_MAX, FP32_MEAN = 1e-3, 1e-4
BF16_MAX = 2e-2
# The output scale shrinks like 1/sqrt(keys), so a max-abs bound alone cannot
# tell a wrong (e.g. all-zero) result from a right one at long spans: every
# bf16 case also bounds the error relative to the oracle's L2 norm.
BF16_REL_L2 = 1e-2


def rel_l2(got, want):
    return float(np.linalg.norm((got - want).ravel()) / max(np.linalg.norm(want.ravel()), 1e-30))


@pytest.fixture(params=["pair", "one_sm"])
def kernel(request, monkeypatch):
    """Both bf16 kernels: the one-SM kernel (attn_sm100.cu, the default) and
    the SM-pair kernel (attn_pair_sm100.cu, KVP_ATTN_PAIR=1)."""
    monkeypatch.setenv("KVP_ATTN_PAIR", "1" if request.param == "pair" else "0")
    return request.param


def check_bf16(got, want, what=""):
    mx, _ = errors(got, want)
    rl = rel_l2(got, want)
    assert mx < BF16_MAX and rl < BF16_REL_L2, (what, mx, rl)


def _dev(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    return t if dtype is None else t.to(dtype)


def _session_map(mode, policy, frames, T, hidden, elem, set_aside, streaming, seed, window=0,
                 upto=None):
    """KVMap + copies from the product planner for the last planned frame."""
    from kvp import traces
    from kvp.session import Session
    rng = np.random.default_rng(seed)
    scores = rng.random((frames, (T + 15) // 16)).astype(np.float32)
    s = Session(mode=mode, policy=policy, frames=frames, tokens=T, hidden=hidden,
                elem_bytes=elem, set_aside=set_aside, streaming=streaming, window=window)
    last = frames - 1 if upto is None else upto
    for f in range(last + 1):
        s.plan_frame(f, scores)
    return s.host_map(), s.cap_rows


def _scattered_map(kv_rows, arena_rows, seed, frac=0.4):
    rng = np.random.default_rng(seed)
    m = np.full(kv_rows, -1, dtype=np.int64)
    rows = rng.choice(kv_rows, size=min(int(frac * kv_rows), arena_rows), replace=False)
    m[rows] = rng.permutation(arena_rows)[: len(rows)]
    return m


# --------------------------------------------------------------------- FP32
def test_fp32_config1_intra_motion(cuda):
    """Config 1: 1560 tokens, 12 heads, MotionGated 22 tiles, fp32."""
    from kvp import traces
    from kvp.attention import attn_forward_single_frame
    from kvp.session import Session
    import kvp
    T, D, H = 1560, 1536, 12
    q, k, v = rand_qkv(T, D, seed=0)
    scores = traces.motion_config1(seed=0)
    s = Session(mode="intra", policy="motion", frames=1, tokens=T, hidden=D, elem_bytes=4,
                set_aside=4325376)
    info = s.plan_frame(0, scores)
    assert info.staged_tiles == 22 and info.copies == 22 * 16
    kvmap = s.host_map()
    pairs = s.copies()
    arena = torch.zeros(s.cap_rows, 2 * D, dtype=torch.float32, device=cuda)
    qd, kd, vd = _dev(q), _dev(k), _dev(v)
    dpairs = _dev(pairs.reshape(-1).astype(np.int32))
    assert kvp.lib().kvp_stage_rows(kd.data_ptr(), vd.data_ptr(), arena.data_ptr(),
                                    dpairs.data_ptr(), len(pairs), D * 4, 0) == 0
    torch.cuda.synchronize()
    assert np.array_equal(arena.cpu().numpy(), build_arena(k, v, kvmap, s.cap_rows))
    out = torch.empty_like(qd)
    out_none = torch.empty_like(qd)
    dmap = _dev(kvmap)
    attn_forward_single_frame(qd, kd, vd, arena, dmap, out, T, D, H, 0, 0)
    attn_forward_single_frame(qd, kd, vd, None, None, out_none, T, D, H, 0, 0)
    torch.cuda.synchronize()
    got, got_none = out.cpu().numpy(), out_none.cpu().numpy()
    assert np.array_equal(got, got_none), "remapped output differs from the None policy"
    mx, mn = errors(got, attention_intra(q, k, v, H, 128))
    assert mx < FP32_MAX and mn < FP32_MEAN, (mx, mn)


def test_fp32_cross_and_launchers(cuda):
    from kvp.attention import attn_forward_launcher, attn_forward_single_frame
    F, T, H = 3, 300, 2
    D = H * 128
    q, k, v = rand_qkv(F * T, D, seed=1)
    kvmap, cap = _session_map("cross", "recency", F, T, D, 4, 2 * 11 * 16 * D * 4, False, seed=2)
    arena = build_arena(k, v, kvmap, cap)
    qd, kd, vd, ad, md = _dev(q), _dev(k), _dev(v), _dev(arena), _dev(kvmap)
    want = attention_frames(q, k, v, frames=F, tokens=T, heads=H, head_dim=128, mode="cross")
    outs = []
    for use_map in (True, False):
        out = torch.zeros_like(qd)
        f = F - 1
        attn_forward_single_frame(qd[f * T:], kd, vd, ad if use_map else None,
                                  md if use_map else None, out[f * T:], T, D, H, 1, f)
        torch.cuda.synchronize()
        outs.append(out[f * T:].cpu().numpy())
        mx, mn = errors(outs[-1], want[f * T:])
        assert mx < FP32_MAX and mn < FP32_MEAN, (use_map, mx, mn)
    assert np.array_equal(outs[0], outs[1])
    # baseline launcher: every frame attends to itself, no map
    out = torch.zeros_like(qd)
    attn_forward_launcher(qd, kd, vd, None, None, out, F, T, D, H, False)
    torch.cuda.synchronize()
    want_i = attention_frames(q, k, v, frames=F, tokens=T, heads=H, head_dim=128, mode="intra")
    mx, mn = errors(out.cpu().numpy(), want_i)
    assert mx < FP32_MAX and mn < FP32_MEAN


def test_fp32_map_out_of_range_reports_status(cuda):
    from kvp.attention import attn_fp32, read_status
    T, H = 200, 1
    D = 128
    q, k, v = rand_qkv(T, D, seed=3)
    kvmap = np.full(T, -1, np.int64)
    kvmap[5] = 10_000  # outside an arena of 8 rows
    arena = np.zeros((8, 2 * D), np.float32)
    qd, kd, vd = _dev(q), _dev(k), _dev(v)
    read_status()
    out = torch.empty_like(qd)
    attn_fp32(qd, kd, vd, out, T=T, heads=H, k_lo=0, k_hi=T, arena=_dev(arena),
              kvmap=_dev(kvmap), arena_rows=8)
    assert read_status() & 1
    ref = torch.empty_like(qd)
    attn_fp32(qd, kd, vd, ref, T=T, heads=H, k_lo=0, k_hi=T)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert read_status() == 0


# --------------------------------------------------------------------- BF16
def _bf16_case(F, T, H, seed):
    D = H * 128
    q, k, v = (bf16_round(x) for x in rand_qkv(F * T, D, seed=seed))
    return D, q, k, v


def _run_bf16(q, k, v, kvmap, arena, **kw):
    from kvp.attention import attn_bf16
    qd = _dev(q, torch.bfloat16)
    kd = _dev(k, torch.bfloat16)
    vd = _dev(v, torch.bfloat16)
    out = torch.zeros_like(qd)
    ad = None if arena is None else _dev(arena, torch.bfloat16)
    md = None if kvmap is None else _dev(kvmap)
    from kvp.attention import read_status
    attn_bf16(qd, kd, vd, out, arena=ad, kvmap=md,
              arena_rows=0 if arena is None else arena.shape[0], **kw)
    torch.cuda.synchronize()
    assert read_status() == 0, "kernel reported a device status (timeout or bad map entry)"
    return out.float().cpu().numpy()


@pytest.mark.parametrize("T", [300, 1560])
def test_bf16_causal_policies_bitwise(cuda, kernel, T):
    """Causal cross-frame, per-frame launches: none / dense / streaming /
    scattered maps give bitwise-identical outputs within tolerance of the oracle."""
    from kvp.attention import read_status
    F, H = 3, 2
    D, q, k, v = _bf16_case(F, T, H, seed=4)
    want = attention_frames(q, k, v, frames=F, tokens=T, heads=H, head_dim=128, mode="cross")
    budget = 2 * 22 * 16 * D * 2
    maps = {"none": None}
    maps["dense"], cap_d = _session_map("cross", "recency", F, T, D, 2, budget, False, seed=5)
    maps["streaming"], cap_s = _session_map("cross", "motion", F, T, D, 2, budget, True, seed=6)
    maps["scattered"] = _scattered_map(F * T, 700, seed=7)
    caps = {"dense": cap_d, "streaming": cap_s, "scattered": 700}
    read_status()
    results = {}
    for name, m in maps.items():
        arena = None if m is None else build_arena(k, v, m, caps[name])
        results[name] = _run_bf16(q, k, v, m, arena, tokens=T, frames=F, heads=H, mode="causal")
        check_bf16(results[name], want, name)
    for name in maps:
        assert np.array_equal(results[name], results["none"]), name


def _tile_slot_map(F, T, n_tiles, order, seed):
    """KVMap of whole 16-row admission tiles whose rows sit on arena slots in
    the given order: "desc" puts each tile on descending slots (what LIFO slot
    reuse in streaming mode produces), "perm" scatters every row over the
    arena at random."""
    rng = np.random.default_rng(seed)
    tpf = (T + 15) // 16
    m = np.full(F * T, -1, dtype=np.int64)
    rows, nxt = [], 0
    for gid in rng.choice(F * tpf, size=n_tiles, replace=False):
        f, i = divmod(int(gid), tpf)
        cnt = min(16, T - 16 * i)
        r = np.arange(f * T + 16 * i, f * T + 16 * i + cnt)
        rows.append(r)
        if order == "desc":
            m[r] = nxt + cnt - 1 - np.arange(cnt)
        nxt += cnt
    if order == "perm":
        allr = np.concatenate(rows)
        m[allr] = rng.permutation(len(allr))
    return m, nxt


@pytest.mark.parametrize("T", [300, 1560])
@pytest.mark.parametrize("flat", [False, True])
def test_bf16_tile_slots_in_any_order_bitwise(cuda, kernel, T, flat):
    """Admitted tiles on descending or scattered arena slots: 8-row key
    groups wholly in the arena are fetched by TMA gather (four rows per
    instruction), groups that mix base and arena rows (frames of 300 tokens
    start off the 8-row grid) by cp.async.  Outputs bitwise equal to None and
    within tolerance of the oracle."""
    from kvp.attention import read_status
    F, H = 3, 2
    D, q, k, v = _bf16_case(F, T, H, seed=21)
    want = attention_frames(q, k, v, frames=F, tokens=T, heads=H, head_dim=128, mode="cross")
    kw = dict(tokens=T, frames=F, heads=H, mode="causal", flat=flat)
    read_status()
    none = _run_bf16(q, k, v, None, None, **kw)
    check_bf16(none, want, "none")
    n_tiles = F * ((T + 15) // 16) // 2
    for order in ("desc", "perm"):
        m, cap = _tile_slot_map(F, T, n_tiles, order, seed=22)
        got = _run_bf16(q, k, v, m, build_arena(k, v, m, cap), **kw)
        assert np.array_equal(got, none), order


def test_bf16_flat_stack_matches_per_frame(cuda, kernel):
    """Flat query tiling across frame edges (the stack layout) vs the oracle."""
    F, T, H = 4, 300, 2
    D, q, k, v = _bf16_case(F, T, H, seed=8)
    want = attention_frames(q, k, v, frames=F, tokens=T, heads=H, head_dim=128, mode="cross")
    m, cap = _session_map("cross", "reuse_weighted", F, T, D, 2, 2 * 30 * 16 * D * 2, False, seed=9)
    arena = build_arena(k, v, m, cap)
    a = _run_bf16(q, k, v, m, arena, tokens=T, frames=F, heads=H, mode="causal", flat=True)
    b = _run_bf16(q, k, v, None, None, tokens=T, frames=F, heads=H, mode="causal", flat=True)
    assert np.array_equal(a, b)
    check_bf16(a, want, "flat")


@pytest.mark.parametrize("T,mode,window", [(300, "intra", 0), (40, "intra", 0), (40, "causal", 0),
                                           (300, "causal", 2), (130, "causal", 1)])
def test_bf16_modes_and_ragged(cuda, kernel, T, mode, window):
    F, H = 3, 1
    D, q, k, v = _bf16_case(F, T, H, seed=10 + T)
    want = attention_frames(q, k, v, frames=F, tokens=T, heads=H, head_dim=128,
                            mode="intra" if mode == "intra" else "cross", window=window)
    m = _scattered_map(F * T, 64, seed=11)
    arena = build_arena(k, v, m, 64)
    a = _run_bf16(q, k, v, m, arena, tokens=T, frames=F, heads=H, mode=mode, window=window)
    b = _run_bf16(q, k, v, None, None, tokens=T, frames=F, heads=H, mode=mode, window=window)
    assert np.array_equal(a, b)
    check_bf16(a, want, (T, mode, window))


def test_bf16_head_subset_and_frame_offset(cuda, kernel):
    F, T, H = 3, 300, 3
    D, q, k, v = _bf16_case(F, T, H, seed=12)
    want = attention_frames(q, k, v, frames=F, tokens=T, heads=H, head_dim=128, mode="cross")
    got = _run_bf16(q, k, v, None, None, tokens=T, frames=1, q_frame0=2, heads=H, head0=1,
                    nheads=2, mode="causal")
    sl = slice(2 * T, 3 * T)
    check_bf16(got[sl, 128:], want[sl, 128:], "subset")
    assert np.all(got[sl, :128] == 0) and np.all(got[: 2 * T] == 0)


@pytest.mark.parametrize("splits", ["1", "3", "7"])
def test_bf16_key_split_matches_oracle(cuda, kernel, monkeypatch, splits):
    """Per-frame launches with the key range split over several CTAs (forced
    through KVP_ATTN_SPLITS; 7 leaves some chunks of the short frames empty):
    same results as the oracle, and policies stay bitwise identical."""
    monkeypatch.setenv("KVP_ATTN_SPLITS", splits)
    F, T, H = 4, 300, 2
    D, q, k, v = _bf16_case(F, T, H, seed=21)
    want = attention_frames(q, k, v, frames=F, tokens=T, heads=H, head_dim=128, mode="cross")
    m = _scattered_map(F * T, 200, seed=22)
    arena = build_arena(k, v, m, 200)
    a = _run_bf16(q, k, v, m, arena, tokens=T, frames=F, heads=H, mode="causal")
    b = _run_bf16(q, k, v, None, None, tokens=T, frames=F, heads=H, mode="causal")
    assert np.array_equal(a, b)
    check_bf16(a, want, ("split", splits))


@pytest.mark.parametrize("mode,flat", [("causal", False), ("causal", True), ("intra", False)])
def test_bf16_peaked_scores_exercise_rescale(cuda, kernel, mode, flat):
    """Scores with a wide, growing range: unit-scale Q, and K rows whose size
    ramps up along the key index, so a row's maximum keeps rising from tile
    to tile by more than the lazy-rescale threshold (8 in log2 units).  The
    softmax then takes its recompute-and-rescale path on most steps; results
    must still match the oracle within the bf16 gates, mapped or not."""
    F, T, H = 3, 300, 2
    D = H * 128
    rng = np.random.default_rng(31)
    q = bf16_round(rng.standard_normal((F * T, D)).astype(np.float32))
    # about 3/4 of the rows see their max rise by > 8 (log2) from the first
    # key tile to the second, 1/5 again from the second to the third
    ramp = (0.1 + 8.0 * (np.arange(F * T) % T) / T).astype(np.float32)[:, None]
    k = bf16_round((rng.standard_normal((F * T, D)) * ramp).astype(np.float32))
    v = bf16_round(rng.standard_normal((F * T, D)).astype(np.float32))
    want = attention_frames(q, k, v, frames=F, tokens=T, heads=H, head_dim=128,
                            mode="intra" if mode == "intra" else "cross")
    m = _scattered_map(F * T, 250, seed=32)
    arena = build_arena(k, v, m, 250)
    a = _run_bf16(q, k, v, m, arena, tokens=T, frames=F, heads=H, mode=mode, flat=flat)
    b = _run_bf16(q, k, v, None, None, tokens=T, frames=F, heads=H, mode=mode, flat=flat)
    assert np.array_equal(a, b)
    check_bf16(a, want, ("peaked", mode, flat))


@pytest.mark.parametrize("flat", [True, False])
def test_bf16_multi_layer_launch_matches_single_launches(cuda, monkeypatch, flat):
    """kvp_attn_bf16_multi over chunks of 1 to 3 heads (14 chunks: two
    launches of at most 12), some with a KVMap into their own arena: every
    chunk's output is bitwise the output of its own kvp_attn_bf16 call (key
    split off, which the multi-chunk launch never uses) and within the bf16
    gates of the oracle."""
    from kvp.attention import attn_bf16, attn_bf16_multi, read_status
    monkeypatch.setenv("KVP_ATTN_SPLITS", "1")
    F, T = 3, 300
    mode = "causal"
    chunks = []
    for i in range(14):
        h = 1 + i % 3
        D, q, k, v = _bf16_case(F, T, h, seed=40 + i)
        c = dict(q=_dev(q, torch.bfloat16), k=_dev(k, torch.bfloat16), v=_dev(v, torch.bfloat16),
                 heads=h, np=(q, k, v))
        if i % 2:
            m = _scattered_map(F * T, 128, seed=60 + i)
            c.update(kvmap=_dev(m), arena=_dev(build_arena(k, v, m, 128), torch.bfloat16),
                     arena_rows=128)
        chunks.append(c)
    read_status()
    for c in chunks:
        c["out"] = torch.zeros_like(c["q"])
    attn_bf16_multi([{kk: vv for kk, vv in c.items() if kk != "np"} for c in chunks], tokens=T,
                    frames=F, mode=mode, flat=flat)
    torch.cuda.synchronize()
    assert read_status() == 0
    for i, c in enumerate(chunks):
        ref = torch.zeros_like(c["q"])
        attn_bf16(c["q"], c["k"], c["v"], ref, tokens=T, frames=F, heads=c["heads"], mode=mode,
                  flat=flat, kvmap=c.get("kvmap"), arena=c.get("arena"),
                  arena_rows=c.get("arena_rows", 0))
        torch.cuda.synchronize()
        assert torch.equal(c["out"], ref), i
        q, k, v = c["np"]
        want = attention_frames(q, k, v, frames=F, tokens=T, heads=c["heads"], head_dim=128,
                                mode="cross")
        check_bf16(c["out"].float().cpu().numpy(), want, ("multi", i))
    assert read_status() == 0
