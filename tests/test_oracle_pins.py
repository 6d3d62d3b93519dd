"""The oracle is pinned to the reference before it is trusted (CPU only).

* KVMap / admission: the C restatement (oracle/kvp_oracle.c) reproduces the
  per-frame KVMap digests and staged-byte counters that the reference's own
  driver produced (tests/golden/kvmap_ref.json, written by make_golden.py
  from src/run_policy_experiment.cu built host-only).
* Attention: the numpy restatement (oracle/attention.py) reproduces the
  reference golden functions' outputs (tests/golden/attn_golden.npz) and,
  on the reference's own seed-42 8-frame trace, the per-frame statistics the
  reference ships in traces/golden_meta.json.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
T = 1560


def digest(a):
    return hashlib.sha256(np.ascontiguousarray(a, dtype="<i8").tobytes()).hexdigest()[:16]


def _cases():
    return json.loads((GOLDEN / "kvmap_ref.json").read_text())["cases"]


CSV = {"ref8f": "motion_ref8f.csv", "config1": "motion_config1.csv",
       "config2": "motion_config2.csv", "config3": "motion_config3.csv",
       "config4": "motion_config4.csv", "config5_static": "motion_config5_static.csv",
       "config5_high": "motion_config5_high.csv"}


@pytest.mark.parametrize("case", _cases(), ids=lambda c: "{trace}-{policy}-{mode}-s{streaming}-{set_aside}".format(**c))
def test_oracle_kvmap_matches_reference(oracle, case):
    frames = case["frames"]
    scores = oracle.read_motion_csv(GOLDEN / CSV[case["trace"]], frames, 98)
    window = case.get("window", 0)
    res = oracle.run_trace(scores, policy=case["policy"], cross=case["mode"] == "cross",
                           streaming=case["streaming"], frames=frames,
                           set_aside=case["set_aside"], window=window)
    for f, want in enumerate(case["per_frame"]):
        r0, sl = res.uploaded_slice(f, T, case["mode"] == "cross", window)
        assert (r0, len(sl), int((sl >= 0).sum()), digest(sl)) == \
            (want["row0"], want["n"], want["mapped"], want["sha"]), f"frame {f}"
    if case["staged_bytes"] is not None:
        assert int(res.staged_bytes[-1]) == case["staged_bytes"]


def test_oracle_bf16_accounting_equals_fp32_at_half_budget(oracle):
    """Every byte gate scales with the element size: bf16 at budget B admits
    the rows fp32 admits at 2B (the fixtures are in fp32 accounting)."""
    scores = oracle.read_motion_csv(GOLDEN / "motion_config2.csv", 8, 98)
    for st in (0, 1):
        a = oracle.run_trace(scores, policy="recency", cross=True, streaming=st, frames=8,
                             set_aside=4325376, elem_bytes=4)
        b = oracle.run_trace(scores, policy="recency", cross=True, streaming=st, frames=8,
                             set_aside=2162688, elem_bytes=2)
        assert np.array_equal(a.maps, b.maps)
        assert np.array_equal(a.copy_slots, b.copy_slots)


def test_oracle_attention_matches_reference_golden():
    from oracle.attention import attention_frames
    g = np.load(GOLDEN / "attn_golden.npz")
    q, k, v = g["q"], g["k"], g["v"]
    F, Tq, D = q.shape
    for mode in ("intra", "cross"):
        got = attention_frames(q.reshape(-1, D), k.reshape(-1, D), v.reshape(-1, D), frames=F,
                               tokens=Tq, heads=D // 128, head_dim=128, mode=mode)
        assert np.abs(got.reshape(F, Tq, D) - g[mode]).max() < 2e-6, mode


def test_torch_restatement_matches_reference_golden():
    """oracle/golden_torch.py, the CPU baseline bench.py times, gives the
    reference golden's cross-frame outputs."""
    import torch
    from oracle import golden_torch
    g = np.load(GOLDEN / "attn_golden.npz")
    F, Tq, D = g["q"].shape
    q, k, v = (torch.from_numpy(np.ascontiguousarray(g[n].reshape(-1, D))) for n in "qkv")
    got = golden_torch.attention_frames(q, k, v, frames=F, tokens=Tq, heads=D // 128,
                                        head_dim=128).numpy()
    assert np.abs(got.reshape(F, Tq, D) - g["cross"]).max() < 2e-6
    assert golden_torch.set_threads(2) == 2


def test_reference_trace_and_golden_statistics():
    """Our restatement of the reference trace generator (kvp.traces) plus the
    attention oracle reproduce the reference's shipped 8-frame statistics."""
    import torch
    from kvp import traces
    from oracle.attention import attention_frames
    meta = json.loads((GOLDEN / "reference_meta.json").read_text())
    scores, is_static, q, k, v = traces.reference_synthetic_trace(frames=8, seed=42)
    assert int(is_static.sum()) == meta["tiles"]["static"]
    assert int((~is_static).sum()) == meta["tiles"]["moving"]
    # CSV text is byte-identical to the one the reference generator wrote
    written = traces.write_motion_csv(GOLDEN.parent / "_tmp_ref8f.csv", scores, is_static)
    try:
        assert written.read_text() == (GOLDEN / "motion_ref8f.csv").read_text()
    finally:
        written.unlink()
    tok_static = np.repeat(is_static, traces.tile_counts())
    kt = torch.from_numpy(k)
    cos = torch.nn.functional.cosine_similarity(kt[0], kt[-1], dim=1).numpy()
    want = meta["validation_cosine_first_vs_last"]["K"]
    assert round(float(cos[tok_static].mean()), 6) == want["static"]["mean"]
    assert round(float(cos[~tok_static].max()), 6) == want["moving"]["max"]
    out = attention_frames(q.reshape(-1, 1536), k.reshape(-1, 1536), v.reshape(-1, 1536),
                           frames=8, tokens=T, heads=12, head_dim=128, mode="intra")
    out = torch.from_numpy(out.reshape(8, T, 1536))
    for f, st in enumerate(meta["golden_per_frame_stats"]):
        assert round(float(out[f].mean()), 6) == st["mean"], f
        assert round(float(out[f].std()), 6) == st["std"], f


def test_qkv_oracle_matches_reference_block():
    """oracle/qkv.py (LayerNorm, qkv_proj, column split) against the
    reference's DiTSelfAttentionBlock run on the same seeded inputs
    (tests/golden/qkv_ref.npz, written by make_golden.py --only qkv)."""
    from oracle.qkv import layernorm, qkv_params, qkv_split
    g = np.load(GOLDEN / "qkv_ref.npz")
    x, gamma, beta, w, b = qkv_params(int(g["seed"]), int(g["rows"]), int(g["D"]))
    h = layernorm(x, gamma, beta)
    q, k, v = qkv_split(h, w, b)
    rows = g["sample_rows"]
    np.testing.assert_allclose(h[rows], g["h"], rtol=0, atol=1e-5)
    for name, got in (("q", q), ("k", k), ("v", v)):
        np.testing.assert_allclose(got[rows], g[name], rtol=0, atol=1e-5, err_msg=name)
        np.testing.assert_allclose(got.sum(0), g[f"{name}_colsum"], rtol=0, atol=1e-3, err_msg=name)
