"""Regenerates the committed golden fixtures from the reference's own code.

    python tests/golden/make_golden.py --ref <reference checkout> [--only reuse|qkv|motion|cxx]

(--ref defaults to $KVP_REF_ROOT.)

Needs the reference sources (read, never copied) and is run once, on a host
where they exist; the tests only read the files it writes:

* ``motion_*.csv``        motion traces: the reference's synthetic 8-frame
                          trace (seed 42, produced by importing the
                          reference's traces/gen_synthetic_motion.py) and the
                          benchmark config generators (kvp/traces.py).
* ``kvmap_ref.json``      per-frame SHA-256 (first 16 hex) of the KVMap slice
                          each kernel launch receives, plus the staged-byte
                          counters, from the reference's UNMODIFIED driver
                          main() (src/run_policy_experiment.cu) built
                          host-only as oracle/_ref/policy_experiment_ref;
                          window cases come from the reference's policy and
                          manager classes driven by oracle/ref_stub/ref_shims.cpp.
                          Every case is also checked against the C oracle
                          here before it is written.
* ``attn_golden.npz``     outputs of the reference's golden functions
                          (traces/gen_golden.py attention_reference /
                          attention_reference_cross) on small seeded inputs.
* ``reference_meta.json`` numbers the reference ships as text for the seed-42
                          8-frame trace (traces/trace_meta_8f.json tile counts
                          and cosines, traces/golden_meta.json per-frame stats).
* ``kvmap_reuse_ref.json`` the temporal-reuse streaming loop (slots keyed by
                          token position, changed = !reuse) run on the
                          reference's KVTileManager through the shims, with
                          ``motion_config2_reuse.csv`` (a trace carrying the
                          optional reuse column).  ``--only reuse`` rewrites
                          just these two files.
* ``qkv_ref.npz``         the reference's DiTSelfAttentionBlock (its
                          LayerNorm, qkv_proj and view/permute) on seeded
                          inputs (``oracle/qkv.py qkv_params``): sampled rows of h, Q, K, V
                          and per-column sums.  ``--only qkv``.
* ``motion_ref_clip.csv`` / ``.json`` the reference's own
                          traces/gen_motion_from_video.py (OpenCV Farneback)
                          run on a seeded synthetic clip: per-tile change
                          rates, is_static and reuse, tau.  ``--only motion``.
* ``cxx_layout_ref.json`` sizes, member offsets and enum values of the
                          reference's C++ classes as a caller compiled
                          against its headers sees them
                          (``cxx_layout_probe.cpp``).  ``--only cxx``.
"""

from __future__ import annotations

import argparse
import os
import hashlib
import importlib.util
import json
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "cuda-kv-persistence_b200"))

from oracle import oracle as orc  # noqa: E402

MAX_PERSIST_B200 = 82_903_040  # cudaDevAttrMaxPersistingL2CacheSize measured on the pool's B200s
T, D, TT = 1560, 1536, 16


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a, dtype="<i8").tobytes()).hexdigest()[:16]


def ref_case(csv, *, policy, mode, streaming, frames, set_aside, window=0, scores=None):
    """Run the reference (driver main, or the window shim) and return per-frame digests."""
    if window == 0:
        run = orc.run_ref_driver(csv, policy=policy, attn_mode=mode, streaming=streaming,
                                 frames=frames, set_aside=set_aside)
        out = []
        for f, row0, n, vals in run.launches:
            arr = np.full(n, -1, np.int64)
            for r, v in vals.items():
                arr[r - row0] = v
            out.append({"row0": row0, "n": n, "mapped": len(vals), "sha": digest(arr)})
        import re
        m = re.search(r"staged_bytes=(\d+)", run.stdout)
        return out, (int(m.group(1)) if m else None)
    lib = orc.RefLib()
    maps, staged = lib.run_window(scores, policy=policy, streaming=streaming, window=window,
                                  frames=frames, set_aside=set_aside)
    out = []
    for f in range(frames):
        base = max(0, f - window + 1)
        sl = maps[f, base * T:(f + 1) * T]
        out.append({"row0": base * T, "n": len(sl), "mapped": int((sl >= 0).sum()),
                    "sha": digest(sl)})
    return out, int(staged[-1]) if streaming else None


def oracle_case(scores, *, policy, mode, streaming, frames, set_aside, window=0):
    res = orc.Oracle().run_trace(scores, policy=policy, cross=(mode == "cross"),
                                 streaming=streaming, frames=frames, set_aside=set_aside,
                                 window=window)
    out = []
    for f in range(frames):
        r0, sl = res.uploaded_slice(f, T, mode == "cross", window)
        out.append({"row0": r0, "n": len(sl), "mapped": int((sl >= 0).sum()), "sha": digest(sl)})
    return out, int(res.staged_bytes[-1]) if streaming else None


def reuse_fixtures():
    """kvmap_reuse_ref.json: the temporal-reuse streaming loop run on the
    reference's own KVTileManager (oracle/ref_stub/ref_shims.cpp
    kvpref_run_reuse), per frame: KVMap digest, copies, re-copies into held
    slots, sticky hits, cumulative staged bytes, window bytes.  The oracle's
    restatement must agree before anything is written."""
    from kvp import traces
    R, O = orc.RefLib(), orc.Oracle()
    sc2 = traces.motion_config2()
    traces.write_motion_csv(HERE / "motion_config2_reuse.csv", sc2, reuse=traces.reuse_flags(sc2))
    sources = {"config2_reuse": (HERE / "motion_config2_reuse.csv", 8, "csv"),
               "config5_high": (HERE / "motion_config5_high.csv", 16, "derived"),
               "config3": (HERE / "motion_config3.csv", 50, "derived")}
    cases = []
    for pol in ("uniform", "recency", "motion", "reuse_weighted"):
        for sa in (2162688, 4325376, 8650752):
            for flags in ("csv", "none"):
                cases.append(dict(trace="config2_reuse", policy=pol, set_aside=sa, flags=flags))
        for pct in (10, 25, 50, 100):
            cases.append(dict(trace="config5_high", policy=pol,
                              set_aside=2 * MAX_PERSIST_B200 * pct // 100, flags="derived"))
    for pol in ("recency", "reuse_weighted"):
        cases.append(dict(trace="config3", policy=pol, set_aside=2 * MAX_PERSIST_B200,
                          flags="derived"))
    fixtures = []
    for c in cases:
        csv, frames, _ = sources[c["trace"]]
        scores, col = O.read_motion_csv(csv, frames, 98, with_reuse=True)
        reuse = {"csv": col, "derived": traces.reuse_flags(scores), "none": None}[c["flags"]]
        got = R.run_reuse(scores, reuse, policy=c["policy"], frames=frames,
                          set_aside=c["set_aside"])
        mine = O.run_reuse(scores, reuse, policy=c["policy"], frames=frames,
                           set_aside=c["set_aside"])
        for key in ("copies", "restaged", "hits", "staged_bytes", "window_bytes", "maps"):
            assert np.array_equal(got[key], mine[key]), (c, key)
        per = [{"sha": digest(got["maps"][f]), "mapped": int((got["maps"][f] >= 0).sum()),
                "copies": int(got["copies"][f]), "restaged": int(got["restaged"][f]),
                "hits": int(got["hits"][f]), "staged_bytes": int(got["staged_bytes"][f]),
                "window_bytes": int(got["window_bytes"][f])} for f in range(frames)]
        fixtures.append({**c, "frames": frames, "elem_bytes": 4, "per_frame": per})
        print("ok", c, flush=True)
    (HERE / "kvmap_reuse_ref.json").write_text(json.dumps(
        {"generator": "tests/golden/make_golden.py --only reuse", "tokens": T, "hidden": D,
         "tile_tokens": TT, "reuse_rule": "traces/gen_motion_from_video.py:118-122, percentile 50",
         "cases": fixtures}, indent=1))


QKV_SEED, QKV_ROWS, QKV_D = 31, 160, 256
QKV_SAMPLE_ROWS = [0, 1, 57, 127, 128, 159]


def qkv_fixture(ref: Path):
    """qkv_ref.npz: the reference's own DiTSelfAttentionBlock
    (src/backbone.py:8-33), loaded with oracle.qkv.qkv_params(), run on one frame: its
    LayerNorm output and the Q (qkv_proj(norm(x)) split by the module's own
    view/permute) and the K, V its forward returns, for QKV_SAMPLE_ROWS
    (full rows) plus every column's sum over all rows."""
    import torch
    sys.path.insert(0, str(ref))
    from src.backbone import DiTSelfAttentionBlock
    from src.config import BackboneConfig
    cfg = BackboneConfig(num_layers=1, hidden_dim=QKV_D, num_heads=QKV_D // 128, head_dim=128,
                         tokens_per_frame=QKV_ROWS, latent_grid_rows=10, latent_grid_cols=16)
    blk = DiTSelfAttentionBlock(cfg).eval()
    from oracle.qkv import qkv_params
    x, gamma, beta, w, b = qkv_params(QKV_SEED, QKV_ROWS, QKV_D)
    with torch.no_grad():
        blk.norm.weight.copy_(torch.from_numpy(gamma))
        blk.norm.bias.copy_(torch.from_numpy(beta))
        blk.attn.qkv_proj.weight.copy_(torch.from_numpy(w))
        blk.attn.qkv_proj.bias.copy_(torch.from_numpy(b))
        xt = torch.from_numpy(x)[None]
        h = blk.norm(xt)
        _, k, v = blk(xt)                                   # [1, heads, t, hd]
        qkv = blk.attn.qkv_proj(h).view(1, QKV_ROWS, 3, cfg.num_heads, cfg.head_dim)
        q = qkv.permute(2, 0, 3, 1, 4).unbind(0)[0]
    flat = lambda t: t[0].permute(1, 0, 2).reshape(QKV_ROWS, QKV_D).numpy()   # [t, heads*hd]
    q, k, v, h = flat(q), flat(k), flat(v), h[0].numpy()
    rows = np.array(QKV_SAMPLE_ROWS)
    np.savez_compressed(HERE / "qkv_ref.npz", seed=QKV_SEED, rows=QKV_ROWS, D=QKV_D,
                        sample_rows=rows, h=h[rows], q=q[rows], k=k[rows], v=v[rows],
                        q_colsum=q.sum(0), k_colsum=k.sum(0), v_colsum=v.sum(0))


MOTION_SEED, MOTION_FRAMES = 5, 6


def motion_fixture(ref: Path):
    """motion_ref_clip.csv + motion_ref_clip.json: the reference's own
    traces/gen_motion_from_video.py (OpenCV Farneback + its aggregation) run
    on the seeded synthetic clip kvp.traces.synthetic_video(MOTION_FRAMES,
    seed=MOTION_SEED), written as PNG frames.  The script writes a heatmap
    beside itself, so it runs from a temporary copy (with src/config.py)
    under /tmp; nothing is written into the reference tree."""
    import shutil
    import subprocess
    import cv2
    from kvp.traces import synthetic_video
    work = Path(tempfile.mkdtemp(prefix="kvp_motion_"))
    try:
        clip = work / "clip"
        clip.mkdir()
        for i, fr in enumerate(synthetic_video(MOTION_FRAMES, seed=MOTION_SEED)):
            cv2.imwrite(str(clip / f"{i:05d}.png"), fr)
        (work / "ref" / "traces").mkdir(parents=True)
        (work / "ref" / "src").mkdir(parents=True)
        shutil.copy(ref / "traces" / "gen_motion_from_video.py", work / "ref" / "traces")
        shutil.copy(ref / "src" / "config.py", work / "ref" / "src")
        (work / "ref" / "src" / "__init__.py").write_text("")
        out = work / "out"
        out.mkdir()
        subprocess.run([sys.executable, str(work / "ref" / "traces" / "gen_motion_from_video.py"),
                        "--source", str(clip), "--frames", str(MOTION_FRAMES), "--out-dir", str(out),
                        "--config", str(ref / "configs" / "grounding_config.json")],
                       check=True, cwd=str(work))
        shutil.copy(out / "motion_trace_real.csv", HERE / "motion_ref_clip.csv")
        meta = json.loads((out / "trace_real_meta.json").read_text())
        (HERE / "motion_ref_clip.json").write_text(json.dumps(
            {"generator": "tests/golden/make_golden.py --only motion",
             "clip": f"kvp.traces.synthetic_video({MOTION_FRAMES}, seed={MOTION_SEED})",
             "opencv": cv2.__version__, "farneback": meta["farneback"],
             "tau_reuse": meta["tau_reuse"], "reuse_fraction": meta["reuse_fraction_achieved"],
             "frames": meta["frames"], "num_tiles": meta["num_tiles"]}, indent=1))
    finally:
        shutil.rmtree(work, ignore_errors=True)


def cxx_layout_fixture(ref: Path):
    """cxx_layout_ref.json: the object layout (sizes, member offsets, enum
    values) that a caller compiled against the reference's own C++ headers
    (src/kv_tile_manager.h, src/tile_gating_policy.h) allocates.
    tests/test_cxx_boundary.py compiles the same probe against include/cxx/
    and requires the same numbers."""
    with tempfile.TemporaryDirectory() as td:
        exe = Path(td) / "probe"
        subprocess.run(["g++", "-std=c++17", "-I", str(ref / "src"), str(HERE / "cxx_layout_probe.cpp"),
                        "-o", str(exe)], check=True)
        out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    layout = json.loads(out)
    layout["generator"] = "tests/golden/make_golden.py --only cxx (probe built against the reference's src/*.h)"
    (HERE / "cxx_layout_ref.json").write_text(json.dumps(layout, indent=1) + "\n")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("KVP_REF_ROOT"),
                    help="root of a GauthamMK-0/cuda-kv-persistence checkout (default: $KVP_REF_ROOT)")
    ap.add_argument("--only", choices=("reuse", "qkv", "motion", "cxx"), default=None,
                    help="regenerate one fixture set only")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give --ref or set KVP_REF_ROOT to the reference checkout")
    ref = Path(args.ref)
    orc.build(str(ref))
    if args.only == "reuse":
        reuse_fixtures()
        return
    if args.only == "qkv":
        qkv_fixture(ref)
        return
    if args.only == "motion":
        motion_fixture(ref)
        return
    if args.only == "cxx":
        cxx_layout_fixture(ref)
        return
    from kvp import traces

    # ---- motion traces -------------------------------------------------
    spec = importlib.util.spec_from_file_location("ref_gen", ref / "traces" / "gen_synthetic_motion.py")
    sys.path.insert(0, str(ref))
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    import torch
    from src.config import BackboneConfig  # the reference's config class (imported, not copied)
    cfg = BackboneConfig.from_grounding(str(ref / "configs" / "grounding_config.json"))
    g = torch.Generator().manual_seed(42)
    starts, counts = gen.build_tiles(cfg)
    scores8, static8 = gen.generate_motion_scores(g, int(counts.numel()), 8, 0.65)
    traces.write_motion_csv(HERE / "motion_ref8f.csv", scores8.numpy(), static8.numpy())
    csvs = {
        "ref8f": (HERE / "motion_ref8f.csv", 8),
        "config1": (traces.write_motion_csv(HERE / "motion_config1.csv", traces.motion_config1()), 1),
        "config2": (traces.write_motion_csv(HERE / "motion_config2.csv", traces.motion_config2()), 8),
        "config3": (traces.write_motion_csv(HERE / "motion_config3.csv", traces.motion_config3()), 50),
        "config4": (traces.write_motion_csv(HERE / "motion_config4.csv", traces.motion_config4()), 21),
        "config5_static": (traces.write_motion_csv(HERE / "motion_config5_static.csv",
                                                   traces.motion_config5("static")), 16),
        "config5_high": (traces.write_motion_csv(HERE / "motion_config5_high.csv",
                                                 traces.motion_config5("high")), 16),
    }

    # ---- KVMap digests from the reference ------------------------------
    cases = []
    for pol in ("uniform", "recency", "motion", "reuse_weighted"):
        for mode in ("intra", "cross"):
            for st in (0, 1):
                for sa in (2162688, 4325376):
                    cases.append(dict(trace="ref8f", policy=pol, mode=mode, streaming=st,
                                      set_aside=sa))
    for st in (0, 1):
        cases.append(dict(trace="config1", policy="motion", mode="intra", streaming=st,
                          set_aside=4325376))
        cases.append(dict(trace="config2", policy="recency", mode="cross", streaming=st,
                          set_aside=4325376))
        cases.append(dict(trace="config3", policy="reuse_weighted", mode="cross", streaming=st,
                          set_aside=2 * MAX_PERSIST_B200, window=5))
    cases.append(dict(trace="config4", policy="reuse_weighted", mode="cross", streaming=0,
                      set_aside=2 * MAX_PERSIST_B200))
    # Uniform with more slots than frame 0's candidates makes the reference
    # write past its selection vector (src/run_policy_experiment.cu:170-172;
    # the host build aborts): those config-5 cells have no reference answer.
    for regime in ("static", "high"):
        for pol in ("recency", "motion", "reuse_weighted"):
            for pct in (10, 25, 50, 100):
                cases.append(dict(trace=f"config5_{regime}", policy=pol, mode="cross",
                                  streaming=0, set_aside=2 * MAX_PERSIST_B200 * pct // 100))
    fixtures = []
    O = orc.Oracle()
    for c in cases:
        csv, frames = csvs[c["trace"]]
        scores = O.read_motion_csv(csv, frames, 98)
        kw = dict(policy=c["policy"], mode=c["mode"], streaming=c["streaming"], frames=frames,
                  set_aside=c["set_aside"], window=c.get("window", 0))
        got, staged = ref_case(csv, scores=scores, **kw)
        mine, mstaged = oracle_case(scores, **kw)
        assert got == mine, f"oracle disagrees with the reference on {c}"
        assert staged is None or staged == mstaged, (c, staged, mstaged)
        fixtures.append({**c, "frames": frames, "elem_bytes": 4, "per_frame": got,
                         "staged_bytes": staged})
        print("ok", c, flush=True)
    (HERE / "kvmap_ref.json").write_text(json.dumps(
        {"generator": "tests/golden/make_golden.py", "tokens": T, "hidden": D, "tile_tokens": TT,
         "note": "set_aside is in the reference's fp32 accounting; a bf16 run with budget "
                 "set_aside/2 admits the same rows", "cases": fixtures}, indent=1))

    # ---- golden attention vectors --------------------------------------
    spec2 = importlib.util.spec_from_file_location("ref_golden", ref / "traces" / "gen_golden.py")
    gg = importlib.util.module_from_spec(spec2)
    spec2.loader.exec_module(gg)
    rng = np.random.default_rng(2024)
    F2, T2, H2, dh = 3, 48, 2, 128
    q, k, v = (rng.standard_normal((F2, T2, H2 * dh)).astype(np.float32) / np.sqrt(dh)
               for _ in range(3))
    intra = np.stack([gg.attention_reference(torch.from_numpy(q[f]), torch.from_numpy(k[f]),
                                             torch.from_numpy(v[f]), H2, dh)[0].numpy()
                      for f in range(F2)])
    cross = np.stack([gg.attention_reference_cross(
        torch.from_numpy(q[f]), [torch.from_numpy(k[i]) for i in range(f + 1)],
        [torch.from_numpy(v[i]) for i in range(f + 1)], H2, dh)[0].numpy() for f in range(F2)])
    np.savez_compressed(HERE / "attn_golden.npz", q=q, k=k, v=v, intra=intra, cross=cross)

    # ---- the reference's shipped trace / golden statistics -------------
    tm = json.loads((ref / "traces" / "trace_meta_8f.json").read_text())
    gm = json.loads((ref / "traces" / "golden_meta.json").read_text())
    (HERE / "reference_meta.json").write_text(json.dumps({
        "source": "traces/trace_meta_8f.json and traces/golden_meta.json of the reference",
        "seed": tm["seed"], "frames": tm["frames"], "tiles": tm["tiles"],
        "validation_cosine_first_vs_last": tm["validation_cosine_first_vs_last"],
        "golden_per_frame_stats": gm["per_frame_stats"]}, indent=1))
    reuse_fixtures()
    qkv_fixture(ref)
    motion_fixture(ref)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
