"""bench.py's per-frame measurements (`--matrix N`): benchmark config 5
(policy x budget x motion regime), config 2 (8-frame cross, Recency),
config 3 (50-frame trace, 30 layers, 5-frame causal window,
ReuseWeighted) and the extension legs (temporal reuse, QKV producer,
motion producer, against torch SDPA, arena slot orders).

Measurement code, not part of the library: one cell is the reference
driver's per-frame loop (src/run_policy_experiment.cu:156-274) as the
library runs it (kvp.frames.run_frames), timed with CUDA events.

`cell_order` fixes the order of the cells (regime, budget, policy) and the
repetition order: forward, then backward (ABBA), as the reference's variance
test does (tests/test_variance.py:141-147).  The DRAM bytes of a cell come
from an ncu pass over one repetition (`--metrics dram__bytes_read.sum,...`):
each cell launches exactly `frames` attention kernels, in cell order.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from kvp.attention import attn_bf16, attn_bf16_multi, read_status
from kvp.frames import run_frames, run_frames_batched, run_reuse_frames
from kvp.session import Session
from kvp.traces import motion_config2, motion_config3, motion_config5, qkv

POLICY_ORDER = ("none", "uniform", "recency", "motion", "reuse_weighted")
BUDGET_FRACS = (0.10, 0.25, 0.50, 1.00)
REGIMES = ("static", "high")


@dataclass
class Cell:
    regime: str
    budget_frac: float
    policy: str


def cell_order() -> list[Cell]:
    return [Cell(r, b, p) for r in REGIMES for b in BUDGET_FRACS for p in POLICY_ORDER]


def cross_flops(frames: int, tokens: int, heads: int, head_dim: int = 128) -> float:
    """4 * T_q * S * head_dim per (frame, head), S = (f+1)*T keys."""
    return float(sum(4 * tokens * (f + 1) * tokens * head_dim for f in range(frames)) * heads)


def run_config5(*, reps: int = 3, frames: int = 16, tokens: int = 1560, heads: int = 12,
                seed: int = 0, max_persist: int | None = None, streaming: bool = False,
                device="cuda", batched: bool = False) -> list[dict]:
    """All 40 cells, `reps` repetitions each in ABBA order; one dict per cell.
    batched (arena mode only): every frame planned first, one grid for all
    frames (kvp.frames.run_frames_batched)."""
    loop = run_frames_batched if batched and not streaming else run_frames
    extra = {} if loop is run_frames_batched else {"streaming": streaming}
    # timed passes run the loop natively (one kvp_session_run_frames or
    # kvp_session_run_frames_batched call)
    timed_extra = {**extra, "native": True}
    from kvp._lib import DeviceInfo, lib
    import ctypes as C
    if max_persist is None:
        info = DeviceInfo()
        lib().kvp_query_device(-1, C.byref(info))
        max_persist = int(info.max_persisting_l2_bytes)
    hidden = heads * 128
    rows = frames * tokens
    q, k, v = (t.to(device) for t in qkv(rows, hidden, seed=seed))
    out = torch.empty_like(q)
    ref = torch.empty_like(q)
    stream = int(torch.cuda.current_stream().cuda_stream)
    flops = cross_flops(frames, tokens, heads)
    cells = cell_order()
    scores = {r: motion_config5(r, frames=frames, seed=seed) for r in REGIMES}
    times = {i: [] for i in range(len(cells))}
    counters = {}
    read_status()
    # warm-up pass over every cell (also the bitwise check against None)
    for i, c in enumerate(cells):
        counters[i] = loop(q, k, v, out, scores[c.regime], policy=c.policy,
                           set_aside=int(c.budget_frac * max_persist), frames=frames,
                           tokens=tokens, heads=heads, stream=stream, **extra)
        if c.policy == "none":
            ref.copy_(out)
        elif not torch.equal(out, ref):
            raise RuntimeError(f"cell {c} differs from the None policy")
    order = []
    for r in range(reps):
        seq = list(range(len(cells)))
        order += seq if r % 2 == 0 else seq[::-1]
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    for i in order:
        c = cells[i]
        loop(q, k, v, out, scores[c.regime], policy=c.policy,
             set_aside=int(c.budget_frac * max_persist), frames=frames, tokens=tokens,
             heads=heads, stream=stream, events=(e0, e1), **timed_extra)
        times[i].append(e0.elapsed_time(e1))
    status = read_status()
    res = []
    for i, c in enumerate(cells):
        t = np.array(times[i])
        res.append({"regime": c.regime, "budget_frac": c.budget_frac,
                    "loop": "batched" if loop is run_frames_batched else ("streaming" if streaming else "arena"),
                    "set_aside_bytes": int(c.budget_frac * max_persist), "policy": c.policy,
                    "ms_mean": round(float(t.mean()), 4), "ms_std": round(float(t.std(ddof=1)) if len(t) > 1 else 0.0, 4),
                    "cv_pct": round(float(100 * t.std(ddof=1) / t.mean()) if len(t) > 1 else 0.0, 3),
                    "tflops": round(flops / (t.mean() / 1e3) / 1e12, 2), "reps": len(t),
                    "copies_per_pass": counters[i]["copies"],
                    "staged_bytes_per_pass": counters[i]["staged_bytes"], "device_status": status})
    return res


def run_config2(*, reps: int = 3, frames: int = 8, tokens: int = 1560, heads: int = 12,
                seed: int = 0, tiles: int = 22, device="cuda", batched: bool = False) -> dict:
    """Config 2: 8 frames cross, AR(1) motion, Recency with 22 tiles (bf16
    budget), arena mode; batched = one grid for all frames."""
    loop = run_frames_batched if batched else run_frames
    hidden = heads * 128
    rows = frames * tokens
    q, k, v = (t.to(device) for t in qkv(rows, hidden, seed=seed))
    out = torch.empty_like(q)
    stream = int(torch.cuda.current_stream().cuda_stream)
    scores = motion_config2(frames=frames, seed=seed)
    set_aside = tiles * 16 * hidden * 2 * 2
    read_status()
    loop(q, k, v, out, scores, policy="recency", set_aside=set_aside, frames=frames,
         tokens=tokens, heads=heads, stream=stream)
    ts = []
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    for _ in range(reps):
        loop(q, k, v, out, scores, policy="recency", set_aside=set_aside, frames=frames,
             tokens=tokens, heads=heads, stream=stream, events=(e0, e1),
             native=True)
        ts.append(e0.elapsed_time(e1))
    t = float(np.mean(ts))
    return {"config": 2, "policy": "recency", "tiles": tiles, "frames": frames,
            "loop": "batched" if batched else "arena",
            "ms_mean": round(t, 4), "tflops": round(cross_flops(frames, tokens, heads) / (t / 1e3) / 1e12, 2),
            "device_status": read_status()}


def window_flops(frames: int, tokens: int, heads: int, layers: int, window: int,
                 head_dim: int = 128) -> float:
    """4 * T_q * S * head_dim per (frame, head, layer), S = min(f+1, window)*T keys."""
    units = sum(min(f + 1, window) for f in range(frames))
    return float(4 * tokens * tokens * head_dim * units * heads * layers)


def run_config3(*, reps: int = 2, frames: int = 50, tokens: int = 1560, heads: int = 12,
                layers: int = 30, window: int = 5, seed: int = 0, streaming: bool = False,
                device="cuda", launch: str = "multi") -> list[dict]:
    """Config 3: per frame one admission (ReuseWeighted over the window's
    tiles, budget = the device's max persisting L2), the admitted rows staged
    into every layer's arena with one launch, then the attention of query
    frame f over key frames max(0, f-window+1)..f in every layer: launch
    "layer" sets each layer's persisting window over its arena and launches
    that layer alone (the reference driver's structure); launch "multi" runs
    every layer through one kvp_attn_bf16_multi call (10 layers a launch)
    under one window over the first layer's arena.  Also the None policy on
    the same inputs."""
    from kvp._lib import DeviceInfo, lib
    import ctypes as C
    info = DeviceInfo()
    lib().kvp_query_device(-1, C.byref(info))
    budget = int(info.max_persisting_l2_bytes)
    hidden = heads * 128
    rows = frames * tokens
    qs, ks, vs = [], [], []
    for layer in range(layers):
        q, k, v = qkv(rows, hidden, seed=seed * 1000 + layer, device=device)
        qs.append(q); ks.append(k); vs.append(v)
    outs = [torch.empty_like(qs[0]) for _ in range(layers)]
    refs = None
    stream = int(torch.cuda.current_stream().cuda_stream)
    scores = motion_config3(frames=frames, seed=seed)
    flops = window_flops(frames, tokens, heads, layers, window)

    def one_pass(policy, events=None):
        s = Session(mode="cross", policy=policy, frames=frames, tokens=tokens, hidden=hidden,
                    elem_bytes=2, set_aside=budget, window=window, layers=layers,
                    streaming=streaming)
        try:
            if events:
                events[0].record()
            for f in range(frames):
                s.plan_frame(f, scores)
                persist = policy != "none"
                if persist:
                    s.upload(stream)
                    s.stage([t.data_ptr() for t in ks], [t.data_ptr() for t in vs], stream)
                if launch == "multi":
                    group = []
                    for layer in range(layers):
                        L = dict(q=qs[layer], k=ks[layer], v=vs[layer], out=outs[layer], heads=heads)
                        if persist:
                            L.update(kvmap_ptr=s.device_map_ptr(), arena_ptr=s.arena_ptr(layer),
                                     arena_rows=s.cap_rows)
                        group.append(L)
                    if persist:
                        s.window(0, stream)
                    attn_bf16_multi(group, tokens=tokens, frames=1, q_frame0=f, mode="causal",
                                    window=window, stream=stream)
                    continue
                for layer in range(layers):
                    if persist:
                        s.window(layer, stream)
                        attn_bf16(qs[layer], ks[layer], vs[layer], outs[layer], tokens=tokens,
                                  frames=1, q_frame0=f, heads=heads, mode="causal", window=window,
                                  kvmap_ptr=s.device_map_ptr(), arena_ptr=s.arena_ptr(layer),
                                  arena_rows=s.cap_rows, stream=stream)
                    else:
                        attn_bf16(qs[layer], ks[layer], vs[layer], outs[layer], tokens=tokens,
                                  frames=1, q_frame0=f, heads=heads, mode="causal", window=window,
                                  stream=stream)
            if policy != "none":
                s.clear_window(stream)
            if events:
                events[1].record()
            torch.cuda.synchronize()
            s.finish()
        finally:
            s.close()

    read_status()
    res = []
    for policy in ("none", "reuse_weighted"):
        one_pass(policy)   # warm-up
        if policy == "none":
            refs = [o.clone() for o in outs]
        else:
            for a, b in zip(outs, refs):
                if not torch.equal(a, b):
                    raise RuntimeError("config 3: ReuseWeighted output differs from None")
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        ts = []
        for _ in range(max(1, reps)):
            one_pass(policy, (e0, e1))
            ts.append(e0.elapsed_time(e1))
        t = float(np.mean(ts))
        res.append({"config": 3, "policy": policy, "streaming": streaming, "launch": launch,
                    "frames": frames,
                    "layers": layers,
                    "window": window, "set_aside_bytes": budget, "ms_mean": round(t, 3),
                    "ms_runs": [round(x, 3) for x in ts],
                    "tflops": round(flops / (t / 1e3) / 1e12, 2), "flop": flops,
                    "device_status": read_status()})
    return res


def run_reuse_matrix(*, reps: int = 3, frames: int = 16, tokens: int = 1560, heads: int = 12,
                     seed: int = 0, max_persist: int | None = None, device="cuda") -> list[dict]:
    """Temporal reuse against re-staging every frame, per (trace, budget,
    policy): intra attention per frame on K/V whose unchanged tiles hold the
    previous frame's rows.  Legs: "none" (no map), "dense" (dense arena, every
    admitted row copied every frame, the reference's staging), "reuse"
    (Session mode reuse).  Every leg's output must equal None's bitwise.
    Traces: AR(1) rho 0.9 (benchmark config 2's motion model, temporally
    coherent) and config 5 'high' (i.i.d. per frame); reuse flags by the
    percentile-50 rule."""
    from kvp._lib import DeviceInfo, lib
    from kvp.traces import hold_reused_tiles, reuse_flags
    import ctypes as C
    if max_persist is None:
        info = DeviceInfo()
        lib().kvp_query_device(-1, C.byref(info))
        max_persist = int(info.max_persisting_l2_bytes)
    hidden = heads * 128
    nt = (tokens + 15) // 16
    traces = {"ar1": motion_config2(frames=frames, seed=seed, tiles=nt),
              "iid": motion_config5("high", frames=frames, seed=seed, tiles=nt)}
    stream = int(torch.cuda.current_stream().cuda_stream)
    flops = float(4 * tokens * tokens * 128 * frames * heads)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    res = []
    for name, scores in traces.items():
        reuse = reuse_flags(scores)
        q, k, v = qkv(frames * tokens, hidden, seed=seed)
        hold_reused_tiles(k, v, reuse, tokens=tokens)
        q, k, v = q.to(device), k.to(device), v.to(device)
        out = torch.empty_like(q)
        ref = torch.empty_like(q)

        def leg(kind, policy, sa, events=None):
            if kind == "reuse":
                return run_reuse_frames(q, k, v, out, scores, reuse, policy=policy, set_aside=sa,
                                        frames=frames, tokens=tokens, heads=heads, stream=stream,
                                        events=events)
            st = run_frames(q, k, v, out, scores, policy=policy, set_aside=sa, frames=frames,
                            tokens=tokens, heads=heads, stream=stream, events=events,
                            mode="intra")
            return {"copies": st["copies"], "staged_bytes": st["staged_bytes"], "hits": 0,
                    "restaged": 0}

        read_status()
        leg("dense", "none", 0)
        ref.copy_(out)
        cells = [("none", "none", 0)]
        for frac in BUDGET_FRACS:
            for policy in POLICY_ORDER[1:]:
                for kind in ("dense", "reuse"):
                    cells.append((kind, policy, int(frac * max_persist)))
        counters = {}
        for c in cells:                       # warm-up + bitwise gate
            counters[c] = leg(*c)
            if not torch.equal(out, ref):
                raise RuntimeError(f"reuse matrix: {name} {c} differs from the None policy")
        times = {c: [] for c in cells}
        order = []
        for r in range(reps):
            order += cells if r % 2 == 0 else cells[::-1]
        for c in order:
            leg(*c, events=(e0, e1))
            times[c].append(e0.elapsed_time(e1))
        status = read_status()
        for c in cells:
            t = np.array(times[c])
            kind, policy, sa = c
            cnt = counters[c]
            copied = cnt["copies"] * 2 * hidden * 2
            res.append({"trace": name, "leg": kind, "policy": policy, "set_aside_bytes": sa,
                        "budget_frac": round(sa / max_persist, 2) if max_persist else 0,
                        "rows_copied": cnt["copies"], "bytes_copied": copied,
                        "rows_restaged": cnt["restaged"], "sticky_hits": cnt["hits"],
                        "ms_mean": round(float(t.mean()), 4),
                        "cv_pct": round(float(100 * t.std(ddof=1) / t.mean()) if len(t) > 1 else 0.0, 3),
                        "tflops": round(flops / (t.mean() / 1e3) / 1e12, 2), "reps": len(t),
                        "device_status": status})
    return res



def run_producer(*, reps: int = 20, warmup: int = 3, frames: int = 21, tokens: int = 1560,
                 heads: int = 12, seed: int = 0, set_aside: int | None = None,
                 device="cuda") -> list[dict]:
    """One layer's K/V production for benchmark config 4 (21 frames x 1560
    tokens, D = 1536, stack admission by ReuseWeighted at the device's max
    persisting L2), CUDA events over `reps` calls each:
      fused         LayerNorm + the tcgen05 producer, which writes every
                    admitted row into the arena in its epilogue (no gather)
      unfused       LayerNorm + three cuBLAS GEMMs on the Q/K/V weight blocks
                    (torch.mm into contiguous q/k/v, bias added) + the
                    session's gather of the admitted rows
      gemm_ours     the producer alone, no map
      gemm_cublas   cuBLAS on the same [rows, 3D] product (torch.addmm)
    x (100 MB) and the outputs (300 MB) exceed L2; W (14 MB) stays in it.
    Arena equality of the fused and gather paths is checked by the GPU tests
    (tests/test_gpu_producer.py)."""
    from kvp._lib import DeviceInfo, lib
    from kvp.producer import layernorm, qkv_project
    from kvp.traces import motion_config4
    import ctypes as C
    if set_aside is None:
        info = DeviceInfo()
        lib().kvp_query_device(-1, C.byref(info))
        set_aside = int(info.max_persisting_l2_bytes)
    D = heads * 128
    rows = frames * tokens
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(rows, D, generator=g).to(torch.bfloat16).to(device)
    w = (0.02 * torch.randn(3 * D, D, generator=g)).to(torch.bfloat16).to(device)
    b = (0.1 * torch.randn(3 * D, generator=g)).to(device)
    gamma = (1 + 0.1 * torch.randn(D, generator=g)).to(device)
    beta = (0.1 * torch.randn(D, generator=g)).to(device)
    h = torch.empty_like(x)
    q, k, v = (torch.empty(rows, D, dtype=torch.bfloat16, device=device) for _ in range(3))
    y3 = torch.empty(rows, 3 * D, dtype=torch.bfloat16, device=device)
    wq, wk, wv = (w[i * D:(i + 1) * D] for i in range(3))
    b16 = b.to(torch.bfloat16)
    bq, bk, bv = (b16[i * D:(i + 1) * D] for i in range(3))
    stream = int(torch.cuda.current_stream().cuda_stream)
    scores = motion_config4(frames=frames, seed=seed, tiles=(tokens + 15) // 16)
    s = Session(mode="stack", policy="reuse_weighted", frames=frames, tokens=tokens, hidden=D,
                elem_bytes=2, set_aside=set_aside, layers=1)
    try:
        st = s.plan_stack(scores)
        s.upload(stream)

        def fused():
            layernorm(x, gamma, beta, h, stream=stream)
            s.produce(0, h, w, b, q, k, v, row0=0, stream=stream)

        def unfused():
            layernorm(x, gamma, beta, h, stream=stream)
            torch.mm(h, wq.t(), out=q)
            q.add_(bq)
            torch.mm(h, wk.t(), out=k)
            k.add_(bk)
            torch.mm(h, wv.t(), out=v)
            v.add_(bv)
            s.stage([k.data_ptr()], [v.data_ptr()], stream)

        def gemm_ours():
            qkv_project(h, w, b, q, k, v, stream=stream)

        def gemm_cublas():
            torch.addmm(b16, h, w.t(), out=y3)

        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)

        def timed(fn):
            for _ in range(warmup):
                fn()
            torch.cuda.synchronize()
            e0.record()
            for _ in range(reps):
                fn()
            e1.record()
            torch.cuda.synchronize()
            return e0.elapsed_time(e1) / reps

        read_status()
        flop = 2.0 * rows * 3 * D * D
        res = []
        for name, fn in (("fused", fused), ("unfused", unfused), ("gemm_ours", gemm_ours),
                         ("gemm_cublas", gemm_cublas)):
            ms = timed(fn)
            res.append({"leg": name, "ms": round(ms, 4),
                        "gemm_tflops": round(flop / (ms / 1e3) / 1e12, 1), "rows": rows, "D": D,
                        "admitted_rows": st.copies, "reps": reps})
        status = read_status()
        for r in res:
            r["device_status"] = status
        return res
    finally:
        torch.cuda.synchronize()
        s.close()


def run_motion(*, frames: int = 20, reps: int = 5, seed: int = 0, cpu_pairs: int = 4,
               device="cuda") -> list[dict]:
    """The motion-trace producer on a seeded 480 x 832 clip: GPU change rates
    for all frame pairs (CUDA events over `reps` passes), and the
    reference's own flow call (OpenCV Farneback on the host cores, the
    threads OpenCV uses) timed on `cpu_pairs` pairs of the same clip."""
    import time
    from kvp.motion import MotionProducer
    from kvp.traces import synthetic_video
    clip = synthetic_video(frames, seed=seed)
    mp = MotionProducer()
    d = torch.from_numpy(clip).to(device)
    change = torch.empty(frames, mp.tiles, device=device)
    stream = int(torch.cuda.current_stream().cuda_stream)
    for _ in range(2):
        mp.change(d, change, stream)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        mp.change(d, change, stream)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    pairs = frames - 1
    res = [{"leg": "gpu", "frames": frames, "pairs": pairs, "ms_per_pass": round(ms, 3),
            "pairs_per_s": round(pairs / (ms / 1e3), 1), "device_status": 0}]
    try:
        import cv2
    except ImportError:
        res.append({"leg": "cpu_opencv", "unavailable": "cv2 not importable"})
        mp.close()
        return res
    t = time.perf_counter()
    for f in range(1, cpu_pairs + 1):
        cv2.calcOpticalFlowFarneback(clip[f - 1], clip[f], None, 0.5, 3, 15, 3, 5, 1.2, 0)
    dt = (time.perf_counter() - t) / cpu_pairs
    res.append({"leg": "cpu_opencv", "pairs": cpu_pairs, "ms_per_pair": round(dt * 1e3, 2),
                "pairs_per_s": round(1.0 / dt, 2), "threads": cv2.getNumThreads(),
                "opencv": cv2.__version__})
    mp.close()
    return res


def run_sdpa_compare(*, reps: int = 20, warmup: int = 3, shapes=((21, 1560), (2, 16380)),
                     heads: int = 12, seed: int = 0, device="cuda") -> list[dict]:
    """The tcgen05 kernel against torch's scaled_dot_product_attention
    backends (cuDNN's fused attention first) on the same work, per (frames,
    tokens) shape: intra-frame attention of `frames` frames x `tokens`
    tokens x `heads` heads, bf16, no mask (per frame, softmax over its own
    tokens).  Inputs are laid out for each side outside the timed region."""
    res = []
    for frames, tokens in shapes:
        for r in _sdpa_compare_one(reps=reps, warmup=warmup, frames=frames, tokens=tokens,
                                   heads=heads, seed=seed, device=device):
            res.append({"frames": frames, "tokens": tokens, **r})
    return res


def _sdpa_compare_one(*, reps, warmup, frames, tokens, heads, seed, device):
    from torch.nn.attention import SDPBackend, sdpa_kernel
    import torch.nn.functional as Fn
    D = heads * 128
    q, k, v = qkv(frames * tokens, D, seed=seed, device=device)
    out = torch.empty_like(q)
    flop = 4.0 * tokens * tokens * 128 * heads * frames
    stream = int(torch.cuda.current_stream().cuda_stream)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    read_status()
    ms = timed(lambda: attn_bf16(q, k, v, out, tokens=tokens, frames=frames, heads=heads,
                                 mode="intra", stream=stream))
    res = [{"leg": "kvp tcgen05", "ms": round(ms, 4), "tflops": round(flop / (ms / 1e3) / 1e12, 1),
            "device_status": read_status()}]
    to4 = lambda t: t.view(frames, tokens, heads, 128).transpose(1, 2).contiguous()
    q4, k4, v4 = to4(q), to4(k), to4(v)
    ref = out.view(frames, tokens, heads, 128).transpose(1, 2).float()
    for name, be in (("cudnn", SDPBackend.CUDNN_ATTENTION), ("flash", SDPBackend.FLASH_ATTENTION),
                     ("efficient", SDPBackend.EFFICIENT_ATTENTION)):
        try:
            with sdpa_kernel(be):
                o4 = Fn.scaled_dot_product_attention(q4, k4, v4)
                torch.cuda.synchronize()
                ms = timed(lambda: Fn.scaled_dot_product_attention(q4, k4, v4))
            err = float((o4.float() - ref).abs().max())
            res.append({"leg": f"sdpa {name}", "ms": round(ms, 4),
                        "tflops": round(flop / (ms / 1e3) / 1e12, 1), "max_abs_vs_kvp": round(err, 5)})
        except Exception as e:  # backend not available for this device / layout
            res.append({"leg": f"sdpa {name}", "unavailable": str(e).splitlines()[0][:160]})
    return res


def slot_order_map(rows_total: int, tile_tokens: int, n_tiles: int, order: str, *, seed: int,
                   device="cuda"):
    """KVMap + arena slots for `n_tiles` admitted tiles (every other
    `tile_tokens`-row tile from row 0) in one of three slot orders:
    "ascending" (each tile on consecutive rising slots, what arena mode
    produces), "descending" (each tile on falling slots, what LIFO slot reuse
    in streaming mode produces) or "permuted" (every row on a random slot).
    Returns (kvmap int64 [rows_total], admitted rows, their slots)."""
    tiles = torch.arange(0, rows_total // tile_tokens, 2, device=device)[:n_tiles]
    rows = (tiles[:, None] * tile_tokens + torch.arange(tile_tokens, device=device)).reshape(-1)
    base = torch.arange(rows.numel(), device=device).view(-1, tile_tokens)
    if order == "ascending":
        slots = base
    elif order == "descending":
        slots = base.flip(1)
    elif order == "permuted":
        g = torch.Generator(device="cpu").manual_seed(seed)
        slots = torch.randperm(rows.numel(), generator=g).to(device)
    else:
        raise ValueError(order)
    slots = slots.reshape(-1)
    kvmap = torch.full((rows_total,), -1, dtype=torch.int64, device=device)
    kvmap[rows] = slots
    return kvmap, rows, slots


def run_slot_orders(*, reps: int = 40, warmup: int = 3, frames: int = 21, tokens: int = 1560,
                    heads: int = 12, admitted_tiles: int = 640, seed: int = 0,
                    device="cuda") -> list[dict]:
    """One config-4 layer (flat causal tiles, 21 frames x 1560 tokens, 12
    heads) with `admitted_tiles` 16-row tiles (10,240 of 32,760 key rows at
    the default) held in the arena in each slot order of `slot_order_map`,
    against the same launch without a map.  The producer fetches ascending
    runs with TMA boxes and scattered all-arena 8-row groups with TMA gathers;
    every output must be bitwise equal to the unmapped launch's."""
    R, D = frames * tokens, heads * 128
    q, k, v = qkv(R, D, seed=seed, device=device)
    out = torch.empty_like(q)
    flop = sum(4.0 * tokens * (f + 1) * tokens * 128 for f in range(frames)) * heads
    stream = int(torch.cuda.current_stream().cuda_stream)
    legs = {"none": (None, None, 0)}
    for order in ("ascending", "descending", "permuted"):
        kvmap, rows, slots = slot_order_map(R, 16, admitted_tiles, order, seed=seed + 1, device=device)
        arena = torch.empty(rows.numel(), 2 * D, dtype=torch.bfloat16, device=device)
        arena[slots, :D] = k[rows]
        arena[slots, D:] = v[rows]
        legs[order] = (kvmap, arena, rows.numel())

    def launch(leg):
        kvmap, arena, arows = legs[leg]
        attn_bf16(q, k, v, out, tokens=tokens, frames=frames, heads=heads, mode="causal", flat=True,
                  kvmap=kvmap, arena=arena, arena_rows=arows, stream=stream)

    read_status()
    launch("none")
    torch.cuda.synchronize()
    ref = out.clone()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    res = []
    for leg in legs:
        for _ in range(warmup):
            launch(leg)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            launch(leg)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        res.append({"slots": leg, "arena_rows": legs[leg][2], "ms": round(ms, 4),
                    "tflops": round(flop / (ms / 1e3) / 1e12, 1),
                    "bitwise_eq_none": bool(torch.equal(out, ref)), "device_status": read_status()})
    return res


def run_config5_producer(*, reps: int = 3, frames: int = 16, tokens: int = 1560, heads: int = 12,
                         seed: int = 0, budgets=(0.10, 1.00), regimes=REGIMES,
                         device="cuda") -> list[dict]:
    """Config 5 cells with the K/V produced inside the per-frame loop, so the
    rows a frame admits need no staging copy.  Per frame f, streaming mode:
    admission (Session.plan_frame), the block's LayerNorm and QKV projection
    of frame f's rows (kvp_session_produce: the epilogue also writes those
    rows' K/V into their slots), a gather of only the earlier frames' newly
    admitted rows (stage_except), the window, and the attention of frame f
    over frames 0..f.  The None leg runs the same LayerNorm and projection
    with no arena.  Outputs are checked bitwise against None.  One dict per
    (regime, budget, policy); `reps` passes each, CUDA events."""
    from kvp._lib import DeviceInfo, lib
    from kvp.producer import layernorm, qkv_project
    import ctypes as C
    info = DeviceInfo()
    lib().kvp_query_device(-1, C.byref(info))
    max_persist = int(info.max_persisting_l2_bytes)
    D = heads * 128
    T = tokens
    rows = frames * T
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(rows, D, generator=g).to(torch.bfloat16).to(device)
    w = (0.02 * torch.randn(3 * D, D, generator=g)).to(torch.bfloat16).to(device)
    b = (0.1 * torch.randn(3 * D, generator=g)).to(device)
    gamma = (1 + 0.1 * torch.randn(D, generator=g)).to(device)
    beta = (0.1 * torch.randn(D, generator=g)).to(device)
    h = torch.empty_like(x)
    q, k, v = (torch.empty(rows, D, dtype=torch.bfloat16, device=device) for _ in range(3))
    out = torch.empty_like(q)
    ref = {}
    stream = int(torch.cuda.current_stream().cuda_stream)
    flops = cross_flops(frames, tokens, heads)
    scores = {r: motion_config5(r, frames=frames, seed=seed) for r in regimes}

    def one_pass(regime, budget, policy, events=None):
        persist = policy != "none"
        s = (Session(mode="cross", policy=policy, frames=frames, tokens=T, hidden=D, elem_bytes=2,
                     set_aside=budget, streaming=True, layers=1) if persist else None)
        copies = 0
        try:
            if events:
                events[0].record()
            for f in range(frames):
                sl = slice(f * T, (f + 1) * T)
                layernorm(x[sl], gamma, beta, h[sl], stream=stream)
                if persist:
                    st = s.plan_frame(f, scores[regime])
                    copies += st.copies
                    s.upload(stream)
                    s.produce(0, h[sl], w, b, q[sl], k[sl], v[sl], row0=f * T, stream=stream)
                    s.stage_except([k.data_ptr()], [v.data_ptr()], f * T, T, stream)
                    s.window(0, stream)
                    attn_bf16(q, k, v, out, tokens=T, frames=1, q_frame0=f, heads=heads,
                              mode="causal", kvmap_ptr=s.device_map_ptr(), arena_ptr=s.arena_ptr(0),
                              arena_rows=s.cap_rows, stream=stream)
                else:
                    qkv_project(h[sl], w, b, q[sl], k[sl], v[sl], stream=stream)
                    attn_bf16(q, k, v, out, tokens=T, frames=1, q_frame0=f, heads=heads,
                              mode="causal", stream=stream)
            if persist:
                s.clear_window(stream)
            if events:
                events[1].record()
            torch.cuda.synchronize()
            if persist:
                s.finish()
        finally:
            if s is not None:
                s.close()
        return copies

    read_status()
    res = []
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    for regime in regimes:
        for frac in budgets:
            budget = int(frac * max_persist)
            for policy in POLICY_ORDER:
                copies = one_pass(regime, budget, policy)   # warm-up and check
                if policy == "none":
                    ref[regime] = out.clone()
                elif not torch.equal(out, ref[regime]):
                    raise RuntimeError(f"producer cell {regime} {frac} {policy} differs from None")
                ts = []
                for _ in range(max(1, reps)):
                    one_pass(regime, budget, policy, (e0, e1))
                    ts.append(e0.elapsed_time(e1))
                t = np.array(ts)
                res.append({"regime": regime, "budget_frac": frac, "set_aside_bytes": budget,
                            "policy": policy, "loop": "streaming+producer",
                            "ms_mean": round(float(t.mean()), 4),
                            "cv_pct": round(float(100 * t.std(ddof=1) / t.mean()) if len(t) > 1 else 0.0, 3),
                            "attention_tflops": round(flops / (t.mean() / 1e3) / 1e12, 2),
                            "staging_copies_per_pass": copies, "reps": len(t)})
    status = read_status()
    for r in res:
        r["device_status"] = status
    return res
