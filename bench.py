"""Benchmark: remapped-MHA TFLOP/s on the Wan2.1-1.3B-shaped causal stack.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl kvp|reference]

Workload (benchmark config 4): 21 latent frames x 1560 tokens = 32,760 tokens,
30 layers x 12 heads x 128 (hidden 1536), bf16, Q/K/V ~ N(0,1)/sqrt(128),
block-causal by frame.  The 360 (layer, head) pairs are split into
contiguous blocks over the ranks (fixed total work: strong scaling); each
rank runs its pairs through the remapped-attention path and the per-rank
outputs are all-gathered over NVLink on separate streams, one step behind,
so the transfer overlaps the next step's compute: by NCCL (the default) or
by the copy engines (peer copies over CUDA IPC, `--gather ce`).

One step = one stack admission (ReuseWeighted over all 21*98 tiles, budget
= this GPU's cudaDevAttrMaxPersistingL2CacheSize), KVMap upload, one
compaction launch into every layer's arena, then per layer a persisting
window and one tcgen05 attention launch (1.0362e14 FLOP over 360 pairs,
counted on real tokens only).  The inputs (12.1 GB) exceed the 126 MB L2,
so no explicit flush is needed between steps.

Printed JSON keys follow the driver contract; `value` times device-resident
inputs, `e2e` times the same work through the public API with host buffers
(pinned H2D of Q/K/V and D2H of O every step, pipelined per layer chunk).
`--impl reference` times the reference's CPU path (the golden attention of
traces/gen_golden.py, restated with the same torch calls in
oracle/golden_torch.py) on all host threads, set explicitly, over a bounded
sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "cuda-kv-persistence_b200"
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(PKG))

FRAMES, TOKENS, LAYERS, HEADS, HEAD_DIM = 21, 1560, 30, 12, 128
N_PAIRS = LAYERS * HEADS
METRIC = "remapped-MHA TFLOP/s"


def attention_kernel() -> str:
    """The bf16 kernel kvp_attn_bf16 launches: the one-SM kernel unless
    KVP_ATTN_PAIR=1 selects the SM-pair kernel."""
    return "attn_pair_sm100_kernel" if os.environ.get("KVP_ATTN_PAIR") == "1" else "attn_bf16_sm100_kernel"


def stack_flops(frames=FRAMES, tokens=TOKENS, pairs=N_PAIRS):
    return float(sum(4 * tokens * (f + 1) * tokens * HEAD_DIM for f in range(frames)) * pairs)


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("bf16_tflops_sustained") or d.get("bf16_tflops"), d.get("hbm_gbs"), "measured"
    return 1400.0, 6650.0, "fallback"


def profiled_traffic_per_layer(kernel: str):
    """DRAM read + write bytes per stack layer of `kernel`'s attention, from
    the committed ncu summaries of stack layers (profiles/*stack21*.md): a
    `traffic_bytes_per_layer` line, else a one-layer launch's
    `traffic_bytes_per_launch`."""
    best = None
    for p in sorted((ROOT / "profiles").glob("*stack21*.md")):
        text = p.read_text()
        if kernel not in text:
            continue
        m = re.search(r"traffic_bytes_per_layer:\s*([0-9.eE+]+)", text)
        if m:
            return float(m.group(1))
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", text)
        if m and best is None:
            best = float(m.group(1))
    return best


def profiled_dram_per_step():
    """DRAM bytes read per config-4 step under the bench's policy and under
    None, from the committed ncu summary profiles/ncu_dram_stack21_step.md
    (one layer captured, scaled to the 30-layer step there)."""
    p = ROOT / "profiles" / "ncu_dram_stack21_step.md"
    if not p.exists():
        return None
    text = p.read_text()
    vals = {}
    for key in ("read_bytes_per_step", "none_read_bytes_per_step", "write_bytes_per_step",
                "none_write_bytes_per_step"):
        m = re.search(key + r":\s*([0-9.eE+]+)", text)
        if m:
            vals[key] = float(m.group(1))
    if "read_bytes_per_step" not in vals or "none_read_bytes_per_step" not in vals:
        return None
    vals["ratio"] = round(vals["read_bytes_per_step"] / vals["none_read_bytes_per_step"], 4)
    vals["source"] = "profiles/ncu_dram_stack21_step.md (ncu dram__bytes_read.sum, one layer x 30)"
    return vals


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        rows = [r.split(",") for r in Path(self.f.name).read_text().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
            except ValueError:
                continue
            for n, val in zip(names, r[5:9]):
                if "Active" in val and "Not" not in val:
                    reasons.add(n)
        if not sm:
            return None
        busy = [x for x in sm if x > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(busy), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ CPU arms
def cpu_attention_sample(seconds: float = 12.0, max_heads: int = HEADS, seed: int = 0):
    """The reference's CPU path -- the golden attention of traces/gen_golden.py,
    restated with the same torch calls (oracle/golden_torch.py) -- on whole
    (layer 0, head h) pairs of the stack, heads taken until `seconds` pass.
    Returns (TFLOP/s, pairs done, seconds, threads)."""
    import torch
    from oracle import golden_torch
    threads = golden_torch.set_threads()
    rows = FRAMES * TOKENS
    done_flops, t_total, heads_done = 0.0, 0.0, 0
    per_pair = stack_flops(pairs=1)
    for h in range(max_heads):
        g = torch.Generator().manual_seed(seed * 1_000_003 + h)
        s = HEAD_DIM ** -0.5
        q, k, v = ((torch.randn(rows, HEAD_DIM, generator=g) * s).to(torch.bfloat16).float()
                   for _ in range(3))
        t0 = time.perf_counter()
        golden_torch.attention_frames(q, k, v, frames=FRAMES, tokens=TOKENS, heads=1,
                                      head_dim=HEAD_DIM)
        t_total += time.perf_counter() - t0
        done_flops += per_pair
        heads_done += 1
        if t_total >= seconds:
            break
    return done_flops / t_total / 1e12, heads_done, t_total, threads


def run_reference(args, rank: int, world: int) -> int:
    if rank != 0:
        return 0
    # One step = one whole (layer, head) pair, all 21 query frames.
    for _ in range(args.warmup):
        cpu_attention_sample(seconds=0.0, max_heads=1)
    t_steps, cores = [], 1
    for i in range(args.steps):
        t0 = time.perf_counter()
        _, _, _, cores = cpu_attention_sample(seconds=0.0, max_heads=1, seed=i)
        t_steps.append(time.perf_counter() - t0)
    per = stack_flops(pairs=1)
    ms = 1e3 * sum(t_steps) / len(t_steps)
    val = per / (ms / 1e3) / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": round(val, 4), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 2),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "wan21_stack_21f_30L_12H_causal", "frames": FRAMES,
                   "tokens_per_frame": TOKENS, "layers": LAYERS, "heads": HEADS,
                   "head_dim": HEAD_DIM, "sample": "one (layer, head) pair, 21 query frames"},
        "cpu_baseline": {"value": round(val, 4), "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": "one (layer, head) pair per step, 21 query frames, "
                                   "traces/gen_golden.py attention_reference_cross restated "
                                   "with its torch calls (oracle/golden_torch.py), fp32"},
        "e2e": {"value": round(val, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ GPU arm
def run_kvp(args, rank: int, world: int, local_rank: int) -> int:
    import numpy as np
    import torch
    import torch.distributed as dist
    from kvp import traces
    from kvp._lib import DeviceInfo, lib
    from kvp.stack import StackRank, pair_range
    import ctypes as C

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    info = DeviceInfo()
    lib().kvp_query_device(local_rank, C.byref(info))
    set_aside = args.set_aside or int(info.max_persisting_l2_bytes)
    p0, p1 = pair_range(rank, world, args.pairs)
    stack = StackRank(p0=p0, p1=p1, heads=HEADS, frames=FRAMES, tokens=TOKENS,
                      policy=args.policy, set_aside=set_aside, device=dev, seed=args.seed,
                      window=args.window == "on")
    with tempfile.TemporaryDirectory() as td:
        scores = traces.csv_round_trip(traces.motion_config4(frames=FRAMES, seed=args.seed), td)
    stream = torch.cuda.Stream(device=dev)
    sp = int(stream.cuda_stream)
    comm = torch.cuda.Stream(device=dev) if world > 1 else None

    # outputs: two flat buffers per rank (the gather of step s overlaps step s+1)
    local_elems = sum(c.o.numel() for c in stack.chunks)
    flat = [torch.empty(local_elems, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    gathered = (torch.empty(local_elems * world, dtype=torch.bfloat16, device=dev)
                if world > 1 else None)
    ce = CopyEngineGather(gathered, flat, rank, world, dev) if world > 1 and args.gather == "ce" else None
    if ce is not None and not ce.ok:
        ce = None   # every rank falls back to NCCL together

    def bind_outputs(buf):
        off = 0
        for c in stack.chunks:
            n = c.o.numel()
            c.o = buf[off:off + n].view(c.o.shape)
            off += n

    if args.launch == "multi":
        per_call = args.group if args.group > 0 else len(stack.chunks)
        attn_launches = sum(-(-min(per_call, len(stack.chunks) - g0) // 12)
                            for g0 in range(0, len(stack.chunks), per_call))
    else:
        attn_launches = len(stack.chunks)
    launches_per_step = attn_launches + (len(stack.sessions) if stack.persist else 0)
    attn_events = []
    gather_done = [None, None]   # last all-gather that read each output buffer

    def one_step(s_idx: int, timed: bool):
        b = s_idx & 1
        if gather_done[b] is not None:
            stream.wait_event(gather_done[b])   # step s-2's gather has read this buffer
        bind_outputs(flat[b])
        with torch.cuda.stream(stream):
            stack.plan_and_stage(scores, sp)
            if args.launch == "multi":
                if timed:
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                stack.attend_all(sp, group=args.group)
                if timed:
                    e1.record(stream)
                    attn_events.append((e0, e1))
            else:
                for c in stack.chunks:
                    if timed:
                        e0 = torch.cuda.Event(enable_timing=True)
                        e1 = torch.cuda.Event(enable_timing=True)
                        e0.record(stream)
                    stack.attend(c, sp)
                    if timed:
                        e1.record(stream)
                        attn_events.append((e0, e1))
            if stack.persist and stack.use_window:
                stack.sessions[0].clear_window(sp)
        if world > 1:
            ev = torch.cuda.Event()
            ev.record(stream)
            if ce is not None:
                gather_done[b] = ce.push(b, ev)
            else:
                comm.wait_event(ev)
                with torch.cuda.stream(comm):
                    dist.all_gather_into_tensor(gathered, flat[b])
                done = torch.cuda.Event()
                done.record(comm)
                gather_done[b] = done

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier(device_ids=[local_rank])
            torch.cuda.synchronize(dev)

    for i in range(args.warmup):
        one_step(i, False)
    barrier()
    sampler = ClockSampler(local_rank) if rank == 0 else None
    if sampler:
        sampler.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        one_step(args.warmup + i, True)
    if world > 1:
        stream.wait_stream(comm)
        if ce is not None:
            ce.join(stream)
    t1.record(stream)
    barrier()
    clocks = sampler.stop() if sampler else None
    ms = t0.elapsed_time(t1) / args.steps
    attn_ms = sum(a.elapsed_time(b) for a, b in attn_events)
    n_attn = len(attn_events)
    status = lib().kvp_read_status(C.c_void_p(sp))
    if world > 1:
        t = torch.tensor([ms, attn_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, attn_ms = float(t[0]), float(t[1])
        st = torch.tensor([status], device=dev, dtype=torch.int32)
        dist.all_reduce(st, op=dist.ReduceOp.MAX)
        status = int(st[0])
    total_flops = stack_flops(pairs=args.pairs)
    value = total_flops / (ms / 1e3) / 1e12

    gather_check = None
    if world > 1:
        # The last step's gather must hold every rank's outputs: compare each
        # rank's own checksum with the checksum of its segment on rank 0.
        last = flat[(args.warmup + args.steps - 1) & 1]
        mine = torch.tensor([last.double().sum().item()], device=dev, dtype=torch.float64)
        sums = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(sums, mine)
        seg = gathered.view(world, -1).double().sum(dim=1)
        gather_check = bool(torch.allclose(seg, torch.cat(sums), rtol=0, atol=0))

    # ---------------- e2e through the public API with pinned host buffers
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, stack, scores, dev, stream, world, local_rank)

    if world > 1:
        dist.barrier(device_ids=[local_rank])
    result = 0
    if rank == 0:
        peak, hbm, peak_kind = measured_peaks()
        local_attn_flops = stack.flops() * args.steps
        achieved = local_attn_flops / (attn_ms / 1e3) / 1e12 if attn_ms > 0 else None
        per_launch_flops = local_attn_flops / max(n_attn, 1)
        traffic_layer = profiled_traffic_per_layer(attention_kernel())
        layers_per_event = stack.n_pairs / HEADS * args.steps / max(n_attn, 1)
        roofline = {"bound": "tensor", "achieved": round(achieved, 2) if achieved else None,
                    "peak": peak, "unit": "TFLOP/s",
                    "frac": round(achieved / peak, 4) if achieved else None,
                    "traffic": (round(traffic_layer * layers_per_event) if traffic_layer else None),
                    "traffic_unit": "DRAM bytes per timed attention unit (the step's attention "
                                    "launches on this rank), from the per-layer ncu figure",
                    "kernel": attention_kernel(),
                    "peak_kind": f"{peak_kind} bf16 sustained (cuBLAS)",
                    "flop_per_launch": per_launch_flops,
                    "avg_launch_ms": round(attn_ms / max(n_attn, 1), 4)}
        cpu = None
        if world == 1 and not args.no_cpu:
            tf, heads_done, secs, threads = cpu_attention_sample(seconds=args.cpu_seconds)
            cpu = {"value": round(tf, 4), "unit": "TFLOP/s", "cores": threads,
                   "kind": "port",
                   "sample": f"layer 0, {heads_done} head(s) x 21 query frames ({secs:.1f} s), "
                             "traces/gen_golden.py attention_reference_cross restated with its "
                             "torch calls (oracle/golden_torch.py), fp32"}
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1)/sqrt(128) Q/K/V, U[0,1) tile motion)",
            "config": {"workload": "wan21_stack_21f_30L_12H_causal", "frames": FRAMES,
                       "tokens_per_frame": TOKENS, "layers": LAYERS, "heads": HEADS,
                       "head_dim": HEAD_DIM, "pairs": args.pairs, "policy": args.policy,
                       "set_aside_bytes": set_aside, "persisting_window": args.window,
                       "attention_launches": f"{args.launch} ({attn_launches} per step)",
                       "mask": "block-causal by frame",
                       "flop_per_step": total_flops,
                       "l2": "inputs 12.1 GB exceed the 126 MB L2 (no flush needed)",
                       "parallelism": f"pairs/{world}" + ((" + nccl all_gather" if ce is None else
                                                           " + copy-engine all_gather (peer copies)")
                                                          if world > 1 else "")},
            "roofline": roofline,
            "dram": profiled_dram_per_step(),
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
            "device_status": status,
            "gather_check": gather_check,
        }
        print(json.dumps(line), flush=True)
        if status != 0:
            result = 3
    if world > 1:
        torch.cuda.synchronize(dev)
        dist.barrier(device_ids=[local_rank])
        if ce is not None:
            ce.close()
            dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    return result


class CopyEngineGather:
    """The outputs' all-gather done by the copy engines instead of NCCL's
    kernels: each rank writes its segment straight into every peer's
    gathered buffer (CUDA IPC, cudaMemcpyAsync over NVLink), one stream per
    peer.  The attention grid fills every SM, and a collective's CTAs would
    take SMs from it; copy engines take none."""

    def __init__(self, gathered, flat, rank, world, dev):
        import torch
        import torch.distributed as dist
        from cuda.bindings import driver as cu, runtime as rt
        self.rt, self.rank, self.world, self.torch = rt, rank, world, torch
        self.nbytes = flat[0].numel() * flat[0].element_size()
        self.flat_ptr = [t.data_ptr() for t in flat]
        self.opened, self.dst = [], {}
        ptr = gathered.data_ptr()
        # Every rank takes the same collective steps whatever fails locally:
        # export, exchange, import, then agree; if any rank could not, none
        # uses the copy engines (self.ok False: the caller falls back).
        mine = None
        try:
            err, base, _ = cu.cuMemGetAddressRange(ptr)
            self._check(err, "cuMemGetAddressRange")
            err, handle = rt.cudaIpcGetMemHandle(int(base))
            self._check(err, "cudaIpcGetMemHandle")
            mine = (bytes(handle.reserved), ptr - int(base))
        except Exception as e:  # noqa: BLE001 -- reported, then agreed on below
            print(f"rank {rank}: copy-engine gather unavailable ({e})", flush=True)
        objs = [None] * world
        dist.all_gather_object(objs, mine)
        ok = all(o is not None for o in objs)
        if ok:
            try:
                for p in range(world):
                    if p == rank:
                        self.dst[p] = ptr + rank * self.nbytes
                        continue
                    h = rt.cudaIpcMemHandle_t()
                    h.reserved = objs[p][0]
                    err, pbase = rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess)
                    self._check(err, f"cudaIpcOpenMemHandle(rank {p})")
                    self.opened.append(int(pbase))
                    self.dst[p] = int(pbase) + objs[p][1] + rank * self.nbytes
            except Exception as e:  # noqa: BLE001
                print(f"rank {rank}: copy-engine gather unavailable ({e})", flush=True)
                ok = False
        flag = torch.tensor([1 if ok else 0], device=dev, dtype=torch.int32)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        self.ok = bool(flag.item())
        if not self.ok:
            self.close()
        self.streams = {p: torch.cuda.Stream(device=dev) for p in range(world)} if self.ok else {}

    @staticmethod
    def _check(err, what):
        if int(err) != 0:
            raise RuntimeError(f"{what} failed: {err}")

    def push(self, b, ready):
        """Copy output buffer b to every rank once `ready` has passed; returns
        an event that passes once every copy has read the buffer."""
        kind = self.rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice
        dones = []
        for p, st in self.streams.items():
            st.wait_event(ready)
            err, = self.rt.cudaMemcpyAsync(self.dst[p], self.flat_ptr[b], self.nbytes, kind,
                                           self.rt.cudaStream_t(st.cuda_stream))
            self._check(err, "cudaMemcpyAsync")
            e = self.torch.cuda.Event()
            e.record(st)
            dones.append(e)
        # one event on the first stream that follows every copy
        head = self.streams[0]
        for e in dones[1:]:
            head.wait_event(e)
        done = self.torch.cuda.Event()
        done.record(head)
        return done

    def join(self, stream):
        for st in self.streams.values():
            stream.wait_stream(st)

    def close(self):
        for pb in self.opened:
            self.rt.cudaIpcCloseMemHandle(pb)
        self.opened = []


def run_e2e(args, stack, scores, dev, stream, world, local_rank):
    """Same step with Q/K/V copied from pinned host memory and O copied back,
    per layer chunk: H2D(chunk c+1) overlaps compute(c), D2H(c) overlaps
    compute(c+1).

    Every host-to-device copy of a step -- the KVMap upload first, then the
    Q/K/V chunks -- goes through the one copy stream, in the order the
    compute needs it.  A small copy queued on the compute stream instead
    waits behind every bulk copy already queued on the copy stream (the copy
    engine does not interleave them), which held each step's first layer
    back until the copy stream had drained.  The copy stream waits for the
    previous step's last layer before it overwrites the map and the chunk
    buffers; each layer waits for the previous step's read-back of its
    output buffer."""
    import torch
    import torch.distributed as dist
    h2d = torch.cuda.Stream(device=dev)
    d2h = torch.cuda.Stream(device=dev)
    host = []
    for c in stack.chunks:
        host.append(tuple(t.to("cpu").pin_memory() for t in (c.q, c.k, c.v)) +
                    (torch.empty(c.o.shape, dtype=torch.bfloat16).pin_memory(),))
    sp = int(stream.cuda_stream)
    hp = int(h2d.cuda_stream)
    h2d_bytes = sum(sum(t.numel() * 2 for t in h[:3]) for h in host)
    d2h_bytes = sum(h[3].numel() * 2 for h in host)
    prev = {"done": None, "read_back": [None] * len(stack.chunks)}

    def step():
        with torch.cuda.stream(h2d):
            if prev["done"] is not None:
                h2d.wait_event(prev["done"])      # last step's layers have read map and inputs
            # admission + map upload for the step, ahead of the bulk copies
            for s in stack.sessions:
                s.plan_stack(scores)
                if stack.persist:
                    s.upload(hp)
            map_ready = torch.cuda.Event()
            map_ready.record(h2d)
            loaded = []
            for i, c in enumerate(stack.chunks):
                hq, hk, hv, _ = host[i]
                c.k.copy_(hk, non_blocking=True)
                c.v.copy_(hv, non_blocking=True)
                c.q.copy_(hq, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(h2d)
                loaded.append(ev)
        stream.wait_event(map_ready)
        for i, c in enumerate(stack.chunks):
            stream.wait_event(loaded[i])
            if prev["read_back"][i] is not None:
                stream.wait_event(prev["read_back"][i])
            if stack.persist:
                stack.sessions[c.session].stage_layer(c.slot, c.k.data_ptr(), c.v.data_ptr(), sp)
            stack.attend(c, sp)
            ev = torch.cuda.Event()
            ev.record(stream)
            d2h.wait_event(ev)
            with torch.cuda.stream(d2h):
                host[i][3].copy_(c.o, non_blocking=True)
                rb = torch.cuda.Event()
                rb.record(d2h)
            prev["read_back"][i] = rb
        prev["done"] = ev
        if stack.persist and stack.use_window:
            stack.sessions[0].clear_window(sp)

    for _ in range(max(1, min(args.warmup, 2))):
        step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    n = max(1, min(args.steps, 5))
    e0.record(stream)
    for _ in range(n):
        step()
    stream.wait_stream(d2h)
    stream.wait_stream(h2d)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / n
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
    return {"value": round(stack_flops(pairs=args.pairs) / (ms / 1e3) / 1e12, 2), "unit": "TFLOP/s",
            "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": d2h_bytes,
            "ms_per_step": round(ms, 2), "steps": n,
            "path": "kvp Session + kvp_attn_bf16 C ABI, pinned host Q/K/V/O per layer chunk"}


def run_matrix(args) -> int:
    """Per-frame cross-attention measurements (bench_matrix.py), 1 GPU."""
    import torch
    import bench_matrix as matrix
    torch.cuda.set_device(0)
    if args.matrix == 5:
        for row in matrix.run_config5(reps=max(1, args.reps), seed=args.seed,
                                      streaming=args.streaming, batched=args.batched):
            print(json.dumps({"metric": "config5 cell", "streaming": args.streaming, **row}),
                  flush=True)
    elif args.matrix == 11:
        regimes = ("static", "high") if args.regime == "both" else (args.regime,)
        budgets = tuple(float(x) for x in args.budgets.split(","))
        for row in matrix.run_config5_producer(reps=max(1, args.reps), seed=args.seed,
                                               regimes=regimes, budgets=budgets):
            print(json.dumps({"metric": "config5 cell, K/V produced in the loop", **row}), flush=True)
    elif args.matrix == 10:
        for row in matrix.run_slot_orders(reps=max(1, args.reps) * 10, seed=args.seed):
            print(json.dumps({"metric": "one config-4 layer by arena slot order", **row}), flush=True)
    elif args.matrix == 9:
        for row in matrix.run_sdpa_compare(reps=max(1, args.reps), seed=args.seed):
            print(json.dumps({"metric": "intra-frame attention, 12 heads, bf16", **row}), flush=True)
    elif args.matrix == 8:
        for row in matrix.run_motion(reps=max(1, args.reps), seed=args.seed):
            print(json.dumps({"metric": "motion-trace producer, 480x832 frame pairs", **row}),
                  flush=True)
    elif args.matrix == 7:
        for row in matrix.run_producer(reps=max(1, args.reps), seed=args.seed):
            print(json.dumps({"metric": "qkv producer, one layer of config 4", **row}), flush=True)
    elif args.matrix == 6:
        for row in matrix.run_reuse_matrix(reps=max(1, args.reps), seed=args.seed):
            print(json.dumps({"metric": "temporal reuse cell", **row}), flush=True)
    elif args.matrix == 3:
        for row in matrix.run_config3(reps=max(1, args.reps), seed=args.seed,
                                      streaming=args.streaming, launch=args.launch):
            print(json.dumps({"metric": "config3", **row}), flush=True)
    else:
        # the per-frame loop, then all frames in one grid (--batched: that alone)
        for batched in ((True,) if args.batched else (False, True)):
            print(json.dumps({"metric": "config2", **matrix.run_config2(reps=max(1, args.reps),
                                                                       seed=args.seed,
                                                                       batched=batched)}),
                  flush=True)
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["kvp", "reference"], default="kvp")
    ap.add_argument("--policy", default="reuse_weighted",
                    choices=["none", "uniform", "recency", "motion", "reuse_weighted"])
    ap.add_argument("--set-aside", type=int, default=0, help="bytes (0 = device max persisting L2)")
    ap.add_argument("--window", choices=["on", "off"], default="on",
                    help="persisting access-policy window over each layer's arena")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--pairs", type=int, default=N_PAIRS,
                    help="(layer, head) pairs of the stack (360 = the full config; fewer only for profiling)")
    ap.add_argument("--launch", choices=["multi", "layer"], default="multi",
                    help="attention launches: several layer chunks per launch (kvp_attn_bf16_multi) "
                         "or one per layer chunk (kvp_attn_bf16)")
    ap.add_argument("--group", type=int, default=0,
                    help="layer chunks per kvp_attn_bf16_multi call with --launch multi (0 = all; "
                         "the library then spreads them evenly over launches of at most 12)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--matrix", type=int, choices=[2, 3, 5, 6, 7, 8, 9, 10, 11], default=0,
                    help="instead of the config-4 line: config 5 (policy x budget x regime, one "
                         "JSON line per cell), config 3 (50 frames x 30 layers, window 5; None "
                         "and ReuseWeighted) or config 2 (one line), per-frame cross attention; "
                         "6: temporal reuse (intra per frame, tiles re-copied only when changed) "
                         "against re-staging every frame, per trace x budget x policy; 7: one "
                         "layer's K/V production for config 4 (LayerNorm + tcgen05 QKV producer "
                         "writing the arena, against cuBLAS + gather); 8: the motion-trace "
                         "producer (GPU optical flow + tile rates) against OpenCV on the host; 9: "
                         "the attention kernel against torch SDPA backends (cuDNN first) on "
                         "intra-frame attention; 10: one config-4 layer with admitted tiles on "
                         "ascending, descending and permuted arena slots against no map; 11: "
                         "config-5 cells (10 %% and 100 %% budgets) with the K/V produced in the "
                         "per-frame streaming loop, so admitted rows of the current frame are "
                         "written by the QKV epilogue instead of staged")
    ap.add_argument("--reps", type=int, default=3, help="repetitions per cell with --matrix (ABBA)")
    ap.add_argument("--gather", choices=["nccl", "ce"], default="nccl",
                    help="with --gpus > 1: all-gather the outputs with NCCL's all_gather_into_tensor, "
                         "or with the copy engines (every rank writes its segment into each peer's "
                         "buffer over CUDA IPC; no SMs taken from the attention)")
    ap.add_argument("--regime", choices=["static", "high", "both"], default="both",
                    help="--matrix 11: motion regimes")
    ap.add_argument("--budgets", default="0.1,1.0",
                    help="--matrix 11: budget fractions of the max persisting L2, comma-separated")
    ap.add_argument("--batched", action="store_true",
                    help="--matrix 2/5 arena mode: plan every frame first, one grid for all frames "
                         "(one kvp_session_run_frames_batched call); --matrix 2 runs both loops "
                         "without it")
    ap.add_argument("--streaming", action="store_true",
                    help="with --matrix 3 or 5: streaming arena (sticky slots, LIFO reuse) instead of "
                         "re-staging every admitted row every frame")
    args = ap.parse_args()
    if args.matrix:
        return run_matrix(args)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and "WORLD_SIZE" in os.environ:
        world = int(os.environ["WORLD_SIZE"])
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if world > 1 and "RANK" not in os.environ:
        print("for --gpus > 1 launch with torch.distributed.run", file=sys.stderr)
        return 2
    return run_kvp(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
