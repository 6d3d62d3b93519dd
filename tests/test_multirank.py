"""Multi-rank host logic on the CPU (gloo, world size 2).

The GPU path shards (layer, head) pairs across ranks and all-gathers the
outputs over NCCL; here the same sharding, admission and gather layout run
as gloo ranks: every pair is owned exactly once, every rank plans the same
KVMap, and each pair's output is found where ``kvp.shard.pair_block`` says.
Failure detection is host-side: a rank that never joins makes the others'
next collective end with an error after a short timeout (no GPU involved).
"""

from __future__ import annotations

import hashlib
import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    for p in (str(ROOT), str(ROOT / "cuda-kv-persistence_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=timeout_s))


def _worker_shard_and_gather(rank, world, port, out_dir):
    _init(rank, world, port)
    from kvp.session import Session
    from kvp.shard import local_layout, pair_block, pair_range
    from kvp.traces import read_motion_csv
    heads, layers, rows = 12, 30, 64
    n_pairs = heads * layers
    p0, p1 = pair_range(rank, world, n_pairs)
    # 1) ownership: every pair exactly once
    rng_t = torch.tensor([p0, p1], dtype=torch.int64)
    got = [torch.zeros(2, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(got, rng_t)
    flat = sorted(p for a, b in got for p in range(int(a), int(b)))
    assert flat == list(range(n_pairs))
    # 2) the same stack admission on every rank
    scores = read_motion_csv(ROOT / "tests" / "golden" / "motion_config4.csv", 21, 98)
    s = Session(mode="stack", policy="reuse_weighted", frames=21, elem_bytes=2,
                set_aside=82_903_040)
    s.plan_stack(scores)
    h = hashlib.sha256(s.host_map().tobytes()).digest()
    ht = torch.tensor(list(h), dtype=torch.uint8)
    hs = [torch.zeros(32, dtype=torch.uint8) for _ in range(world)]
    dist.all_gather(hs, ht)
    assert all(torch.equal(x, hs[0]) for x in hs)
    # 3) gather layout: pair-coded outputs land where pair_block says
    lay, local_elems = local_layout(p0, p1, heads, rows)
    buf = torch.empty(local_elems, dtype=torch.float32)
    for layer, h0, n, off in lay:
        blk = buf[off: off + rows * n * 128].view(rows, n * 128)
        for i in range(n):
            blk[:, i * 128:(i + 1) * 128] = float((layer * heads + h0 + i) * 1000)
        blk += torch.arange(rows, dtype=torch.float32).unsqueeze(1)
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf)
    gathered = torch.cat(parts)
    if rank == 0:
        for layer in range(layers):
            for head in range(heads):
                b = pair_block(gathered, world, n_pairs, heads, rows, layer, head)
                want = (layer * heads + head) * 1000 + torch.arange(rows).unsqueeze(1).float()
                assert torch.equal(b, want.expand(rows, 128)), (layer, head)
        (Path(out_dir) / "ok").write_text("ok")
    dist.barrier()
    dist.destroy_process_group()


def test_two_ranks_shard_plan_and_gather(tmp_path):
    mp.spawn(_worker_shard_and_gather, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    assert (tmp_path / "ok").exists()


def _worker_dead_peer(rank, world, port, out_dir):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        # this rank leaves between steps: it never joins the next collective
        os._exit(0)
    try:
        dist.barrier()
        outcome = "no error"
    except Exception as e:  # the survivor learns of the failure on the host
        outcome = "error: " + type(e).__name__
    (Path(out_dir) / f"rank{rank}").write_text(outcome)
    os._exit(0)


def test_dead_peer_is_detected_on_the_host(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    ps = [ctx.Process(target=_worker_dead_peer, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=120)
        assert not p.is_alive()
    assert (tmp_path / "rank0").read_text().startswith("error")


def _worker_ce_fallback(rank, world, port, out_dir):
    _init(rank, world, port, timeout_s=30)
    import bench
    from cuda.bindings import driver as cu, runtime as rt
    if rank == 0:
        # rank 0 exports a (fake) handle; rank 1 fails (no GPU here)
        class _H:
            reserved = bytes(64)
        cu.cuMemGetAddressRange = lambda ptr: (0, ptr, 1 << 20)
        rt.cudaIpcGetMemHandle = lambda base: (0, _H())
    flat = [torch.zeros(16, dtype=torch.bfloat16) for _ in range(2)]
    gathered = torch.zeros(16 * world, dtype=torch.bfloat16)
    ce = bench.CopyEngineGather(gathered, flat, rank, world, "cpu")
    (Path(out_dir) / f"rank{rank}").write_text("ok" if ce.ok else "fallback")
    dist.barrier()
    dist.destroy_process_group()


def test_copy_engine_gather_falls_back_on_every_rank(tmp_path):
    """bench.CopyEngineGather: when one rank cannot export or open its IPC
    handle, every rank takes the same collective steps and all fall back to
    NCCL together (none is left waiting in a collective the others skip)."""
    mp.spawn(_worker_ce_fallback, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    assert (tmp_path / "rank0").read_text() == "fallback"
    assert (tmp_path / "rank1").read_text() == "fallback"
