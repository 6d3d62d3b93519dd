"""Block-causal multi-layer attention stack over (layer, head) pairs.

The Wan2.1-1.3B-shaped workload: F frames of T tokens, L layers x H heads of
128, every query frame attending to key frames 0..f.  Pairs p = layer*H+head
are independent; a rank owns a contiguous block of them and keeps, per
layer, only its heads' columns (Q/K/V/O [F*T, h*128] bf16) and an arena of
those columns.  One stack-mode admission (plan_stack) per step yields one
KVMap shared by every query frame; the rows are gathered into every layer's
arena with one launch, then each layer runs the tcgen05 kernel under a
persisting window over its arena.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .attention import attn_bf16, attn_bf16_multi
from .session import Session
from .shard import chunks_of, pair_range  # noqa: F401  (pair_range re-exported)

HEAD_DIM = 128


@dataclass
class Chunk:
    layer: int
    head0: int      # global head index of the first column block
    nheads: int
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    o: torch.Tensor
    session: int = 0    # index into StackRank.sessions
    slot: int = 0       # arena index within that session


def pair_qkv(layer: int, head: int, rows: int, seed: int, device, heads: int) -> tuple:
    """Q/K/V columns of one (layer, head) pair, N(0,1)/sqrt(128), bf16,
    drawn from a generator seeded by the pair index (independent of sharding)."""
    g = torch.Generator(device=device).manual_seed(seed * 1_000_003 + layer * heads + head)
    s = HEAD_DIM ** -0.5
    return tuple((torch.randn(rows, HEAD_DIM, generator=g, device=device) * s).to(torch.bfloat16)
                 for _ in range(3))


class StackRank:
    def __init__(self, *, p0: int, p1: int, heads: int = 12, frames: int = 21,
                 tokens: int = 1560, policy: str = "reuse_weighted", set_aside: int,
                 streaming: bool = False, device="cuda", seed: int = 0, tile_tokens: int = 16,
                 make_data: bool = True, window: bool = True):
        self.heads, self.frames, self.tokens = heads, frames, tokens
        self.policy = policy
        self.rows = frames * tokens
        self.chunks: list[Chunk] = []
        widths: dict[int, list[int]] = {}
        for layer, h0, n in chunks_of(p0, p1, heads):
            if make_data:
                cols = [pair_qkv(layer, h0 + i, self.rows, seed, device, heads) for i in range(n)]
                q = torch.cat([c[0] for c in cols], 1).contiguous()
                k = torch.cat([c[1] for c in cols], 1).contiguous()
                v = torch.cat([c[2] for c in cols], 1).contiguous()
                del cols
            else:
                q = torch.empty(self.rows, n * HEAD_DIM, dtype=torch.bfloat16, device=device)
                k, v = torch.empty_like(q), torch.empty_like(q)
            o = torch.empty_like(q)
            self.chunks.append(Chunk(layer, h0, n, q, k, v, o))
            widths.setdefault(n, []).append(len(self.chunks) - 1)
        self.sessions: list[Session] = []
        for n, idx in widths.items():
            s = Session(mode="stack", policy=policy, frames=frames, tokens=tokens,
                        hidden=n * HEAD_DIM, tile_tokens=tile_tokens, elem_bytes=2,
                        set_aside=set_aside, streaming=streaming, layers=len(idx))
            for slot, ci in enumerate(idx):
                self.chunks[ci].session = len(self.sessions)
                self.chunks[ci].slot = slot
            self.sessions.append(s)
        self.persist = policy != "none"
        # window=False keeps the arena and the KVMap but sets no persisting
        # access-policy window (measures what persistence itself contributes)
        self.use_window = window

    @property
    def n_pairs(self) -> int:
        return sum(c.nheads for c in self.chunks)

    def flops(self) -> float:
        """Algorithmic FLOP per step: 4*T*S*128 per (frame, pair), real tokens only."""
        T = self.tokens
        per_pair = sum(4 * T * (f + 1) * T * HEAD_DIM for f in range(self.frames))
        return float(per_pair * self.n_pairs)

    def plan_and_stage(self, scores, stream: int) -> None:
        for si, s in enumerate(self.sessions):
            s.plan_stack(scores)
            if not self.persist:
                continue
            s.upload(stream)
            mine = [c for c in self.chunks if c.session == si]
            mine.sort(key=lambda c: c.slot)
            s.stage([c.k.data_ptr() for c in mine], [c.v.data_ptr() for c in mine], stream)

    def attend(self, c: Chunk, stream: int) -> None:
        s = self.sessions[c.session]
        if self.persist:
            if self.use_window:
                s.window(c.slot, stream)
            attn_bf16(c.q, c.k, c.v, c.o, tokens=self.tokens, frames=self.frames,
                      heads=c.nheads, mode="causal", flat=True, kvmap_ptr=s.device_map_ptr(),
                      arena_ptr=s.arena_ptr(c.slot), arena_rows=s.cap_rows, stream=stream)
        else:
            attn_bf16(c.q, c.k, c.v, c.o, tokens=self.tokens, frames=self.frames,
                      heads=c.nheads, mode="causal", flat=True, stream=stream)

    def attend_all(self, stream: int, group: int = 0) -> None:
        """Every chunk through kvp_attn_bf16_multi: the ramp-down of a short
        chunk overlaps the next chunk's work.  group = 0 passes all chunks in
        one call (the library spreads them evenly over as few launches as its
        segment table allows); group > 0 makes one call per `group` chunks.
        One persisting window per call, over the arena of its first chunk."""
        step = group if group > 0 else len(self.chunks)
        for g0 in range(0, len(self.chunks), step):
            grp = self.chunks[g0:g0 + step]
            layers = []
            for c in grp:
                L = dict(q=c.q, k=c.k, v=c.v, out=c.o, heads=c.nheads)
                if self.persist:
                    s = self.sessions[c.session]
                    L.update(kvmap_ptr=s.device_map_ptr(), arena_ptr=s.arena_ptr(c.slot),
                             arena_rows=s.cap_rows)
                layers.append(L)
            if self.persist and self.use_window:
                self.sessions[grp[0].session].window(grp[0].slot, stream)
            attn_bf16_multi(layers, tokens=self.tokens, frames=self.frames, mode="causal",
                            flat=True, stream=stream)

    def step(self, scores, stream: int) -> None:
        self.plan_and_stage(scores, stream)
        for c in self.chunks:
            self.attend(c, stream)
        if self.persist and self.use_window:
            self.sessions[0].clear_window(stream)
