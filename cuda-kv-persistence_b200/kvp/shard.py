"""(layer, head) pair sharding and the layout of gathered outputs.

A rank owns the contiguous pair block [p0, p1) of p = layer*heads + head.
Its outputs live in one flat bf16 buffer: for each layer chunk in pair
order, an [rows, nheads*128] block (heads interleaved per row, as Q/K/V).
All ranks' buffers have the same length (the pair count divides evenly for
1, 2, 4 and 8 GPUs at 360 pairs), so one all_gather lays rank r's buffer at
offset r * local_elems; ``pair_block`` finds any pair's [rows, 128] output
inside the gathered buffer.
"""

from __future__ import annotations

HEAD_DIM = 128


def pair_range(rank: int, world: int, n_pairs: int):
    """Contiguous block of pairs for `rank` (sizes differ by at most one)."""
    base, extra = divmod(n_pairs, world)
    p0 = rank * base + min(rank, extra)
    return p0, p0 + base + (1 if rank < extra else 0)


def chunks_of(p0: int, p1: int, heads: int):
    """[(layer, head0, nheads)] covering pairs [p0, p1) in order."""
    out = []
    p = p0
    while p < p1:
        layer, h = divmod(p, heads)
        n = min(heads - h, p1 - p)
        out.append((layer, h, n))
        p += n
    return out


def local_layout(p0: int, p1: int, heads: int, rows: int):
    """[(layer, head0, nheads, element offset)] of the rank's flat buffer."""
    off, out = 0, []
    for layer, h0, n in chunks_of(p0, p1, heads):
        out.append((layer, h0, n, off))
        off += rows * n * HEAD_DIM
    return out, off


def pair_block(gathered, world: int, n_pairs: int, heads: int, rows: int, layer: int, head: int):
    """The [rows, 128] output of pair (layer, head) inside a gathered buffer
    (a torch tensor or numpy array of world * local_elems elements)."""
    p = layer * heads + head
    for r in range(world):
        p0, p1 = pair_range(r, world, n_pairs)
        if p0 <= p < p1:
            lay, local_elems = local_layout(p0, p1, heads, rows)
            for lyr, h0, n, off in lay:
                if lyr == layer and h0 <= head < h0 + n:
                    base = r * local_elems + off
                    block = gathered[base: base + rows * n * HEAD_DIM].reshape(rows, n * HEAD_DIM)
                    c = (head - h0) * HEAD_DIM
                    return block[:, c: c + HEAD_DIM]
    raise IndexError((layer, head))
