"""The reference's CPU attention path, restated with the torch calls it makes.

TEST INFRASTRUCTURE ONLY: timed by bench.py's CPU arms (the `cpu_baseline`
leg and `--impl reference`) and pinned by tests/test_oracle_pins.py; never
imported by the product.

The reference's CPU path is its golden, traces/gen_golden.py:46-74
(attention_reference_cross): per head, query rows in chunks of 128, scores
``q_h[c0:c1] @ k_h.T * (1/sqrt(dh))``, ``torch.softmax`` over the keys, the
row-sum check ``(attn.sum(-1) - 1).abs().max()``, then ``attn @ v_h``, all
fp32 on the host.  That file is Python and cannot travel with this
repository, so this module makes the same library calls in the same order,
which is what its speed depends on; oracle/attention.py is the numpy
checker.  The thread count is set explicitly (torch.set_num_threads), so a
launcher that exports OMP_NUM_THREADS=1 (torchrun does) cannot starve it.
"""

from __future__ import annotations

import math
import os

import torch


def set_threads(n: int | None = None) -> int:
    """Use n host threads (default: every core this process may run on)."""
    if n is None:
        try:
            n = len(os.sched_getaffinity(0))
        except AttributeError:
            n = os.cpu_count() or 1
    torch.set_num_threads(int(n))
    return torch.get_num_threads()


def attention_cross(q: torch.Tensor, ks: list, vs: list, heads: int, head_dim: int,
                    chunk: int = 128):
    """q [T, D] against the key frames ks/vs (lists of [T, D], frames 0..f,
    concatenated first as the reference does); returns (out [T, D], max
    row-sum error).  traces/gen_golden.py:46-74."""
    t = q.shape[0]
    k_all = torch.cat(ks, dim=0)
    v_all = torch.cat(vs, dim=0)
    kh = k_all.view(-1, heads, head_dim).transpose(0, 1)
    vh = v_all.view(-1, heads, head_dim).transpose(0, 1)
    out = torch.empty(t, heads * head_dim)
    scale = 1.0 / math.sqrt(head_dim)
    max_err = 0.0
    with torch.no_grad():
        for h in range(heads):
            q_h = q.view(t, heads, head_dim)[:, h]
            k_h, v_h = kh[h], vh[h]
            for c0 in range(0, t, chunk):
                c1 = min(c0 + chunk, t)
                scores = q_h[c0:c1] @ k_h.transpose(0, 1) * scale
                attn = torch.softmax(scores, dim=-1)
                max_err = max(max_err, float((attn.sum(dim=-1) - 1.0).abs().max()))
                out[c0:c1, h * head_dim:(h + 1) * head_dim] = attn @ v_h
    return out, max_err


def attention_frames(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, frames: int,
                     tokens: int, heads: int, head_dim: int, frame_list=None) -> torch.Tensor:
    """Causal cross-frame attention over a trace of `frames` frames
    ([frames*tokens, D] fp32 tensors): query frame f attends to key frames
    0..f, fed one frame at a time as the reference's golden main() does
    (traces/gen_golden.py:95-110)."""
    out = torch.zeros(frames * tokens, heads * head_dim)
    kf = [k[g * tokens:(g + 1) * tokens] for g in range(frames)]
    vf = [v[g * tokens:(g + 1) * tokens] for g in range(frames)]
    for f in (range(frames) if frame_list is None else frame_list):
        qs = slice(f * tokens, (f + 1) * tokens)
        out[qs], _ = attention_cross(q[qs], kf[:f + 1], vf[:f + 1], heads, head_dim)
    return out
