"""CPU oracle for the attention math (numpy restatement of the reference golden).

TEST INFRASTRUCTURE ONLY: the checker for tests/, __graft_entry__.smoke() and
the CPU baseline leg of bench.py.

Restates GauthamMK-0/cuda-kv-persistence traces/gen_golden.py:
  * ``intra``  -- attention_reference (traces/gen_golden.py:30-43): explicit
    matmul, ``/ sqrt(dh)``, softmax over keys, ``@ V``, FP32;
  * ``cross``  -- attention_reference_cross (traces/gen_golden.py:46-74): frame
    f attends to key frames 0..f, query rows processed in chunks of 128,
    scores scaled by ``* (1/sqrt(dh))``.
``window`` extends cross to key frames [max(0, f-W+1), f] (new behaviour, the
reference has no window).  The KVMap never changes results: arena rows are
exact copies of base rows (src/kv_tile_manager.cu:104-121), so the oracle
reads base K/V only.

Layout matches the reference kernel: Q/K/V/O are [rows, D] with D = H*dh and
head h in columns [h*dh, (h+1)*dh) (src/gated_attention_kernel.cu:54-83).
"""

from __future__ import annotations

import math

import numpy as np


def _softmax_rows(s: np.ndarray) -> np.ndarray:
    s = s - s.max(axis=-1, keepdims=True)
    np.exp(s, out=s)
    s /= s.sum(axis=-1, keepdims=True)
    return s


def attention_intra(q: np.ndarray, k: np.ndarray, v: np.ndarray, heads: int,
                    head_dim: int) -> np.ndarray:
    """One frame, keys = the same frame (traces/gen_golden.py:30-43)."""
    t = q.shape[0]
    out = np.empty((t, heads * head_dim), dtype=np.float32)
    for h in range(heads):
        cs = slice(h * head_dim, (h + 1) * head_dim)
        scores = (q[:, cs] @ k[:, cs].T) / np.float32(math.sqrt(head_dim))
        out[:, cs] = _softmax_rows(scores.astype(np.float32)) @ v[:, cs]
    return out


def attention_keys(q: np.ndarray, k_span: np.ndarray, v_span: np.ndarray, heads: int,
                   head_dim: int, chunk: int = 128, heads_subset=None) -> np.ndarray:
    """Query rows against an explicit key span, chunked by 128 query rows
    (traces/gen_golden.py:46-74)."""
    t = q.shape[0]
    scale = np.float32(1.0 / math.sqrt(head_dim))
    out = np.zeros((t, heads * head_dim), dtype=np.float32)
    for h in (range(heads) if heads_subset is None else heads_subset):
        cs = slice(h * head_dim, (h + 1) * head_dim)
        kh = np.ascontiguousarray(k_span[:, cs])
        vh = np.ascontiguousarray(v_span[:, cs])
        for c0 in range(0, t, chunk):
            c1 = min(c0 + chunk, t)
            scores = (q[c0:c1, cs] @ kh.T) * scale
            out[c0:c1, cs] = _softmax_rows(scores) @ vh
    return out


def attention_frames(q: np.ndarray, k: np.ndarray, v: np.ndarray, *, frames: int,
                     tokens: int, heads: int, head_dim: int, mode: str = "cross",
                     window: int = 0, frame_list=None, heads_subset=None) -> np.ndarray:
    """Full-trace golden: q/k/v are [frames*tokens, D]; returns [frames*tokens, D].

    mode 'intra' | 'cross'; window > 0 restricts cross keys to the last W
    frames.  frame_list limits which query frames are computed (others stay 0).
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    out = np.zeros((frames * tokens, heads * head_dim), dtype=np.float32)
    for f in (range(frames) if frame_list is None else frame_list):
        qs = slice(f * tokens, (f + 1) * tokens)
        if mode == "intra":
            if heads_subset is None:
                out[qs] = attention_intra(q[qs], k[qs], v[qs], heads, head_dim)
            else:
                out[qs] = attention_keys(q[qs], k[qs], v[qs], heads, head_dim,
                                         chunk=tokens, heads_subset=heads_subset)
            continue
        base = max(0, f - window + 1) if window > 0 else 0
        ks = slice(base * tokens, (f + 1) * tokens)
        out[qs] = attention_keys(q[qs], k[ks], v[ks], heads, head_dim,
                                 heads_subset=heads_subset)
    return out


def flops(frames: int, tokens: int, heads: int, head_dim: int, mode: str = "cross",
          window: int = 0) -> float:
    """Algorithmic FLOP: 4 * T_q * S * dh per (frame, head) on real tokens."""
    total = 0
    for f in range(frames):
        if mode == "intra":
            s = tokens
        else:
            base = max(0, f - window + 1) if window > 0 else 0
            s = (f + 1 - base) * tokens
        total += 4 * tokens * s * head_dim * heads
    return float(total)
