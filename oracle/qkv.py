"""CPU restatement of the block's attention input (src/backbone.py:13-33):
LayerNorm, then qkv_proj, then the column split of
qkv.view(b, t, 3, heads, head_dim).

TEST INFRASTRUCTURE ONLY (the checker of the tcgen05 producer, never the
product path).  Pinned against the reference's own DiTSelfAttentionBlock by
tests/golden/qkv_ref.npz (tests/test_oracle_pins.py).
"""

from __future__ import annotations

import numpy as np


def qkv_params(seed: int, rows: int, D: int):
    """Seeded inputs of the producer golden (tests/golden/qkv_ref.npz):
    x [rows][D], LayerNorm gamma/beta [D], qkv_proj weight [3D][D] and bias
    [3D], all float32 from one numpy generator."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, D)).astype(np.float32)
    gamma = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(D)).astype(np.float32)
    w = (0.02 * rng.standard_normal((3 * D, D))).astype(np.float32)
    b = (0.1 * rng.standard_normal(3 * D)).astype(np.float32)
    return x, gamma, beta, w, b


def layernorm(x: np.ndarray, gamma: np.ndarray, beta: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """nn.LayerNorm over the last axis: biased variance, float64 statistics
    (src/backbone.py:29 nn.LayerNorm(hidden_dim), eps 1e-5)."""
    x = np.asarray(x, dtype=np.float64)
    mean = x.mean(axis=-1, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=-1, keepdims=True)
    return ((x - mean) / np.sqrt(var + eps) * gamma + beta).astype(np.float32)


def qkv_split(h: np.ndarray, w: np.ndarray, b: np.ndarray | None):
    """y = h . w^T + b (nn.Linear(D, 3D), src/backbone.py:13), then the
    view(b, t, 3, heads, head_dim) of :18: Q = y[:, :D], K = y[:, D:2D],
    V = y[:, 2D:], head h at columns [h*head_dim, (h+1)*head_dim) of each
    (the layout the attention kernel reads)."""
    h = np.asarray(h, dtype=np.float64)
    y = h @ np.asarray(w, dtype=np.float64).T
    if b is not None:
        y = y + np.asarray(b, dtype=np.float64)
    D = h.shape[1]
    y = y.astype(np.float32)
    return y[:, :D], y[:, D:2 * D], y[:, 2 * D:]
