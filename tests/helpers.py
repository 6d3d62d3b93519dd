"""Shared helpers for the parity tests (inputs, oracle comparisons)."""

from __future__ import annotations

import math

import numpy as np
import torch


def rand_qkv(rows: int, hidden: int, seed: int, dtype=np.float32):
    """N(0,1)/sqrt(128) Q/K/V on the CPU (numpy), reproducible."""
    rng = np.random.default_rng(seed)
    s = 1.0 / math.sqrt(128)
    return [(rng.standard_normal((rows, hidden), dtype=np.float32) * s).astype(dtype)
            for _ in range(3)]


def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 values exactly representable in bf16 (round to nearest even)."""
    return torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16).float().numpy()


def build_arena(k: np.ndarray, v: np.ndarray, kvmap: np.ndarray, arena_rows: int) -> np.ndarray:
    """Arena [arena_rows, 2D] = K row || V row for every mapped key row."""
    D = k.shape[1]
    arena = np.zeros((arena_rows, 2 * D), dtype=k.dtype)
    rows = np.nonzero(kvmap >= 0)[0]
    arena[kvmap[rows], :D] = k[rows]
    arena[kvmap[rows], D:] = v[rows]
    return arena


def errors(got: np.ndarray, want: np.ndarray):
    d = np.abs(got.astype(np.float64) - want.astype(np.float64))
    return float(d.max()), float(d.mean())
