"""Synthetic inputs and the motion-trace CSV format.

* ``reference_synthetic_trace`` restates the reference's synthetic trace
  generator (traces/gen_synthetic_motion.py:41-89 scores, :125-171 Q/K/V
  with motion-coupled K/V drift) with the same constants and the same draw
  order from one seeded torch.Generator, so seed 42 / 8 frames reproduces
  the reference's trace_meta_8f.json and golden_meta.json statistics.
* ``motion_config{1..5}`` are seeded motion generators for the five
  benchmark configurations (the reference ships no generator for them; each
  docstring states its distribution).  Each uses its own
  ``torch.Generator().manual_seed(seed)``; Q/K/V come from ``qkv``.
* ``reuse_flags``, ``hold_reused_tiles`` and ``synthetic_video`` feed the
  temporal-reuse and motion-producer paths.
* ``write_motion_csv`` writes the reference CSV
  (frame_id,tile_id,motion_score,is_static,token_start,token_count) with
  6-decimal scores, the text the reference driver parses with "%f".
"""

from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import torch

TOKENS, HIDDEN, HEADS, HEAD_DIM, TILE = 1560, 1536, 12, 128, 16

# traces/gen_synthetic_motion.py:32-39
_STATIC_MEAN, _STATIC_STD, _STATIC_JITTER = 0.05, 0.02, 0.01
_MOVING_MEAN, _MOVING_STD, _MOVING_WALK = 1.5, 0.4, 0.25
_MOVING_CLIP = (0.8, 4.0)
_KV_DRIFT = 0.15


def tile_counts(tokens: int = TOKENS, tile_tokens: int = TILE) -> np.ndarray:
    full, rem = divmod(tokens, tile_tokens)
    c = [tile_tokens] * full + ([rem] if rem else [])
    return np.asarray(c, dtype=np.int64)


def reference_synthetic_trace(frames: int = 8, seed: int = 42, frac_static: float = 0.65,
                              tokens: int = TOKENS, hidden: int = HIDDEN,
                              tile_tokens: int = TILE):
    """(scores [F, tiles] f32, is_static [tiles] bool, Q, K, V [F, T, D] f32 numpy)."""
    g = torch.Generator().manual_seed(seed)
    counts = torch.from_numpy(tile_counts(tokens, tile_tokens))
    n = counts.numel()
    # motion: regime flag, static base, moving start, then per-frame jitter/walk pairs
    is_static = torch.rand(n, generator=g) < frac_static
    static0 = (_STATIC_MEAN + _STATIC_STD * torch.randn(n, generator=g)).clamp(min=0.005)
    moving0 = (_MOVING_MEAN + _MOVING_STD * torch.randn(n, generator=g)).clamp(*_MOVING_CLIP)
    scores = torch.empty(frames, n)
    scores[0] = torch.where(is_static, static0, moving0)
    for f in range(1, frames):
        jitter = _STATIC_JITTER * torch.randn(n, generator=g)
        walk = _MOVING_WALK * torch.randn(n, generator=g)
        scores[f] = torch.where(is_static, (scores[f - 1] + jitter).clamp(min=0.0),
                                (scores[f - 1] + walk).clamp(*_MOVING_CLIP))
    # Q, then K0, V0, then per frame K and V drift scaled by the tile's motion
    per_token = torch.repeat_interleave(scores, counts, dim=1)
    q = torch.randn(frames, tokens, hidden, generator=g)
    k = torch.empty(frames, tokens, hidden)
    v = torch.empty(frames, tokens, hidden)
    k[0] = torch.randn(tokens, hidden, generator=g)
    v[0] = torch.randn(tokens, hidden, generator=g)
    for f in range(1, frames):
        scale = _KV_DRIFT * per_token[f].unsqueeze(1)
        k[f] = k[f - 1] + scale * torch.randn(tokens, hidden, generator=g)
        v[f] = v[f - 1] + scale * torch.randn(tokens, hidden, generator=g)
    return scores.numpy(), is_static.numpy(), q.numpy(), k.numpy(), v.numpy()


def reuse_flags(scores: np.ndarray, percentile: float = 50.0) -> np.ndarray:
    """The CSV reuse column from per-tile change rates [frames][tiles]:
    1 where the rate is below the `percentile`-th percentile of frames 1..F-1
    (linear interpolation), frame 0 always 0 (written fresh).  The rule of
    traces/gen_motion_from_video.py:118-122, whose motion_score is that
    change rate."""
    s = np.asarray(scores, dtype=np.float64)
    reuse = np.zeros(s.shape, dtype=np.int8)
    if s.shape[0] > 1:
        tau = float(np.percentile(s[1:], percentile))
        reuse[1:] = (s[1:] < tau).astype(np.int8)
    return reuse


def write_motion_csv(path, scores: np.ndarray, is_static=None, tokens: int = TOKENS,
                     tile_tokens: int = TILE, reuse=None) -> Path:
    """Reference trace CSV; with `reuse` ([frames][tiles]) the optional 7th
    column of traces/gen_motion_from_video.py is written too."""
    scores = np.asarray(scores, dtype=np.float32)
    frames, n = scores.shape
    counts = tile_counts(tokens, tile_tokens)
    starts = np.cumsum(counts) - counts
    if is_static is None:
        is_static = np.zeros(n, dtype=bool)
    head = "frame_id,tile_id,motion_score,is_static,token_start,token_count"
    lines = [head + (",reuse" if reuse is not None else "")]
    for f in range(frames):
        for t in range(n):
            row = (f"{f},{t},{float(scores[f, t]):.6f},{int(is_static[t])},"
                   f"{int(starts[t])},{int(counts[t])}")
            if reuse is not None:
                row += f",{int(reuse[f][t])}"
            lines.append(row)
    p = Path(path)
    p.write_text("\n".join(lines) + "\n")
    return p


def read_motion_csv(path, frames: int, num_tiles: int, with_reuse: bool = False):
    """Scores exactly as the reference parses them (sscanf %f), via the C ABI;
    with_reuse also returns the reuse column (int8, 0 where absent)."""
    from ._lib import lib
    s = np.zeros((frames, num_tiles), dtype=np.float32)
    r = np.zeros((frames, num_tiles), dtype=np.int8)
    n = lib().kvp_read_motion_csv(str(path).encode(), frames, num_tiles, s.ctypes.data,
                                  r.ctypes.data if with_reuse else None)
    if n < 0:
        raise FileNotFoundError(path)
    return (s, r) if with_reuse else s


def csv_round_trip(scores: np.ndarray, workdir) -> np.ndarray:
    """Scores after the CSV text round trip the reference driver applies."""
    p = Path(workdir) / "motion_trace.csv"
    write_motion_csv(p, scores)
    return read_motion_csv(p, *np.asarray(scores).shape)


# ---------------------------------------------------------------- benchmark configs
def motion_config1(seed: int = 0, tiles: int = 98) -> np.ndarray:
    """Config 1: one frame, U[0,1) per tile."""
    g = torch.Generator().manual_seed(seed)
    return torch.rand(1, tiles, generator=g).numpy()


def motion_config2(frames: int = 8, seed: int = 0, tiles: int = 98, rho: float = 0.9,
                   sigma: float = 0.1) -> np.ndarray:
    """Config 2: AR(1) per tile, m_0 ~ U[0,1), m_f = clamp(rho m_{f-1} + N(0, sigma^2), 0, 1)."""
    g = torch.Generator().manual_seed(seed)
    m = torch.empty(frames, tiles)
    m[0] = torch.rand(tiles, generator=g)
    for f in range(1, frames):
        m[f] = (rho * m[f - 1] + sigma * torch.randn(tiles, generator=g)).clamp(0.0, 1.0)
    return m.numpy()


def motion_config3(frames: int = 50, seed: int = 0, tiles: int = 98, blob_frac: float = 0.2):
    """Config 3: background U[0,0.1); a blob of round(0.2*tiles) consecutive
    tile ids with motion U[0.9,1.0] starting at tile f (mod tiles): it
    translates one tile per frame."""
    g = torch.Generator().manual_seed(seed)
    m = 0.1 * torch.rand(frames, tiles, generator=g)
    blob = int(round(blob_frac * tiles))
    hot = 0.9 + 0.1 * torch.rand(frames, blob, generator=g)
    for f in range(frames):
        idx = (torch.arange(blob) + f) % tiles
        m[f, idx] = hot[f]
    return m.numpy()


def motion_config4(frames: int = 21, seed: int = 0, tiles: int = 98) -> np.ndarray:
    """Config 4 (no motion model given): U[0,1) per tile and frame."""
    g = torch.Generator().manual_seed(seed)
    return torch.rand(frames, tiles, generator=g).numpy()


def motion_config5(regime: str, frames: int = 16, seed: int = 0, tiles: int = 98) -> np.ndarray:
    """Config 5: 'static' U[0,0.05) or 'high' U[0,1) i.i.d. per tile and frame."""
    g = torch.Generator().manual_seed(seed)
    u = torch.rand(frames, tiles, generator=g)
    return (0.05 * u if regime == "static" else u).numpy()


def qkv(rows: int, hidden: int = HIDDEN, *, seed: int = 0, dtype=torch.bfloat16,
        device="cpu", head_dim: int = HEAD_DIM):
    """Q, K, V ~ N(0,1)/sqrt(head_dim), [rows, hidden], from one generator on
    `device` (drawn in fp32, then cast)."""
    g = torch.Generator(device=device).manual_seed(seed)
    s = 1.0 / math.sqrt(head_dim)
    out = []
    for _ in range(3):
        t = torch.randn(rows, hidden, generator=g, device=device, dtype=torch.float32) * s
        out.append(t.to(dtype))
    return tuple(out)


def hold_reused_tiles(k: torch.Tensor, v: torch.Tensor, reuse: np.ndarray, *, tokens: int = TOKENS,
                      tile_tokens: int = TILE) -> None:
    """In place: the rows of every tile flagged unchanged in frame f (reuse
    [frames][tiles] == 1) become copies of frame f-1's rows, i.e. K/V as a
    model that skips recomputing static tiles would hold them."""
    frames, nt = np.asarray(reuse).shape
    for f in range(1, frames):
        for t in np.nonzero(np.asarray(reuse)[f])[0]:
            a = f * tokens + int(t) * tile_tokens
            b = min(a + tile_tokens, (f + 1) * tokens)
            k[a:b] = k[a - tokens:b - tokens]
            v[a:b] = v[a - tokens:b - tokens]


# ------------------------------------------------------------ synthetic video
VIDEO_H, VIDEO_W = 480, 832      # the reference's frame size (30 x 52 cells of 16 px)


def synthetic_video(frames: int = 8, *, seed: int = 0, height: int = VIDEO_H, width: int = VIDEO_W,
                    pan=(0.7, 0.3), zoom: float = 0.004, rot: float = 0.002, blobs: int = 6,
                    noise: float = 1.0) -> np.ndarray:
    """Seeded grayscale clip, uint8 [frames, height, width]: a smooth random
    texture under a camera motion (pan by `pan` pixels, zoom by `zoom` and
    rotation by `rot` radians per frame about the centre: displacements grow
    from the centre outwards, so per-tile motion is spread out), plus `blobs`
    textured discs each moving on its own straight path at 1-6 px/frame,
    plus N(0, noise) sensor noise; sub-pixel sampling is bilinear.  Stands
    in for the DAVIS clip the reference's traces/gen_motion_from_video.py
    reads, which is not available here."""
    rng = np.random.default_rng(seed)

    def texture(h, w, scale):
        # band-limited noise: white noise blurred by a separable box cascade
        t = rng.standard_normal((h + 64, w + 64)).astype(np.float32)
        for _ in range(3):
            t = (np.cumsum(np.cumsum(t, 0), 1))
            t = (t[scale:, scale:] - t[:-scale, scale:] - t[scale:, :-scale] + t[:-scale, :-scale])
            t /= scale * scale
        t = t[:h, :w]
        return (t - t.mean()) / (t.std() + 1e-6)

    H2, W2 = height + 64, width + 64
    bg = 0.6 * texture(H2, W2, 9) + 0.4 * texture(H2, W2, 3)
    yy, xx = np.mgrid[0:height, 0:width].astype(np.float32)

    def sample(img, x, y):
        x0 = np.floor(x).astype(np.int64)
        y0 = np.floor(y).astype(np.int64)
        fx, fy = x - x0, y - y0
        x0 = np.clip(x0, 0, img.shape[1] - 2)
        y0 = np.clip(y0, 0, img.shape[0] - 2)
        return ((1 - fx) * (1 - fy) * img[y0, x0] + fx * (1 - fy) * img[y0, x0 + 1] +
                (1 - fx) * fy * img[y0 + 1, x0] + fx * fy * img[y0 + 1, x0 + 1])

    specs = []
    for _ in range(blobs):
        r = rng.uniform(25, 70)
        c = (rng.uniform(r, width - r), rng.uniform(r, height - r))
        ang = rng.uniform(0, 2 * np.pi)
        spd = rng.uniform(1.0, 6.0)
        tex = texture(int(2 * r) + 8, int(2 * r) + 8, 4)
        specs.append((r, c, (spd * np.cos(ang), spd * np.sin(ang)), tex, rng.uniform(-1.5, 1.5)))
    out = np.empty((frames, height, width), np.uint8)
    cx0, cy0 = width / 2.0, height / 2.0
    for f in range(frames):
        sc = (1.0 + zoom) ** (-f)
        ca, sa = np.cos(-rot * f) * sc, np.sin(-rot * f) * sc
        ux, uy = xx - cx0, yy - cy0
        img = sample(bg, cx0 + ca * ux - sa * uy + 32 + pan[0] * f,
                     cy0 + sa * ux + ca * uy + 32 + pan[1] * f)
        for r, c, v, tex, off in specs:
            cx, cy = c[0] + v[0] * f, c[1] + v[1] * f
            m = (xx - cx) ** 2 + (yy - cy) ** 2 < r * r
            if m.any():
                tx = np.clip(xx[m] - cx + r + 4, 0, tex.shape[1] - 1.001)
                ty = np.clip(yy[m] - cy + r + 4, 0, tex.shape[0] - 1.001)
                img[m] = sample(tex, tx, ty) + off
        img = 128 + 40 * img + noise * rng.standard_normal(img.shape)
        out[f] = np.clip(np.rint(img), 0, 255).astype(np.uint8)
    return out


def write_driver_inputs(directory, frames: int, tokens: int = TOKENS, hidden: int = HIDDEN,
                        seed: int = 0) -> Path:
    """Q/K/V of `frames` frames in the files the reference's driver reads
    (src/run_policy_experiment.cu:32-43, 120-122): raw fp32
    [frames*tokens][hidden] in q.bin, k.bin, v.bin, drawn as `qkv(...,
    dtype=float32)`."""
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    for name, t in zip(("q", "k", "v"), qkv(frames * tokens, hidden, seed=seed, dtype=torch.float32)):
        t.numpy().tofile(d / f"{name}.bin")
    return d


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser(description="write the reference driver's Q/K/V input files")
    ap.add_argument("command", choices=["driver-inputs"])
    ap.add_argument("directory")
    ap.add_argument("--frames", type=int, default=8)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args()
    print(write_driver_inputs(a.directory, a.frames, seed=a.seed))
