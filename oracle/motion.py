"""CPU restatement of the reference's motion-trace producer
(traces/gen_motion_from_video.py): dense optical flow between consecutive
frames, per-pixel magnitude, 16 x 16-pixel cell means over the 30 x 52
latent grid (:61-67), means over row-major 16-token tiles (:108-114),
change[0] = change[1] (:117), the percentile-50 reuse threshold (:119-121).

TEST INFRASTRUCTURE ONLY: the checker of the GPU motion producer and the
CPU baseline of its bench leg, never the product path.

The flow is Farnebaeck's two-frame method (G. Farnebaeck, "Two-Frame Motion
Estimation Based on Polynomial Expansion", SCIA 2003), which the reference
calls through OpenCV (cv2.calcOpticalFlowFarneback, pinned at 5.0.0.93 by
scripts/setup_env.sh; 4.13.0 in this image) with pyr_scale 0.5, levels 3,
winsize 15, iterations 3, poly_n 5, poly_sigma 1.2, flags 0 (:103-105).
It is restated here from the paper, with these choices:
  * polynomial expansion: Gaussian applicability (sigma, 2n+1 taps),
    separable correlations with {1, x, x^2}, the closed-form solve of the
    decoupled normal equations; mirrored borders;
  * displacement: A = (A1(x) + A2(x~)) / 2,
    db = -(b2(x~) - b1(x)) / 2 + A d~, with x~ = x + d~ and R2 sampled
    bilinearly (clamped to the image); G = A^T A and h = A^T db averaged
    over a winsize x winsize box (mirrored borders); d = G^-1 h;
    `iterations` updates per level;
  * pyramid: `levels` + 1 layers at scales 0.5^k, each the full-resolution
    frame blurred (Gaussian, sigma = (1/scale - 1)/2) and resized
    bilinearly (half-pixel centres); the coarser flow is resized the same
    way and scaled by 2.
Parity with OpenCV is by tolerance (tests/test_motion_host.py); the GPU
kernels (csrc/motion_sm100.cu) follow this file step by step.
"""

from __future__ import annotations

import math

import numpy as np
from scipy.ndimage import correlate1d

FARNEBACK = dict(pyr_scale=0.5, levels=3, winsize=15, iterations=3, poly_n=5, poly_sigma=1.2)
GRID = (30, 52)          # latent grid rows, cols (configs/grounding_config.json)
TILE_TOKENS = 16
TOKENS = GRID[0] * GRID[1]


def gaussian_taps(n: int, sigma: float) -> np.ndarray:
    """Normalised Gaussian weights at offsets -n..n."""
    x = np.arange(-n, n + 1, dtype=np.float64)
    g = np.exp(-x * x / (2.0 * sigma * sigma))
    return g / g.sum()


def poly_consts(n: int, sigma: float):
    """Taps k0 = g, k1 = g*x, k2 = g*x^2 and the solve constants: rx = cx*ix,
    ry = cy*ix, rxy = cxy*ixy, rxx = a*c1 + b*cxx + c*cyy (ryy symmetric)."""
    x = np.arange(-n, n + 1, dtype=np.float64)
    g = gaussian_taps(n, sigma)
    m0, m2, m4 = g.sum(), (g * x * x).sum(), (g * x ** 4).sum()
    G = np.array([[m0 * m0, m0 * m2, m0 * m2],
                  [m0 * m2, m0 * m4, m2 * m2],
                  [m0 * m2, m2 * m2, m0 * m4]])
    Gi = np.linalg.inv(G)
    return (g, g * x, g * x * x), dict(ix=1.0 / (m0 * m2), ixy=1.0 / (m2 * m2), a=Gi[1, 0],
                                       b=Gi[1, 1], c=Gi[1, 2])


def poly_exp(img: np.ndarray, n: int = 2, sigma: float = 1.2) -> np.ndarray:
    """Local quadratic model f(p + x) ~ x^T A x + b^T x + c per pixel.
    Returns float32 [5, H, W] = (bx, by, Axx, Ayy, Axy) with
    A = [[Axx, Axy], [Axy, Ayy]] (Axy = rxy / 2)."""
    (k0, k1, k2), C = poly_consts(n, sigma)
    f = img.astype(np.float32)
    v0 = correlate1d(f, k0.astype(np.float32), axis=0, mode="mirror")
    v1 = correlate1d(f, k1.astype(np.float32), axis=0, mode="mirror")
    v2 = correlate1d(f, k2.astype(np.float32), axis=0, mode="mirror")
    c1 = correlate1d(v0, k0.astype(np.float32), axis=1, mode="mirror")
    cx = correlate1d(v0, k1.astype(np.float32), axis=1, mode="mirror")
    cxx = correlate1d(v0, k2.astype(np.float32), axis=1, mode="mirror")
    cy = correlate1d(v1, k0.astype(np.float32), axis=1, mode="mirror")
    cxy = correlate1d(v1, k1.astype(np.float32), axis=1, mode="mirror")
    cyy = correlate1d(v2, k0.astype(np.float32), axis=1, mode="mirror")
    a, b, c = (np.float32(C[k]) for k in ("a", "b", "c"))
    out = np.empty((5,) + f.shape, np.float32)
    out[0] = cx * np.float32(C["ix"])
    out[1] = cy * np.float32(C["ix"])
    out[2] = a * c1 + b * cxx + c * cyy
    out[3] = a * c1 + c * cxx + b * cyy
    out[4] = cxy * np.float32(C["ixy"] * 0.5)
    return out


def bilinear(img: np.ndarray, x: np.ndarray, y: np.ndarray) -> np.ndarray:
    """img sampled at (x, y), coordinates clamped to [0, W-1] x [0, H-1]."""
    H, W = img.shape[-2:]
    x = np.clip(x, 0, W - 1).astype(np.float32)
    y = np.clip(y, 0, H - 1).astype(np.float32)
    x0 = np.minimum(np.floor(x).astype(np.int64), W - 2)
    y0 = np.minimum(np.floor(y).astype(np.int64), H - 2)
    fx, fy = x - x0, y - y0
    return ((1 - fy) * ((1 - fx) * img[..., y0, x0] + fx * img[..., y0, x0 + 1]) +
            fy * ((1 - fx) * img[..., y0 + 1, x0] + fx * img[..., y0 + 1, x0 + 1])).astype(np.float32)


def resize_bilinear(img: np.ndarray, h: int, w: int) -> np.ndarray:
    """Half-pixel-centre bilinear resize of [..., H, W] to [..., h, w]."""
    H, W = img.shape[-2:]
    ys = (np.arange(h, dtype=np.float32) + 0.5) * np.float32(H / h) - 0.5
    xs = (np.arange(w, dtype=np.float32) + 0.5) * np.float32(W / w) - 0.5
    yy, xx = np.meshgrid(ys, xs, indexing="ij")
    return bilinear(img, xx, yy)


def gaussian_blur(img: np.ndarray, sigma: float) -> np.ndarray:
    """Separable Gaussian blur, round(sigma*5)|1 taps (at least 3), mirrored."""
    ks = max(3, int(round(sigma * 5)) | 1)
    g = gaussian_taps(ks // 2, sigma).astype(np.float32)
    t = correlate1d(img.astype(np.float32), g, axis=0, mode="mirror")
    return correlate1d(t, g, axis=1, mode="mirror")


def pyramid_sizes(H: int, W: int, levels: int, pyr_scale: float):
    return [(int(round(H * pyr_scale ** k)), int(round(W * pyr_scale ** k))) for k in range(levels + 1)]


def pyramid(img: np.ndarray, levels: int, pyr_scale: float):
    """Layers finest first: the frame itself, then blurred + resized copies."""
    f = img.astype(np.float32)
    out = [f]
    for k, (h, w) in enumerate(pyramid_sizes(*f.shape, levels, pyr_scale)[1:], start=1):
        sigma = (1.0 / pyr_scale ** k - 1.0) * 0.5
        out.append(resize_bilinear(gaussian_blur(f, sigma), h, w))
    return out


def update_matrices(R1: np.ndarray, R2: np.ndarray, flow: np.ndarray) -> np.ndarray:
    """[5, H, W] = (G11, G12, G22, h1, h2): G = A^T A, h = A^T db."""
    H, W = R1.shape[1:]
    yy, xx = np.mgrid[0:H, 0:W].astype(np.float32)
    dx, dy = flow[0], flow[1]
    R2s = bilinear(R2, xx + dx, yy + dy)
    a11 = (R1[2] + R2s[2]) * np.float32(0.5)
    a22 = (R1[3] + R2s[3]) * np.float32(0.5)
    a12 = (R1[4] + R2s[4]) * np.float32(0.5)
    db1 = (R1[0] - R2s[0]) * np.float32(0.5) + a11 * dx + a12 * dy
    db2 = (R1[1] - R2s[1]) * np.float32(0.5) + a12 * dx + a22 * dy
    M = np.empty((5, H, W), np.float32)
    M[0] = a11 * a11 + a12 * a12
    M[1] = a12 * (a11 + a22)
    M[2] = a12 * a12 + a22 * a22
    M[3] = a11 * db1 + a12 * db2
    M[4] = a12 * db1 + a22 * db2
    return M


def box_mean(M: np.ndarray, win: int) -> np.ndarray:
    k = np.full(win, 1.0 / win, np.float32)
    t = correlate1d(M, k, axis=-2, mode="mirror")
    return correlate1d(t, k, axis=-1, mode="mirror")


def solve_flow(Mb: np.ndarray) -> np.ndarray:
    g11, g12, g22, h1, h2 = Mb
    det = g11 * g22 - g12 * g12
    idet = np.float32(1.0) / (det + np.float32(1e-3))
    return np.stack([(g22 * h1 - g12 * h2) * idet, (g11 * h2 - g12 * h1) * idet]).astype(np.float32)


def farneback(prev: np.ndarray, nxt: np.ndarray, *, pyr_scale=0.5, levels=3, winsize=15,
              iterations=3, poly_n=5, poly_sigma=1.2) -> np.ndarray:
    """Flow [2, H, W] (dx, dy) with nxt(x + d) ~ prev(x)."""
    P1 = pyramid(prev, levels, pyr_scale)
    P2 = pyramid(nxt, levels, pyr_scale)
    flow = None
    for k in range(levels, -1, -1):
        h, w = P1[k].shape
        flow = np.zeros((2, h, w), np.float32) if flow is None else \
            resize_bilinear(flow, h, w) * np.float32(1.0 / pyr_scale)
        R1 = poly_exp(P1[k], poly_n // 2, poly_sigma)
        R2 = poly_exp(P2[k], poly_n // 2, poly_sigma)
        M = update_matrices(R1, R2, flow)
        for it in range(iterations):
            flow = solve_flow(box_mean(M, winsize))
            if it < iterations - 1:
                M = update_matrices(R1, R2, flow)
    return flow


def cell_means(mag: np.ndarray, grid=GRID) -> np.ndarray:
    """Mean over each (H/rows) x (W/cols) cell (:61-67)."""
    rows, cols = grid
    H, W = mag.shape
    ch, cw = H // rows, W // cols
    return mag[:rows * ch, :cols * cw].reshape(rows, ch, cols, cw).mean(axis=(1, 3))


def tile_means(cells: np.ndarray, tile_tokens: int = TILE_TOKENS) -> np.ndarray:
    """Means over row-major runs of tile_tokens cells, the last run shorter (:108-114)."""
    flat = cells.reshape(-1)
    n = flat.size
    nt = (n + tile_tokens - 1) // tile_tokens
    starts = np.arange(nt) * tile_tokens
    counts = np.minimum(tile_tokens, n - starts)
    return np.add.reduceat(flat, starts) / counts


def trace_from_flows(mags, percentile: float = 50.0):
    """change [F][tiles] (frame 0 copies frame 1), tau, reuse, is_static from
    the F-1 flow magnitudes of consecutive pairs (:101-121, :146-151)."""
    F = len(mags) + 1
    change = np.zeros((F, (TOKENS + TILE_TOKENS - 1) // TILE_TOKENS), np.float64)
    for f, m in enumerate(mags, start=1):
        change[f] = tile_means(cell_means(np.asarray(m, np.float64)))
    change[0] = change[1]
    tau = float(np.percentile(change[1:], percentile))
    reuse = (change < tau).astype(np.int8)
    reuse[0] = 0
    is_static = (change < tau).astype(np.int8)
    return change, tau, reuse, is_static


def motion_trace(frames: np.ndarray, percentile: float = 50.0, **fb):
    """The whole producer on a clip [F, H, W] uint8."""
    params = dict(FARNEBACK, **fb)
    mags = []
    for f in range(1, len(frames)):
        fl = farneback(frames[f - 1], frames[f], **params)
        mags.append(np.sqrt(fl[0] * fl[0] + fl[1] * fl[1]))
    return trace_from_flows(mags, percentile)
