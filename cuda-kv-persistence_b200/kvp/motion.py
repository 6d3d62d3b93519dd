"""GPU motion-trace producer (kvp_motion_*): the reference's
traces/gen_motion_from_video.py with the optical flow on the device.  Fails
loudly without libkvp.so."""

from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import KvpError, MotionParams, check, lib

REFERENCE_FLOW = dict(pyr_scale=0.5, levels=3, winsize=15, iterations=3, poly_n=5, poly_sigma=1.2)


class MotionProducer:
    """Flow and per-tile change rates for clips of height x width uint8
    frames (the reference: 480 x 832, a 30 x 52 grid of 16-pixel cells,
    16-cell tiles)."""

    def __init__(self, height: int = 480, width: int = 832, *, grid=(30, 52), tile_cells: int = 16,
                 **flow):
        f = dict(REFERENCE_FLOW, **flow)
        self.params = MotionParams(height, width, f["levels"], f["winsize"], f["iterations"],
                                   f["poly_n"], f["poly_sigma"], f["pyr_scale"], grid[0], grid[1],
                                   tile_cells)
        self._L = lib()
        self.h = self._L.kvp_motion_create(C.byref(self.params))
        if not self.h:
            raise KvpError("kvp_motion_create failed: " + self._L.kvp_last_error().decode())
        self.height, self.width = height, width
        self.tiles = int(self._L.kvp_motion_tiles(self.h))

    def close(self):
        if getattr(self, "h", None):
            self._L.kvp_motion_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def flow(self, prev, nxt, out, stream: int = 0) -> None:
        """out fp32 [2, H, W] (dx, dy) for two uint8 [H, W] device frames."""
        check(self._L.kvp_motion_flow(self.h, C.c_void_p(prev.data_ptr()), C.c_void_p(nxt.data_ptr()),
                                      C.c_void_p(out.data_ptr()), C.c_void_p(stream)), "motion_flow")

    def change(self, frames, out, stream: int = 0) -> None:
        """out fp32 [F, tiles] from uint8 [F, H, W] device frames."""
        check(self._L.kvp_motion_trace(self.h, C.c_void_p(frames.data_ptr()), frames.shape[0],
                                       C.c_void_p(out.data_ptr()), C.c_void_p(stream)), "motion_trace")


def threshold(change: np.ndarray, percentile: float = 50.0):
    """(tau, reuse int8, is_static int8) from host change rates [F, tiles]."""
    ch = np.ascontiguousarray(change, dtype=np.float32)
    F, T = ch.shape
    reuse = np.zeros((F, T), np.int8)
    static = np.zeros((F, T), np.int8)
    tau = C.c_double(0.0)
    check(lib().kvp_motion_threshold(ch.ctypes.data, F, T, percentile, reuse.ctypes.data,
                                     static.ctypes.data, C.byref(tau)), "motion_threshold")
    return float(tau.value), reuse, static
