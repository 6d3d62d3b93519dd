"""KVTileManager over the kvtm_* C ABI (src/kv_tile_manager.h:21-90).

Method names, arguments and results follow the reference class; device
pointers are plain integers (e.g. ``tensor.data_ptr()``).
"""

from __future__ import annotations

import ctypes as C

from ._lib import KvpError, lib

KVTM_ADMITTED, KVTM_REFUSED_BUDGET, KVTM_INVALID = 1, 0, -1
KVTM_FLAG_DRY_RUN = 1


class KVTileManager:
    def __init__(self, budget_bytes: int, max_window_bytes: int, *, dry_run: bool = False,
                 stream: int | None = None):
        L = lib()
        self._L = L
        self.h = (L.kvtm_create_ex(budget_bytes, max_window_bytes, KVTM_FLAG_DRY_RUN)
                  if dry_run else L.kvtm_create(budget_bytes, max_window_bytes))
        if not self.h:
            raise KvpError("kvtm_create failed")
        if stream is not None:
            L.kvtm_set_stream(self.h, C.c_void_p(stream))

    def close(self):
        if getattr(self, "h", None):
            self._L.kvtm_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    # per-tile admission
    def init(self) -> bool: return self._L.kvtm_init(self.h) == 1
    def query_device_limit(self) -> int: return self._L.kvtm_query_limit(self.h)
    def admit(self, tile_id: int, ptr: int, nbytes: int) -> int:
        return self._L.kvtm_admit(self.h, tile_id, C.c_void_p(ptr), nbytes)
    def release(self, tile_id: int) -> bool: return self._L.kvtm_release(self.h, tile_id) == 1
    def clear(self): self._L.kvtm_clear(self.h)
    def persisted_bytes(self) -> int: return self._L.kvtm_persisted_bytes(self.h)
    def persisted_tiles(self) -> int: return self._L.kvtm_persisted_tiles(self.h)

    # arena mode
    def arena_init(self, capacity_bytes: int, row_stride_floats: int) -> bool:
        return self._L.kvtm_arena_init(self.h, capacity_bytes, row_stride_floats) == 1
    def arena_begin_step(self): self._L.kvtm_arena_begin(self.h)
    def arena_stage(self, k_ptr: int, k_bytes: int, v_ptr: int, v_bytes: int):
        row = C.c_long(-1)
        ok = self._L.kvtm_arena_stage(self.h, C.c_void_p(k_ptr), k_bytes, C.c_void_p(v_ptr),
                                      v_bytes, C.byref(row))
        return ok == 1, row.value
    def arena_apply_window(self) -> bool: return self._L.kvtm_arena_window(self.h) == 1
    def arena_end_step(self): self._L.kvtm_arena_end(self.h)
    def arena_used_bytes(self) -> int: return self._L.kvtm_arena_used(self.h)
    def arena_device_ptr(self) -> int: return self._L.kvtm_arena_ptr(self.h) or 0

    # streaming mode
    def streaming_begin(self) -> bool: return self._L.kvtm_streaming_begin(self.h) == 1
    def streaming_stage(self, row_id: int, k_ptr: int, k_bytes: int, v_ptr: int, v_bytes: int,
                        changed: bool = False):
        slot, rs = C.c_long(-1), C.c_int(0)
        ok = self._L.kvtm_streaming_stage(self.h, row_id, C.c_void_p(k_ptr), k_bytes,
                                          C.c_void_p(v_ptr), v_bytes, int(changed),
                                          C.byref(slot), C.byref(rs))
        return ok == 1, slot.value, bool(rs.value)
    def streaming_release(self, row_id: int) -> bool:
        return self._L.kvtm_streaming_release(self.h, row_id) == 1
    def streaming_apply_window(self) -> bool: return self._L.kvtm_streaming_window(self.h) == 1
    def streaming_end(self): self._L.kvtm_streaming_end(self.h)
    def streaming_staged_bytes(self) -> int: return self._L.kvtm_streaming_staged_bytes(self.h)

    # additions
    def flush(self) -> int: return self._L.kvtm_flush(self.h)
    def pending_copies(self) -> int: return self._L.kvtm_pending_copies(self.h)
    def window_log(self):
        n = self._L.kvtm_window_log(self.h, None, None, 0)
        b = (C.c_long * max(n, 1))()
        p = (C.c_int * max(n, 1))()
        self._L.kvtm_window_log(self.h, b, p, n)
        return [(b[i], p[i]) for i in range(n)]
    def reset_calls(self) -> int: return self._L.kvtm_reset_calls(self.h)
