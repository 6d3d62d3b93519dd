"""kvp: B200-native remapped attention with KV-tile persistence.

Host-side mirror of GauthamMK-0/cuda-kv-persistence's interface for the
remapped attention path, over the C ABI of libkvp.so (include/*.h):

* ``KVTileManager``      -- src/kv_tile_manager.h:21-90 (kvtm_* facade)
* ``select`` / policies  -- src/tile_gating_policy.h:8-68
* ``TileLayout``         -- src/tile_layout.h:13-31
* ``Session``            -- the per-frame KVMap loop of src/run_policy_experiment.cu:156-274
* ``attn_forward_single_frame`` / ``attn_forward_launcher`` -- src/attn_kernel.h:15-29 (fp32)
* ``attn_bf16``          -- the tcgen05 kernel (sm_100a)

PyTorch tensors are used only as device memory and streams.
"""

from ._lib import KvpError, lib  # noqa: F401
from .layout import TileLayout  # noqa: F401
from .manager import KVTileManager, KVTM_ADMITTED, KVTM_INVALID, KVTM_REFUSED_BUDGET  # noqa: F401
from .policies import POLICIES, select  # noqa: F401
from .session import Session  # noqa: F401
