// BF16 tcgen05 remapped attention (csrc/attn_sm100.cu): descriptors and launcher.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "kvp_common.h"

namespace kvp {

// One layer's buffers.  Q/K/V/Out are bf16 [rows][D] (head h at columns
// [h*128, h*128+128)); the arena is bf16 [arena_rows][2*D] (K half, V half);
// kvmap (int64, may be null) is indexed by the absolute key row.
struct LayerIO {
    const void* q;
    const void* k;
    const void* v;
    void* out;
    const void* arena;
    const long long* kvmap;
    long long q_rows, kv_rows, arena_rows;
};

// Which query rows attend to which key rows.
//   query frames [q_frame0, q_frame0 + frames) of `tokens` rows each;
//   mode 0 (intra): frame f's keys are rows [f*T, (f+1)*T);
//   mode 1 (causal): frame f's keys are rows [b*T, (f+1)*T) with
//        b = window ? max(0, f-window+1) : 0;
//   flat = 1 (causal, no window): query tiles run across frame
//        boundaries, each row masked at its own frame's limit (no padding
//        work at the 1560 = 12*128 + 24 frame tail).
struct AttnDesc {
    int tokens;
    int frames;
    int q_frame0;
    int mode;
    int window;
    int heads;
    int head_dim;   // must be 128
    int head0;
    int nheads;
    int flat;
};

// Per-frame (non-flat) launches whose CTAs would not fill the SMs split each
// query tile pair's key range over several CTAs and merge their partial
// (O, max, sum) with a second kernel; the fp32 workspace is stream-ordered
// (a private memory pool that keeps its blocks cached).  allow_split = false
// (callers that may not allocate) always runs one CTA per pair.
int launch_attn_bf16(const LayerIO& io, const AttnDesc& d, int* d_status, cudaStream_t stream,
                     bool allow_split = true);

// Several layers (or head chunks) of the same shape in one launch: ios[i]
// and ds[i] as for launch_attn_bf16; every ds[i] has the same tokens,
// frames, mode, window and flat tiling, and may differ in heads, head0,
// nheads and q_frame0 (e.g. consecutive frames of one layer, each with the
// KVMap and arena its admission step produced).  One grid over all their CTAs, so the ramp-down of a
// short chunk overlaps the next chunk's work; no key-range split.
int launch_attn_bf16_multi(const LayerIO* ios, const AttnDesc* ds, int n, int* d_status,
                           cudaStream_t stream);
// Layers one launch of launch_attn_bf16_multi takes (more are spread evenly
// over several launches).
constexpr int kAttnSegsPerLaunch = 12;

// The launcher's argument checks alone (descriptor, row coverage, 16-byte
// alignment), touching no device state: KVP_OK or KVP_ERR_ARG with a message.
int check_attn_bf16(const LayerIO& io, const AttnDesc& d);

// 2D TMA map of a bf16 row-major tensor [rows][cols] (row pitch `pitch`
// elements), box 64 columns x box_rows rows, 128B swizzle.  Encoded maps are
// cached by (base, shape, pitch, box).
int make_bf16_tensor_map(CUtensorMap* m, const void* base, long long rows, long long cols,
                         long long pitch, uint32_t box_rows);

// A kernel whose bounded mbarrier wait cannot complete: records
// KVP_STATUS_TIMEOUT after limit_ns (<= 5 s).  For tests of the timeout path.
int launch_bounded_wait_probe(long long limit_ns, int* d_status, cudaStream_t stream);

}  // namespace kvp
