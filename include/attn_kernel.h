/* libkvp.so: reference-compatible FP32 attention entry points.
 *
 * Drop-in for GauthamMK-0/cuda-kv-persistence src/attn_kernel.h:15-29
 * (same names, arguments and semantics; C linkage here so any FFI can bind
 * them).  Q/K/V/Out are [rows][D] fp32, D = heads * 128, head h in columns
 * [h*128, h*128+128).  Key row j is read from Arena row KVMap[j] (K half,
 * then V half at +D; row stride 2*D floats) when KVMap[j] >= 0, else from
 * K/V.  Launches go to the legacy default stream, as in the reference, and
 * are stream-ordered after any staging copies queued by kvtm_* calls.
 * Only head_dim 128 is supported (the reference hard-wires it too).
 */
#ifndef KVP_ATTN_KERNEL_H
#define KVP_ATTN_KERNEL_H

#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif

/* src/attn_kernel.h:15-19 / src/gated_attention_kernel.cu:141-168.
 * remap=false: one launch over all frames, frame f attends to itself, no
 * map.  remap=true: per-frame intra launches with KVMap pre-offset by f*T. */
void attn_forward_launcher(const float* d_q, const float* d_k, const float* d_v,
                           const float* d_arena, const long* d_kvmap, float* d_out, int frames,
                           int T, int D, int heads, bool remap);

/* src/attn_kernel.h:25-29 / src/gated_attention_kernel.cu:170-184.
 * cross=0: d_k/d_v/d_kvmap_f pre-offset to the frame, keys [0, T).
 * cross=1: d_k/d_v/d_kvmap_f at buffer bases, keys [0, (frame_idx+1)*T). */
void attn_forward_single_frame(const float* d_q_f, const float* d_k, const float* d_v,
                               const float* d_arena, const long* d_kvmap_f, float* d_out_f,
                               int T, int D, int heads, int cross, int frame_idx);

#define ATTENTION_KTILE 64 /* keys per shared-memory tile (src/attn_kernel.h:31) */

#ifdef __cplusplus
}
#endif
#endif
