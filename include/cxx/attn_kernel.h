/* libkvp.so: the reference's attention entry points with C++ linkage, for
 * callers compiled against the reference's C++ interface.
 *
 * Drop-in for GauthamMK-0/cuda-kv-persistence src/attn_kernel.h:15-32.  The
 * same functions are also exported with C linkage (attn_kernel.h one
 * directory up) for FFI callers; both run this library's fp32 remapped
 * attention kernel on the legacy default stream, after any staging copies a
 * KVTileManager has queued.  Q/K/V/Out are [rows][D] fp32, D = heads * 128.
 */
#ifndef KVP_CXX_ATTN_KERNEL_H
#define KVP_CXX_ATTN_KERNEL_H

/* src/attn_kernel.h:15-19 */
__attribute__((visibility("default")))
void attn_forward_launcher(const float* d_q, const float* d_k, const float* d_v,
                           const float* d_arena, const long* d_kvmap, float* d_out, int frames,
                           int T, int D, int heads, bool remap);

/* src/attn_kernel.h:25-29 */
__attribute__((visibility("default")))
void attn_forward_single_frame(const float* d_q_f, const float* d_k, const float* d_v,
                               const float* d_arena, const long* d_kvmap_f, float* d_out_f,
                               int T, int D, int heads, int cross, int frame_idx);

static const int ATTENTION_KTILE = 64; /* src/attn_kernel.h:31 */
static const int ATTENTION_WARPS = 8;  /* src/attn_kernel.h:32 */

#endif
