/* libkvp.so: KVTileManager C ABI.
 *
 * Drop-in for the extern "C" facade of GauthamMK-0/cuda-kv-persistence
 * src/kv_tile_manager.cu:223-339 (bound by ctypes in
 * tests/test_capacity_admission.py:42-60).  Same symbols, argument meaning
 * and return codes: KvtmResult 1 admitted / 0 refused (budget) / -1 invalid,
 * booleans as 1/0, nullptr from kvtm_create on failure.  `long` is 64-bit.
 *
 * Staging calls (kvtm_arena_stage, kvtm_streaming_stage) queue their row
 * copies; the copies run as one gather kernel at the next kvtm_*_window,
 * kvtm_*_end, kvtm_flush or attention launch, stream-ordered before it
 * (the reference issued two cudaMemcpyAsync per row on stream 0).
 */
#ifndef KVP_KV_TILE_MANAGER_H
#define KVP_KV_TILE_MANAGER_H

#ifdef __cplusplus
extern "C" {
#endif

/* src/kv_tile_manager.cu:225-232  KVTileManager(budget, max_window) */
void* kvtm_create(long budget_bytes, long max_window_bytes);
/* :234                            ~KVTileManager (clear + free arena) */
void kvtm_destroy(void* m);
/* :236-238  init(): cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, budget) -> 1/0 */
int kvtm_init(void* m);
/* :240-242  query_device_limit(): cudaDeviceGetLimit read-back */
long kvtm_query_limit(void* m);
/* :244-247  admit(tile, ptr, bytes) -> 1 / 0 / -1; applies a persisting window */
int kvtm_admit(void* m, long tile_id, void* ptr, long bytes);
/* :249-251  release(tile) -> 1/0 */
int kvtm_release(void* m, long tile_id);
/* :253      clear(): drop all tiles, cudaCtxResetPersistingL2Cache */
void kvtm_clear(void* m);
/* :255-257 */
long kvtm_persisted_bytes(void* m);
/* :259-261 */
int kvtm_persisted_tiles(void* m);
/* :264-268  cudaMalloc helper for tests */
void* kvtm_dev_alloc(long bytes);
/* :270      cudaFree helper */
void kvtm_dev_free(void* p);

/* ---- arena mode: src/kv_tile_manager.cu:274-298 */
int kvtm_arena_init(void* m, long cap_bytes, long row_stride_floats);
void kvtm_arena_begin(void* m);
int kvtm_arena_stage(void* m, const void* k_dev, long k_bytes, const void* v_dev, long v_bytes,
                     long* out_row);
int kvtm_arena_window(void* m);
void kvtm_arena_end(void* m);
long kvtm_arena_used(void* m);
void* kvtm_arena_ptr(void* m);

/* ---- streaming mode: src/kv_tile_manager.cu:302-328 */
int kvtm_streaming_begin(void* m);
int kvtm_streaming_stage(void* m, long row_id, const void* k_dev, long k_bytes,
                         const void* v_dev, long v_bytes, int changed, long* out_slot,
                         int* restaged);
int kvtm_streaming_release(void* m, long row_id);
int kvtm_streaming_window(void* m);
void kvtm_streaming_end(void* m);
long kvtm_streaming_staged_bytes(void* m);

/* ---- tile layout cross-check: src/kv_tile_manager.cu:331-339 (src/tile_layout.h:13-31) */
long kvtm_layout_tiles_per_frame(int tokens_per_frame, int tile_tokens);
long kvtm_layout_tile_start(int tokens_per_frame, int tile_tokens, long id);
int kvtm_layout_tile_count(int tokens_per_frame, int tile_tokens, long id);

/* ---- additions (no counterpart in the reference facade) */
#define KVTM_FLAG_DRY_RUN 1u /* accounting only: no CUDA call, usable without a GPU */
void* kvtm_create_ex(long budget_bytes, long max_window_bytes, unsigned flags);
/* Stream for windows and staging copies (default: legacy stream 0). */
void kvtm_set_stream(void* m, void* cuda_stream);
/* Issue queued staging copies now; returns 0 or a negative kvp status. */
int kvtm_flush(void* m);
long kvtm_pending_copies(void* m);
/* Window requests so far (bytes, hitProp 2 persisting / 0 normal); returns the count. */
long kvtm_window_log(void* m, long* bytes_out, int* prop_out, long cap);
long kvtm_reset_calls(void* m);

#ifdef __cplusplus
}
#endif
#endif
