/* CPU oracle for the remapped-attention admission path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the
 * reference's host algorithm (GauthamMK-0/cuda-kv-persistence):
 *   tile layout          src/tile_layout.h:13-31
 *   gating policies      src/tile_gating_policy.cpp:6-83
 *   KVTileManager        src/kv_tile_manager.cu:12-219
 *   per-frame KVMap loop src/run_policy_experiment.cu:156-274
 *   motion CSV parse     src/run_policy_experiment.cu:45-69
 * It is used by tests/ (as the checker), by __graft_entry__.smoke() and by
 * bench.py's cpu_baseline leg, never by the product path.  Its results are
 * pinned against the reference's own sources compiled on the CPU
 * (oracle/_ref, see oracle/Makefile) and against the committed fixtures in
 * tests/golden/.
 */
#ifndef KVP_ORACLE_H
#define KVP_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_NONE = 0, ORC_UNIFORM = 1, ORC_RECENCY = 2, ORC_MOTION = 3, ORC_REUSE = 4 };

typedef struct {
    int policy;       /* ORC_* */
    int cross;        /* 0 = intra-frame, 1 = causal cross-frame */
    int streaming;    /* 0 = dense arena, 1 = sticky streaming slots */
    int frames;
    int tokens;       /* tokens per frame */
    int hidden;       /* D = heads * head_dim */
    int tile_tokens;
    int elem_bytes;   /* 4 reproduces the reference's fp32 accounting */
    int window;       /* cross only: 0 = full causal prefix, W>0 = frames [f-W+1, f] */
    int64_t set_aside;/* persisting budget in bytes (also arena capacity) */
} orc_params;

int64_t orc_tiles_per_frame(int tpf, int tt);
int64_t orc_tile_start(int tpf, int tt, int64_t id);
int orc_tile_count(int tpf, int tt, int64_t id);

int orc_select(int policy, const float* scores, int n, int max_tiles, int tpf,
               int total_frames, int64_t* out_ids, int* out_count);

typedef struct orc_mgr orc_mgr;
orc_mgr* orc_mgr_create(int64_t budget_bytes, int64_t max_window_bytes);
void orc_mgr_destroy(orc_mgr* m);
int orc_mgr_init(orc_mgr* m);
int64_t orc_mgr_query_limit(orc_mgr* m);
int orc_mgr_admit(orc_mgr* m, int64_t tile_id, uint64_t ptr, int64_t bytes);
int orc_mgr_release(orc_mgr* m, int64_t tile_id);
void orc_mgr_clear(orc_mgr* m);
int64_t orc_mgr_persisted_bytes(orc_mgr* m);
int orc_mgr_persisted_tiles(orc_mgr* m);
int orc_mgr_arena_init(orc_mgr* m, int64_t cap_bytes, int64_t row_stride_floats);
void orc_mgr_arena_begin(orc_mgr* m);
int orc_mgr_arena_stage(orc_mgr* m, int64_t k_bytes, int64_t v_bytes, int64_t* out_row);
int orc_mgr_arena_window(orc_mgr* m);
void orc_mgr_arena_end(orc_mgr* m);
int64_t orc_mgr_arena_used(orc_mgr* m);
int orc_mgr_streaming_begin(orc_mgr* m);
int orc_mgr_streaming_stage(orc_mgr* m, int64_t row_id, int64_t k_bytes, int64_t v_bytes,
                            int changed, int64_t* out_slot, int* restaged);
int orc_mgr_streaming_release(orc_mgr* m, int64_t row_id);
int orc_mgr_streaming_window(orc_mgr* m);
void orc_mgr_streaming_end(orc_mgr* m);
int64_t orc_mgr_streaming_staged_bytes(orc_mgr* m);
/* last persisting-window request: bytes and hit property (2 persisting, 0 normal) */
int64_t orc_mgr_last_window_bytes(orc_mgr* m);
int orc_mgr_last_window_prop(orc_mgr* m);
int64_t orc_mgr_window_calls(orc_mgr* m);
int64_t orc_mgr_reset_calls(orc_mgr* m);

/* Reference CSV reader: frame_id,tile_id,motion_score,is_static,start,count[,reuse].
 * scores_out is [frames][num_tiles] (zero where absent). Returns rows accepted or -1. */
int orc_read_motion_csv(const char* path, int frames, int num_tiles, float* scores_out,
                        int8_t* reuse_out);

/* Whole per-frame admission loop.  Outputs (all caller-allocated):
 *   map_out      [frames][frames*tokens]  host KVMap after frame f's staging
 *   sel_count    [frames]                 raw policy count
 *   sel_ids      [frames][sel_cap]        raw policy ids (window-relative)
 *   copy_count   [frames]                 rows copied into the arena this frame
 *   copy_rows / copy_slots [copy_cap]     (source row -> arena slot), concatenated
 *   window_bytes [frames]                 persisting window span, -1 if refused
 *   staged_bytes [frames]                 streaming: cumulative staged bytes;
 *                                         dense: arena bytes used this frame
 *   staged_tiles [frames]
 * Returns 0, or <0 on bad arguments / capacity overflow. */
int orc_run_trace(const orc_params* p, const float* scores_flat, int64_t* map_out,
                  int* sel_count, int64_t* sel_ids, int sel_cap, int* copy_count,
                  int64_t* copy_rows, int64_t* copy_slots, int64_t copy_cap,
                  int64_t* window_bytes, int64_t* staged_bytes, int* staged_tiles);

/* Temporal-reuse streaming loop (intra attention, streaming manager).  The
 * reference's loop (src/run_policy_experiment.cu:156-274) with two changes:
 * a row's slot key is its token position t0+r, not frame*tokens+t0+r, so a
 * tile's slots outlive the frame; and streaming_stage gets changed =
 * !reuse[f][tile] (the CSV reuse column, 1 = tile unchanged since the
 * previous frame; NULL = every tile changed) instead of the constant false
 * of :211.  A sticky hit on an unchanged tile copies nothing; a changed
 * tile is re-copied into the slot it holds (src/kv_tile_manager.cu:153-175).
 * Tiles selected at f-1 and not at f release their position keys first,
 * last row first, so that slots come back off the LIFO free stack
 * (src/kv_tile_manager.cu:194-200) in ascending order.
 * Outputs (caller-allocated):
 *   map_out       [frames][tokens]   frame f's KVMap (absolute row f*tokens+t)
 *   copy_count    [frames]           rows copied this frame (new + restaged)
 *   restage_count [frames]           rows re-copied into a slot they held
 *   hit_count     [frames]           sticky hits (no copy)
 *   copy_rows / copy_slots [copy_cap] (source row -> slot), concatenated
 *   window_bytes / staged_bytes / staged_tiles [frames] as orc_run_trace.
 * Requires p->streaming and !p->cross.  Returns 0 or < 0. */
int orc_run_reuse(const orc_params* p, const float* scores_flat, const int8_t* reuse_flat,
                  int64_t* map_out, int* copy_count, int* restage_count, int* hit_count,
                  int64_t* copy_rows, int64_t* copy_slots, int64_t copy_cap,
                  int64_t* window_bytes, int64_t* staged_bytes, int* staged_tiles);

#ifdef __cplusplus
}
#endif
#endif
