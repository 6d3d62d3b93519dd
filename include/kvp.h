/* libkvp.so: B200 additions to the reference interface (no torch types).
 *
 * Everything here extends GauthamMK-0/cuda-kv-persistence's surface; the
 * drop-in entry points themselves are in kv_tile_manager.h and
 * attn_kernel.h.  All kvp_* functions return 0 on success or a negative
 * status (-1 argument, -2 CUDA, -3 capacity, -4 unsupported, -5 timeout,
 * -6 KVMap out of range); kvp_last_error() describes the last failure on
 * the calling thread.  Streams are cudaStream_t passed as void*.
 */
#ifndef KVP_H
#define KVP_H

#ifdef __cplusplus
extern "C" {
#endif

const char* kvp_version(void);
const char* kvp_last_error(void);

/* Device status word written by the kernels: bit 0 = a KVMap entry pointed
 * outside the arena (the base row was read instead), bit 1 = a bounded
 * device wait expired.  Synchronises `stream`, returns and clears it. */
int kvp_read_status(void* stream);

/* Diagnostics: launches one kernel whose bounded mbarrier wait can never
 * complete (0 < limit_ns <= 5 s); it gives up after limit_ns and sets status
 * bit 1, exactly as an expired wait in the attention kernel does.  Lets tests
 * exercise failure detection without hanging a GPU. */
int kvp_probe_bounded_wait(long long limit_ns, void* stream);

typedef struct {
    int device, sm_count, cc_major, cc_minor;
    long long l2_bytes;
    long long max_persisting_l2_bytes;        /* cudaDevAttrMaxPersistingL2CacheSize */
    long long max_access_policy_window_bytes; /* cudaDevAttrMaxAccessPolicyWindowSize */
    long long persisting_limit_bytes;         /* current cudaLimitPersistingL2CacheSize */
    long long hbm_bytes;
} kvp_device_info;
/* device < 0: the current device.  Replaces the hard-coded RTX 3060 values
 * of the reference's configs/grounding_config.json and its probe
 * src/l2_persist_smoke.cu:20-35. */
int kvp_query_device(int device, kvp_device_info* out);

/* TileGatingPolicy::select by id, src/tile_gating_policy.h:14-15
 * (0 none, 1 uniform, 2 recency, 3 motion, 4 reuse_weighted; tiles_per_frame
 * and total_frames parameterise reuse_weighted as in its constructor,
 * src/tile_gating_policy.h:51). */
int tgp_select(int policy, const float* scores, int n, int max_tiles, int tiles_per_frame,
               int total_frames, long* out_ids, int* out_count);

/* Motion CSV reader, src/run_policy_experiment.cu:45-69: scores [frames][num_tiles],
 * reuse (may be NULL) [frames][num_tiles]. Returns accepted rows or -1. */
int kvp_read_motion_csv(const char* path, int frames, int num_tiles, float* scores,
                        signed char* reuse);

/* Vectorised arena compaction (replaces the 2 cudaMemcpyAsync per row of
 * src/kv_tile_manager.cu:111-116): for i < n,
 * arena[pairs[2i+1]] = K[pairs[2i]] || V[pairs[2i]], rows of row_bytes
 * (multiple of 16) bytes; d_pairs is device memory. */
int kvp_stage_rows(const void* k, const void* v, void* arena, const int* d_pairs, int n,
                   long long row_bytes, void* stream);

/* FP32 remapped attention over an explicit key span (intra, cross and
 * sliding window in one form): query rows [0, T) of q/out, key rows
 * [k_lo, k_hi) of k/v, kvmap indexed by the absolute key row; map entries
 * >= arena_rows are reported in kvp_read_status (arena_rows < 0: unchecked).
 * src/gated_attention_kernel.cu:34-139. */
int kvp_attn_fp32(const float* q, const float* k, const float* v, const float* arena,
                  const long long* kvmap, float* out, int T, int D, int heads, long long k_lo,
                  long long k_hi, long long arena_rows, void* stream);

/* ---- BF16 tcgen05 remapped attention (sm_100a) ---------------------------
 * Same semantics as attn_forward_kernel (src/gated_attention_kernel.cu:34-139)
 * in bf16 with fp32 accumulation, for one layer and any set of heads.
 * KVP_ATTN_PAIR=1 in the environment runs the SM-pair kernel (two CTAs per
 * 256 query rows, tcgen05 cta_group::2) instead of the one-SM kernel; same
 * arguments and results within the bf16 tolerance, no key-range split. */
typedef struct {
    const void* q;          /* bf16 [q_rows][D], D = heads*128 */
    const void* k;          /* bf16 [kv_rows][D] */
    const void* v;          /* bf16 [kv_rows][D] */
    void* out;              /* bf16 [q_rows][D] */
    const void* arena;      /* bf16 [arena_rows][2*D] (K half, V half) or NULL */
    const long long* kvmap; /* int64 [kv_rows], absolute key rows, or NULL */
    long long q_rows, kv_rows, arena_rows;
} kvp_layer_io;

typedef struct {
    int tokens;    /* rows per frame (T) */
    int frames;    /* query frames [q_frame0, q_frame0 + frames) */
    int q_frame0;
    int mode;      /* 0 intra (keys of the same frame), 1 causal cross-frame */
    int window;    /* causal: 0 = frames 0..f, W = frames max(0,f-W+1)..f */
    int heads;
    int head_dim;  /* 128 */
    int head0;     /* heads [head0, head0 + nheads) */
    int nheads;
    int flat;      /* causal, window 0: 128-row query tiles across frame edges */
} kvp_attn_desc;

int kvp_attn_bf16(const kvp_layer_io* io, const kvp_attn_desc* d, void* stream);

/* No counterpart in the reference (its driver launches one frame of one
 * layer at a time, src/run_policy_experiment.cu:246-255).  kvp_attn_bf16
 * over n layers, head chunks or query frames in one grid: ios[i], ds[i] as
 * for kvp_attn_bf16, all ds[i] equal in tokens, frames, mode, window and
 * flat (heads / head0 / nheads / q_frame0 may differ).  Short chunks then
 * share their ramp-down with the next chunk's work.  A launch holds up to 12
 * of them; more are spread evenly over as few launches as needed.  Results are those of
 * n kvp_attn_bf16 calls; no key-range split is used.  A persisting window
 * set on `stream` covers one address range for the whole launch. */
int kvp_attn_bf16_multi(const kvp_layer_io* ios, const kvp_attn_desc* ds, int n, void* stream);

/* No counterpart in the reference.  kvp_attn_bf16 for callers that cannot
 * allocate device memory -- hosts whose allocator owns all device memory
 * and forbids stray cudaMalloc calls, serving loops that cannot take the
 * device-wide synchronisation of a first-call cudaMalloc.  Nothing is allocated: the status word and a device
 * copy of the KVMap, which the caller passes in HOST memory (host_kvmap,
 * int64, (q_frame0+frames)*tokens rows, at most 65,536; NULL = no remap;
 * io->kvmap must be NULL), live in a static device array of ~512 KB that
 * each GPU holds until exit.  Q/K/V/Out/arena are still device memory from
 * the caller.  The first call on a device looks the array up (make it before
 * any stream capture); all calls share the array (the status word is reset
 * per call), so calls that overlap on the GPU race.  host_status (may be
 * NULL) receives the status word and then the call synchronises `stream`.
 * Without host_status the call returns before the map copy has run: a map
 * in pinned host memory must stay unchanged until `stream` has passed this
 * call (synchronise the stream or an event recorded after it before
 * refilling the buffer); a map in pageable memory is staged before return.
 * The array's device address is looked up once per device in the primary
 * context: do not call this from another context on that device, or after
 * cudaDeviceReset.  Queued kvtm_* staging copies are not flushed: call
 * kvtm_flush first.  Returns -1 for a bad descriptor (checked first), -3
 * when a valid descriptor's map exceeds the limit. */
int kvp_attn_bf16_noalloc(const kvp_layer_io* io, const kvp_attn_desc* d,
                          const long long* host_kvmap, int* host_status, void* stream);

/* ---- QKV producer: the block's LayerNorm and qkv_proj
 * (src/backbone.py:13-33; nn.Linear(D, 3D) + view(b, t, 3, heads, head_dim))
 * in bf16 with fp32 accumulation, tcgen05 GEMM.  x bf16 [rows][D] (rows >=
 * 128, D a multiple of 256), w bf16 [3D][D] (Q rows, then K, then V), bias
 * fp32 [3D] or NULL; Q/K/V bf16 [rows][D] (q may be NULL), head h at columns
 * [128h, 128h+128).  When kvmap != NULL, row r's K and V are also written to
 * arena row kvmap[map_row0 + r] (bf16 [arena_rows][2D], K half then V half)
 * when that entry is in [0, arena_rows); entries >= arena_rows set status
 * bit 0 and are skipped.  No reference counterpart: the reference computes
 * K/V in PyTorch and never hands them to the CUDA path
 * (src/backbone.py:16-22, 246-255).  All buffers 16-byte aligned. */
typedef struct {
    const void* x;
    const void* w;
    const float* bias;
    void* q;
    void* k;
    void* v;
    void* arena;
    const long long* kvmap;
    long long rows, map_row0, arena_rows;
    int D;
} kvp_qkv_io;
int kvp_qkv_project_bf16(const kvp_qkv_io* io, void* stream);
/* y = (x - mean) / sqrt(var + eps) * gamma + beta per row (nn.LayerNorm,
 * biased variance): x, y bf16 [rows][D] (D % 8 == 0), gamma/beta fp32 [D]. */
int kvp_layernorm_bf16(const void* x, const float* gamma, const float* beta, void* y,
                       long long rows, int D, float eps, void* stream);

/* ---- Motion-trace producer on the GPU (traces/gen_motion_from_video.py:
 * 101-121): dense two-frame optical flow between consecutive frames
 * (Farnebaeck's polynomial-expansion method, the one the reference calls
 * through OpenCV with pyr_scale 0.5, levels 3, winsize 15, iterations 3,
 * poly_n 5, poly_sigma 1.2), per-pixel magnitude, means per cell of the
 * latent grid and per row-major tile of tile_cells cells.  Frames are uint8
 * grayscale [frames][height][width] in device memory; height and width must
 * be multiples of grid_rows and grid_cols. */
typedef struct {
    int height, width, levels, winsize, iterations, poly_n;
    float poly_sigma, pyr_scale;
    int grid_rows, grid_cols, tile_cells;
} kvp_motion_params;
void* kvp_motion_create(const kvp_motion_params* p);   /* NULL on bad parameters / no memory */
void kvp_motion_destroy(void* m);
int kvp_motion_tiles(void* m);                         /* tiles per frame */
/* flow fp32 [2][height][width] (dx plane, dy plane): next(x + d) ~ prev(x) */
int kvp_motion_flow(void* m, const void* d_prev, const void* d_next, float* d_flow, void* stream);
/* change fp32 [frames][tiles] on the device: row f >= 1 = mean flow
 * magnitude per tile between frames f-1 and f, row 0 = row 1 (:117) */
int kvp_motion_trace(void* m, const void* d_frames, int frames, float* d_change, void* stream);
/* Host: tau = the percentile (numpy's linear interpolation) of change rows
 * 1..frames-1; reuse = change < tau except row 0 (all 0); is_static =
 * change < tau (:119-121, 146-151).  reuse / is_static / tau may be NULL. */
int kvp_motion_threshold(const float* change, int frames, int tiles, double percentile,
                         signed char* reuse, signed char* is_static, double* tau);

/* ---- Session: the per-frame admission loop / KVMap emitter of
 * src/run_policy_experiment.cu:156-274 as a library. */
typedef struct {
    int mode;        /* 0 intra, 1 cross, 2 stack (one admission for all frames),
                        3 reuse (intra attention; streaming slots keyed by token
                        position, re-copied only when the tile changed; needs
                        streaming = 1) */
    int window;      /* cross: 0 = full prefix, W = candidates of the last W frames */
    int streaming;   /* 0 dense arena, 1 sticky streaming slots */
    int policy;      /* as tgp_select */
    int frames, tokens, hidden, tile_tokens;
    int elem_bytes;  /* 4 fp32 (the reference's accounting), 2 bf16 */
    int layers;      /* device arenas to keep (0 = host planning only, no GPU needed) */
    long long set_aside; /* persisting budget in bytes = arena capacity per layer */
} kvp_session_config;

typedef struct {
    int frame, sel_count, staged_tiles, copies;
    long long map_row0, map_rows, window_bytes, staged_bytes;
    int restaged;    /* reuse mode: rows re-copied into a slot they held */
    int hits;        /* streaming: rows mapped to a held slot without a copy */
} kvp_step_info;

void* kvp_session_create(const kvp_session_config* c);
void kvp_session_destroy(void* s);
int kvp_session_plan_frame(void* s, int frame, const float* scores_flat); /* intra / cross */
int kvp_session_plan_stack(void* s, const float* scores_flat);            /* stack */
/* Reuse mode (no reference counterpart: the reference reads the motion
 * CSV's reuse column, src/run_policy_experiment.cu:114-118, and stages with
 * changed = false, :211).  reuse_flat is [frames][tiles], 1 = tile unchanged
 * since the previous frame; NULL = every tile changed.  A selected,
 * unchanged tile whose rows hold slots copies nothing. */
int kvp_session_plan_frame_reuse(void* s, int frame, const float* scores_flat,
                                 const signed char* reuse_flat);
int kvp_session_finish(void* s);
int kvp_session_info(void* s, kvp_step_info* out);
long long kvp_session_slots(void* s);
long long kvp_session_cap_rows(void* s);
int kvp_session_map(void* s, long long row0, long long n, long long* out);
int kvp_session_copies(void* s, int* pairs_out, int cap);
int kvp_session_selected(void* s, long* ids_out, int cap);
long long* kvp_session_device_map(void* s);
void* kvp_session_arena(void* s, int layer);
int kvp_session_upload(void* s, void* stream);
int kvp_session_stage(void* s, const void* const* k_layers, const void* const* v_layers,
                      void* stream);
int kvp_session_stage_layer(void* s, int layer, const void* k, const void* v, void* stream);
int kvp_session_window(void* s, int layer, void* stream);
int kvp_session_clear_window(void* s, void* stream);
/* kvp_session_stage without the source rows [skip_row0, skip_row0 +
 * skip_rows): the rows a kvp_session_produce call wrote in place. */
int kvp_session_stage_except(void* s, const void* const* k_layers, const void* const* v_layers,
                             long long skip_row0, long long skip_rows, void* stream);
/* Layer `layer`'s kvp_qkv_project_bf16 of rows [row0, row0 + rows) with this
 * step's device KVMap and that layer's arena (after kvp_session_upload): the
 * rows it maps land in the arena with no gather.  bf16 sessions only; not
 * in reuse mode (a sticky hit keeps its old slot contents); the rows must lie
 * in this step's map slice (kvp_step_info map_row0 / map_rows). */
int kvp_session_produce(void* s, int layer, const void* x, const void* w, const float* bias,
                        void* q, void* k, void* v, long long row0, long long rows, void* stream);
/* One per-frame step in one call (no reference counterpart; the reference
 * driver does these steps inline, src/run_policy_experiment.cu:156-274):
 * kvp_session_plan_frame_reuse (reuse_flat is read in reuse mode only),
 * then, unless the policy is None, kvp_session_upload, kvp_session_stage and,
 * when window_layer >= 0, kvp_session_window(window_layer).  Stops at the
 * first error and returns it. */
int kvp_session_step(void* s, int frame, const float* scores_flat, const signed char* reuse_flat,
                     const void* const* k_layers, const void* const* v_layers, int window_layer,
                     void* stream);
/* The per-frame loop of one layer in one call, no reference counterpart
 * (the reference driver runs it inline, src/run_policy_experiment.cu:156-274,
 * with a device synchronisation per frame): for f in [f0, f0 + nframes),
 * kvp_session_step(f, scores_flat, reuse_flat, &io->k, &io->v, window 0),
 * then kvp_attn_bf16 of query frame f (*d with q_frame0 = f, frames = 1)
 * through this step's KVMap and arena 0 (no map for the None policy);
 * finally the persisting window is cleared.  Everything is queued on
 * `stream`; the host plans frame f+1 while the device runs frame f.
 * io->arena / io->kvmap / io->arena_rows are ignored.  Stops at the first
 * error and returns it. */
int kvp_session_run_frames(void* s, int f0, int nframes, const float* scores_flat,
                           const signed char* reuse_flat, const kvp_layer_io* io,
                           const kvp_attn_desc* d, void* stream);
/* The same loop for a dense-arena session (streaming 0, intra or cross) with
 * the frames' attention merged into one grid (no reference counterpart:
 * admission reads only the motion scores, so frames can be planned before
 * any runs).  The frames go in chunks of up to 12 (16 frames: 8 + 8), in
 * frame order.  For each frame f0 + i of a chunk: kvp_session_plan_frame,
 * then, unless the policy is None, its KVMap slice is uploaded into
 * maps + i * (frames * tokens) and its admitted rows are staged into arena
 * i.  When the session's arenas sit back to back a whole number of rows
 * apart (the usual case), frame i's map entries index them as one block from
 * arena 0 (slot + i * that stride), so every frame of a launch shares one
 * set of tensor maps; otherwise they are arena i's own slots.  Then a
 * persisting window over the chunk's last arena and one
 * kvp_attn_bf16_multi launch over the chunk (longest key span first); the
 * host plans the next chunk while the device runs this one.  Finally the
 * window is cleared.  Each frame reads the rows it reads in
 * kvp_session_run_frames, so the outputs are the same bytes.
 * Needs a session with layers >= nframes and, unless the policy is None,
 * `maps`: a device int64 buffer of nframes * frames * tokens entries owned
 * by the caller (only each frame's slice is written).  io->arena /
 * io->kvmap / io->arena_rows are ignored.  Bad arguments are reported before
 * any device work. */
int kvp_session_run_frames_batched(void* s, int f0, int nframes, const float* scores_flat,
                                   const kvp_layer_io* io, const kvp_attn_desc* d,
                                   long long* maps, void* stream);

#ifdef __cplusplus
}
#endif
#endif
