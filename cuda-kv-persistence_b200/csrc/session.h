// Session: the per-frame admission loop that turns policy selections into a
// KVMap plus a list of rows to stage, i.e. the host hot loop of the
// reference driver (src/run_policy_experiment.cu:156-274) as a library.
//
// Per step (one query frame, or the whole stack): select -> release rows of
// tiles that dropped out (streaming) -> stage the selected tiles' rows in
// policy order -> KVMap[row] = arena slot.  Admission, slot numbers and byte
// counts are bit-exact with the reference for intra and cross modes; the
// sliding window (cross, window > 0), the stack mode and the reuse mode are
// extensions, defined as follows:
//   * window W: frame f's candidates are the tiles of frames
//     [max(0, f-W+1), f]; ReuseWeighted counts remaining sweeps from that
//     first frame (total_frames - base); ids are offset to absolute gids;
//   * stack: one admission over all frames' tiles (the cross step of the last
//     frame), one KVMap shared by every query frame of a causal stack.
//   * reuse (temporal reuse, streaming only): intra attention, but a row's
//     streaming slot is keyed by its token position t0+r, so a tile keeps
//     its slots from frame to frame while the policy keeps selecting it; a
//     tile flagged unchanged (the motion CSV's reuse column) is a sticky hit
//     and copies nothing, a changed tile is re-copied into the slots it
//     holds.  The reference loads that column (src/run_policy_experiment.cu:
//     114-118) but stages with changed = false (:211).
// The device side keeps one arena per layer (all layers share the admission:
// motion scores are per tile, not per layer) and stages every layer's rows
// with one gather launch.
#pragma once

#include <cstdint>
#include <memory>
#include <vector>

#include <cuda_runtime.h>

#include "kernels.h"
#include "kv_tile_manager.h"
#include "tile_gating_policy.h"
#include "tile_layout.h"

namespace kvp {

enum SessionMode { MODE_INTRA = 0, MODE_CROSS = 1, MODE_STACK = 2, MODE_REUSE = 3 };

struct SessionConfig {
    int mode;         // SessionMode
    int window;       // cross/stack: 0 = full causal prefix, W > 0 = last W frames
    int streaming;    // 0 dense arena, 1 sticky streaming slots
    int policy;       // PolicyId
    int frames;
    int tokens;       // tokens per frame
    int hidden;       // D = heads * head_dim
    int tile_tokens;
    int elem_bytes;   // 4 = fp32 (reference accounting), 2 = bf16
    int layers;       // arenas kept on device (0 = plan only)
    int64_t set_aside;// persisting budget in bytes; also the arena capacity per layer
};

struct SessionStepInfo {
    int frame;            // -1 for a stack step
    int sel_count;        // raw policy count
    int staged_tiles;
    int copies;           // rows to stage this step
    int64_t map_row0;     // first KVMap row the kernel reads
    int64_t map_rows;     // rows the kernel reads
    int64_t window_bytes; // persisting window span, 0 when none
    int64_t staged_bytes; // streaming: cumulative; dense: arena bytes used this step
    int restaged;         // reuse: rows re-copied into a slot they already held
    int hits;             // streaming: sticky hits (rows mapped without a copy)
};

class Session {
public:
    explicit Session(const SessionConfig& c);
    ~Session();
    int status() const { return status_; }  // KVP_OK after construction

    // Host planning (no GPU needed).
    // intra / cross / reuse; reuse_flat ([frames][tiles], 1 = unchanged)
    // is read in reuse mode only, NULL = every tile changed.
    int plan_frame(int f, const float* scores_flat, const int8_t* reuse_flat = nullptr);
    int plan_stack(const float* scores_flat);         // stack
    const SessionStepInfo& info() const { return info_; }
    const int64_t* host_map() const { return map_.data(); }
    const std::vector<int32_t>& pairs() const { return pairs_; }  // (row, slot) interleaved
    const std::vector<long>& selected_ids() const { return sel_ids_; }
    int64_t slots() const { return slots_; }
    bool persists() const { return c_.policy != POLICY_NONE; }
    int64_t cap_rows() const { return cap_rows_; }
    int64_t map_len() const { return (int64_t)map_.size(); }
    int finish();  // streaming_end / final demote (same as the driver's end of run)

    // Device side (layers > 0).
    int64_t* device_map() const { return d_map_; }
    void* arena(int layer) const;
    int64_t arena_layer_bytes() const { return arena_layer_bytes_; }
    // Uploads this step's map slice and copy list (pinned staging, async).
    int upload(cudaStream_t s);
    // The same with the map slice going to `dmap` (device, map_len() entries,
    // only this step's slice written) instead of the session's own map, and
    // slot_offset added to every slot in the map and the copy list.
    int upload_to(int64_t* dmap, cudaStream_t s, int64_t slot_offset = 0);
    const SessionConfig& config() const { return c_; }
    // Rows from one layer's arena to the next when the arenas sit back to
    // back a whole number of rows apart (every layer's rows then index one
    // arena of layers * stride rows from arena(0)), else 0.
    int64_t arena_stride_rows() const;
    // Dense-arena batch (not streaming, intra or cross, policy not None,
    // arena0 + n <= layers, arena_stride_rows() > 0): frames f0 .. f0+n-1
    // planned in order; frame f0 + i goes to arena a = arena0 + i: its KVMap
    // slice is written (on `s`) to maps + a * map_len() with its slots moved
    // to that arena (slot + a * stride: entries index the back-to-back
    // arenas from arena(0)) and its rows are gathered there.  Entries outside
    // each frame's slice are not written.  info() then describes the last
    // frame.
    int stage_batched(int f0, int n, int arena0, const float* scores_flat, const void* k,
                      const void* v, int64_t* maps, cudaStream_t s);
    // Gathers this step's rows into every layer's arena, except source rows
    // in [skip_row0, skip_row0 + skip_rows) (rows a produce() call wrote).
    int stage(const void* const* k_layers, const void* const* v_layers, cudaStream_t s,
              int64_t skip_row0 = 0, int64_t skip_rows = 0);
    // Layer `layer`'s QKV projection of rows [row0, row0 + rows) (x bf16
    // [rows][D], w bf16 [3D][D], bias fp32 [3D] or null) into q/k/v (bf16
    // [rows][D], row 0 = row0; q may be null), writing every row this step
    // maps into that layer's arena as well -- so stage() can skip them.
    // Needs upload() of this step first, and a step in which every mapped
    // row in the range is a copy (any mode but reuse, whose sticky hits keep
    // their old slot contents); the range must lie in the step's map slice.
    int produce(int layer, const void* x, const void* w, const float* bias, void* q, void* k,
                void* v, int64_t row0, int64_t rows, cudaStream_t s);
    // Same for one layer (used when layers' K/V arrive one at a time).
    int stage_layer(int layer, const void* k, const void* v, cudaStream_t s);
    // Persisting window over layer's arena span (or a normal-property
    // window when this step has no span).
    int apply_window(int layer, cudaStream_t s);
    int clear_window(cudaStream_t s);
    // One per-frame step in a single call: plan_frame, then (unless the
    // policy is None) upload, stage into every layer's arena and, when
    // window_layer >= 0, the persisting window over that layer's arena.
    int step(int f, const float* scores_flat, const int8_t* reuse_flat,
             const void* const* k_layers, const void* const* v_layers, int window_layer,
             cudaStream_t s);

private:
    int stage_rows_of(int64_t gid, int64_t src_frame, int64_t tile);
    int plan_reuse(int f, const float* scores_flat, const int8_t* reuse_flat);

    SessionConfig c_;
    TileLayout layout_;
    std::unique_ptr<TileGatingPolicy> policy_;
    std::unique_ptr<KVTileManager> mgr_;  // dry-run accounting
    int status_ = 0;
    int64_t nt_ = 0, slots_ = 0, cap_rows_ = 0, row_kv_bytes_ = 0;
    std::vector<int64_t> map_;
    std::vector<int32_t> pairs_;
    std::vector<long> ids_;
    std::vector<long> sel_ids_;
    std::vector<char> selected_, prev_selected_;
    // reuse mode: the slots of each tile whose rows all hold one (tile_full_),
    // so kept tiles map and re-copy without a lookup per row
    std::vector<int64_t> tile_slots_;
    std::vector<char> tile_full_;
    int64_t prev_len_ = 0;
    int last_frame_ = -1;
    bool finished_ = false;
    SessionStepInfo info_{};

    // device
    int64_t* d_map_ = nullptr;
    int32_t* d_pairs_ = nullptr;
    void* d_arena_ = nullptr;
    int64_t arena_layer_bytes_ = 0;
    // Pinned staging for the uploads, a ring of kUploadSlots: an upload only
    // waits for the copy made kUploadSlots uploads earlier, so the host can
    // plan the next frame while the device still works on this one.
    static constexpr int kUploadSlots = 2;
    int64_t* h_map_pinned_[kUploadSlots] = {};
    int32_t* h_pairs_pinned_[kUploadSlots] = {};
    cudaEvent_t upload_done_[kUploadSlots] = {};
    int upload_slot_ = 0;
};

// Reference motion CSV reader (src/run_policy_experiment.cu:45-69): rows
// "frame,tile,score,is_static,start,count[,reuse]", score parsed as "%f";
// absent entries stay 0.  Returns accepted rows, or -1 if unreadable.
int read_motion_csv(const char* path, int frames, int num_tiles, float* scores,
                    int8_t* reuse);

}  // namespace kvp
