// KVTileManager: persisting-L2 budget accounting, the compacted K|V arena and
// the access-policy window over it.
//
// Drop-in for the reference's class of the same name
// (src/kv_tile_manager.h:21-90): identical public methods, results and
// admission rules (per-tile admission, dense arena mode, streaming mode with
// sticky LIFO slots).  B200 differences, none of which changes a returned
// value, slot or byte count:
//   * staging copies are queued and issued as ONE vectorised gather kernel
//     (csrc/compaction.cu) at the next window / flush / end call, instead of
//     two cudaMemcpyAsync per row;
//   * windows go to a caller-chosen stream (default: legacy stream 0, as in
//     the reference);
//   * the persisting-L2 limit found at init() is restored on destruction;
//   * a dry-run flag keeps the accounting and skips every CUDA call, so the
//     same code plans KVMaps on a host with no GPU.
#pragma once

#include <cstddef>
#include <cstdint>
#include <unordered_map>

#include "slot_map.h"
#include <vector>

#include <cuda_runtime.h>

// Global, as in the reference (src/kv_tile_manager.h:15-19); the C++ drop-in
// header include/cxx/kv_tile_manager.h declares the same enum under the same
// guard.
#ifndef KVP_KVTM_RESULT_DECLARED
#define KVP_KVTM_RESULT_DECLARED
enum KvtmResult {
    KVTM_ADMITTED = 1,
    KVTM_REFUSED_BUDGET = 0,
    KVTM_INVALID = -1,  // bad args, duplicate admit, or window larger than allowed
};
#endif

namespace kvp {

enum ManagerFlags : unsigned {
    KVTM_FLAG_DRY_RUN = 1u,  // accounting only: no allocation, copy, limit or window call
};

struct CopyOp {          // one contiguous device copy (16-byte aligned fast path)
    const void* src;
    void* dst;
    uint64_t bytes;
};

class KVTileManager {
public:
    KVTileManager(size_t budget_bytes, size_t max_window_bytes, unsigned flags = 0);
    ~KVTileManager();
    KVTileManager(const KVTileManager&) = delete;
    KVTileManager& operator=(const KVTileManager&) = delete;

    bool init();  // cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, budget)

    KvtmResult admit(long tile_id, void* ptr, size_t bytes);
    bool release(long tile_id);
    void clear();

    size_t persisted_bytes() const { return used_bytes_; }
    int persisted_tiles() const { return (int)active_.size(); }
    bool is_persisted(long tile_id) const { return active_.count(tile_id) != 0; }
    size_t query_device_limit() const;

    // ---- dense arena mode: rows are renumbered 0,1,2,... every step
    bool arena_init(size_t capacity_bytes, size_t row_stride_floats);
    void arena_begin_step();
    bool arena_stage(const void* k_dev, size_t k_bytes, const void* v_dev, size_t v_bytes,
                     long* out_row);
    bool arena_apply_window();
    void arena_end_step();
    size_t arena_used_bytes() const { return arena_used_; }
    void* arena_device_ptr() const { return arena_; }

    // ---- streaming mode: a row keeps its slot while it stays admitted
    bool streaming_begin();
    bool streaming_stage(long row_id, const void* k_dev, size_t k_bytes, const void* v_dev,
                         size_t v_bytes, bool changed, long* out_slot, bool* restaged);
    bool streaming_release(long row_id);
    bool streaming_apply_window();
    void streaming_end();
    size_t streaming_staged_bytes() const { return staged_bytes_; }
    // Counts a re-copy of `bytes` into slots already held (what
    // streaming_reserve does for a held row with changed = true), for callers
    // that know the slots without looking them up.
    void streaming_count_restage(size_t bytes) { staged_bytes_ += bytes; }

    // ---- B200 additions
    // Slot accounting without a copy (the caller stages rows itself, e.g. a
    // session's multi-layer gather kernel).  Same results as the staging
    // calls above; *copy_needed tells whether the row's data must be written.
    bool arena_reserve(size_t row_bytes_kv, long* out_row);
    // arena_reserve for up to n rows in order, stopping at the first one it
    // would refuse: returns how many it reserved, as rows *first_row ..
    // *first_row + count - 1.
    size_t arena_reserve_rows(size_t row_bytes_kv, size_t n, long* first_row);
    // *was_held (optional) tells whether row_id held a slot before the call.
    bool streaming_reserve(long row_id, size_t row_bytes_kv, bool changed, long* out_slot,
                           bool* copy_needed, bool* was_held = nullptr);
    // Span in bytes the next window would cover, 0 when none would be applied.
    size_t arena_window_span() const;
    size_t streaming_window_span() const;
    long slot_high_water() const { return slot_high_water_; }
    size_t arena_next_row() const { return arena_next_row_; }
    bool initialized() const { return initialized_; }
    size_t arena_capacity() const { return arena_cap_; }
    size_t row_stride_bytes() const { return arena_row_stride_floats_ * sizeof(float); }

    void set_stream(cudaStream_t s) { stream_ = s; }
    cudaStream_t stream() const { return stream_; }
    // Issues queued staging copies (one kernel); returns a kvp::Status.
    int flush();
    size_t pending_copies() const { return pending_.size(); }
    bool dry_run() const { return (flags_ & KVTM_FLAG_DRY_RUN) != 0; }

    // Every window request since construction: (offset from arena or tile
    // pointer, bytes, hitProp).  Kept for tests; bounded to the last 4096.
    struct WindowRecord { const void* base; size_t bytes; int hit_prop; };
    const std::vector<WindowRecord>& window_log() const { return window_log_; }
    long reset_calls() const { return reset_calls_; }

private:
    void apply_window(void* ptr, size_t bytes, cudaAccessProperty prop);
    void reset_persisting();
    void queue_copy(void* dst, const void* src, size_t bytes);

    struct Entry { void* ptr; size_t bytes; };

    std::unordered_map<long, Entry> active_;
    size_t budget_bytes_;
    size_t max_window_bytes_;
    size_t used_bytes_ = 0;
    bool initialized_ = false;
    unsigned flags_;

    void* arena_ = nullptr;
    bool arena_ready_ = false;
    size_t arena_cap_ = 0;
    size_t arena_row_stride_floats_ = 0;
    size_t arena_next_row_ = 0;
    size_t arena_used_ = 0;

    SlotMap row_slot_;
    std::vector<long> free_slots_;
    long slot_high_water_ = -1;
    size_t staged_bytes_ = 0;

    cudaStream_t stream_ = 0;
    std::vector<CopyOp> pending_;
    CopyOp* d_ops_ = nullptr;     // device copy list
    CopyOp* h_ops_ = nullptr;     // pinned staging of the copy list
    size_t ops_cap_ = 0;
    cudaEvent_t ops_done_ = nullptr;
    bool limit_saved_ = false;
    size_t saved_limit_ = 0;
    std::vector<WindowRecord> window_log_;
    long reset_calls_ = 0;
    int device_ = -1;             // device of the arena and copy-list buffers, -1 before any
};

// Issues the queued copies of every live manager (stream-ordered on each
// manager's stream).  The attention launchers call it so that staged rows
// always precede the kernel that reads them, as cudaMemcpyAsync on stream 0
// guaranteed in the reference.
int flush_all_managers();

}  // namespace kvp
