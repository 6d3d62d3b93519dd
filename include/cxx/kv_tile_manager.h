/* libkvp.so: the C++ KVTileManager class, for callers compiled against the
 * reference's C++ interface.
 *
 * Drop-in for GauthamMK-0/cuda-kv-persistence src/kv_tile_manager.h:15-90.
 * A caller that includes this header (or the reference's own, whose layout
 * this one repeats member for member) and links libkvp.so gets this
 * library's manager: budgeted per-tile admission, the compacted K|V arena,
 * streaming mode with sticky LIFO slots, and persisting access-policy
 * windows.  Return values, slots and byte counts are those of the C facade
 * (kv_tile_manager.h one directory up), which is bit-exact with the
 * reference.
 *
 * Layout.  The class keeps exactly the reference's data members, in the same
 * order and of the same types, because callers allocate it (on the stack or
 * with new) from their own copy of the declaration, and the inline accessors
 * below read the members directly.  The library keeps the members that
 * those accessors read current after every call; the three containers
 * (active_, row_slot_, free_slots_) stay empty, because the working state
 * lives in the library's own manager object, one per KVTileManager.
 *
 * Behaviour the reference leaves to stream 0 stays on stream 0: windows,
 * limits and the staging gather are issued there.  Staging copies are queued
 * and issued as one gather kernel at the next *_apply_window, *_end or
 * attention launch, stream-ordered before it.
 */
#ifndef KVP_CXX_KV_TILE_MANAGER_H
#define KVP_CXX_KV_TILE_MANAGER_H

#include <cstddef>
#include <unordered_map>
#include <vector>

#ifndef KVP_KVTM_RESULT_DECLARED
#define KVP_KVTM_RESULT_DECLARED
/* src/kv_tile_manager.h:15-19 */
enum KvtmResult {
    KVTM_ADMITTED = 1,
    KVTM_REFUSED_BUDGET = 0,
    KVTM_INVALID = -1, /* bad arguments, duplicate admit, unknown tile, window too large */
};
#endif

/* src/kv_tile_manager.h:21-90 */
class __attribute__((visibility("default"))) KVTileManager {
public:
    KVTileManager(size_t budget_bytes, size_t max_window_bytes);
    ~KVTileManager();

    /* Sets cudaLimitPersistingL2CacheSize to the budget. */
    bool init();

    /* Persisting window over [ptr, ptr+bytes) when the budget allows. */
    KvtmResult admit(long tile_id, void* ptr, size_t bytes);
    bool release(long tile_id);
    void clear();

    size_t persisted_bytes() const { return used_bytes_; }
    int persisted_tiles() const;
    bool is_persisted(long tile_id) const;
    size_t query_device_limit() const;

    /* Arena mode: admitted rows are copied into one contiguous buffer of
     * [K half | V half] rows, renumbered 0, 1, 2, ... every step, and one
     * window covers the rows staged so far. */
    bool arena_init(size_t capacity_bytes, size_t row_stride_floats);
    void arena_begin_step();
    bool arena_stage(const void* k_dev, size_t k_bytes, const void* v_dev, size_t v_bytes,
                     long* out_row);
    bool arena_apply_window();
    void arena_end_step();
    size_t arena_used_bytes() const { return arena_used_; }
    void* arena_device_ptr() const { return arena_; }

    /* Streaming mode: a row keeps its slot while it stays admitted; a sticky
     * hit copies nothing unless the caller says the row changed. */
    bool streaming_begin();
    bool streaming_stage(long row_id, const void* k_dev, size_t k_bytes, const void* v_dev,
                         size_t v_bytes, bool changed, long* out_slot, bool* restaged);
    bool streaming_release(long row_id);
    bool streaming_apply_window();
    void streaming_end();
    size_t streaming_staged_bytes() const { return staged_bytes_; }

private:
    /* Library-internal: copies the engine's state into the members below.
     * A non-virtual member function, so it adds nothing to the layout. */
    void kvp_sync_();

    struct Entry {
        void* ptr;
        size_t bytes;
    };

    /* Members in the reference's order (src/kv_tile_manager.h:73-89). */
    std::unordered_map<long, Entry> active_;
    size_t budget_bytes_;
    size_t max_window_bytes_;
    size_t used_bytes_;
    bool initialized_;

    float* arena_;
    size_t arena_cap_;
    size_t arena_row_stride_floats_;
    size_t arena_next_row_;
    size_t arena_used_;

    std::unordered_map<long, long> row_slot_;
    std::vector<long> free_slots_;
    long slot_high_water_;
    size_t staged_bytes_;
};

#endif
