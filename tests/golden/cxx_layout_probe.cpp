// Prints, as JSON, the object layout a C++ caller of KVTileManager and of the
// policy classes compiles in: sizes, alignments and member offsets.  Built
// once against the reference's headers (tests/golden/make_golden.py writes
// cxx_layout_ref.json) and once against include/cxx/ by
// tests/test_cxx_boundary.py; the two must be equal, because the caller
// allocates the objects and the library's code reads and writes them.
#define private public
#include "kv_tile_manager.h"
#include "tile_gating_policy.h"
#undef private

#include <cstddef>
#include <cstdio>

#define OFF(m) std::printf("  \"%s\": %zu,\n", #m, offsetof(KVTileManager, m))

int main() {
    std::printf("{\n");
    std::printf("  \"sizeof_KVTileManager\": %zu,\n", sizeof(KVTileManager));
    std::printf("  \"alignof_KVTileManager\": %zu,\n", alignof(KVTileManager));
    OFF(active_);
    OFF(budget_bytes_);
    OFF(max_window_bytes_);
    OFF(used_bytes_);
    OFF(initialized_);
    OFF(arena_);
    OFF(arena_cap_);
    OFF(arena_row_stride_floats_);
    OFF(arena_next_row_);
    OFF(arena_used_);
    OFF(row_slot_);
    OFF(free_slots_);
    OFF(slot_high_water_);
    OFF(staged_bytes_);
    std::printf("  \"sizeof_Entry\": %zu,\n", sizeof(KVTileManager::Entry));
    std::printf("  \"sizeof_ReuseWeightedPolicy\": %zu,\n", sizeof(ReuseWeightedPolicy));
    std::printf("  \"sizeof_MotionGatedPolicy\": %zu,\n", sizeof(MotionGatedPolicy));
    std::printf("  \"sizeof_TileGatingPolicy\": %zu,\n", sizeof(TileGatingPolicy));
    std::printf("  \"KVTM_ADMITTED\": %d,\n", (int)KVTM_ADMITTED);
    std::printf("  \"KVTM_REFUSED_BUDGET\": %d,\n", (int)KVTM_REFUSED_BUDGET);
    std::printf("  \"KVTM_INVALID\": %d\n", (int)KVTM_INVALID);
    std::printf("}\n");
    return 0;
}
