// The reference's C++ interface, exported from libkvp.so: the global
// KVTileManager class, the five TileGatingPolicy classes and the C++-linkage
// attention entry points (declared in include/cxx/, restating
// src/kv_tile_manager.h:15-90, src/tile_gating_policy.h:8-68 and
// src/attn_kernel.h:15-32).  A program compiled against the reference's
// headers, such as its driver src/run_policy_experiment.cu, links against
// libkvp.so alone and runs on this library's engine.
//
// Every call forwards to the library's own objects (kvp::KVTileManager,
// kvp::*Policy, kvp::fp32_*), which the C facade uses too, so both
// boundaries give the same slots, return codes and byte counts.  The
// caller allocates a KVTileManager from its copy of the declaration, which
// fixes the object's size and member layout; each object's engine therefore
// lives in a side table keyed by the object's address, and every call copies
// back into the object the members that the header's inline accessors read
// (persisted_bytes, arena_used_bytes, arena_device_ptr,
// streaming_staged_bytes) and the other scalar members.
#include "../../include/cxx/attn_kernel.h"
#include "../../include/cxx/kv_tile_manager.h"
#include "../../include/cxx/tile_gating_policy.h"

#include <mutex>
#include <unordered_map>

#include "kernels.h"
#include "kv_tile_manager.h"
#include "tile_gating_policy.h"

namespace {

std::mutex g_engines_mu;

// Never destroyed: a KVTileManager with static storage may be destroyed
// after this translation unit's statics.
std::unordered_map<const KVTileManager*, kvp::KVTileManager*>& engines() {
    static auto* table = new std::unordered_map<const KVTileManager*, kvp::KVTileManager*>();
    return *table;
}

kvp::KVTileManager* engine_of(const KVTileManager* self) {
    std::lock_guard<std::mutex> g(g_engines_mu);
    auto it = engines().find(self);
    return it == engines().end() ? nullptr : it->second;
}

}  // namespace

// ------------------------------------------------------------ KVTileManager

KVTileManager::KVTileManager(size_t budget_bytes, size_t max_window_bytes)
    : budget_bytes_(budget_bytes), max_window_bytes_(max_window_bytes), used_bytes_(0),
      initialized_(false), arena_(nullptr), arena_cap_(0), arena_row_stride_floats_(0),
      arena_next_row_(0), arena_used_(0), slot_high_water_(-1), staged_bytes_(0) {
    auto* e = new kvp::KVTileManager(budget_bytes, max_window_bytes);
    std::lock_guard<std::mutex> g(g_engines_mu);
    engines()[this] = e;
}

KVTileManager::~KVTileManager() {
    kvp::KVTileManager* e = nullptr;
    {
        std::lock_guard<std::mutex> g(g_engines_mu);
        auto it = engines().find(this);
        if (it != engines().end()) {
            e = it->second;
            engines().erase(it);
        }
    }
    delete e;  // clears admitted tiles, issues queued copies, frees the arena
}

void KVTileManager::kvp_sync_() {
    const kvp::KVTileManager* e = engine_of(this);
    if (!e) return;
    used_bytes_ = e->persisted_bytes();
    initialized_ = e->initialized();
    arena_ = static_cast<float*>(e->arena_device_ptr());
    arena_cap_ = e->arena_capacity();
    arena_row_stride_floats_ = e->row_stride_bytes() / sizeof(float);
    arena_next_row_ = e->arena_next_row();
    arena_used_ = e->arena_used_bytes();
    slot_high_water_ = e->slot_high_water();
    staged_bytes_ = e->streaming_staged_bytes();
}

// Forwards one call to the engine and refreshes the mirrored members.
#define KVTM_FORWARD(fail, call)                   \
    kvp::KVTileManager* e = engine_of(this);       \
    if (!e) return fail;                           \
    auto r = e->call;                              \
    kvp_sync_();                                   \
    return r

#define KVTM_FORWARD_VOID(call)                    \
    kvp::KVTileManager* e = engine_of(this);       \
    if (!e) return;                                \
    e->call;                                       \
    kvp_sync_()

bool KVTileManager::init() { KVTM_FORWARD(false, init()); }

KvtmResult KVTileManager::admit(long tile_id, void* ptr, size_t bytes) {
    KVTM_FORWARD(KVTM_INVALID, admit(tile_id, ptr, bytes));
}

bool KVTileManager::release(long tile_id) { KVTM_FORWARD(false, release(tile_id)); }

void KVTileManager::clear() { KVTM_FORWARD_VOID(clear()); }

int KVTileManager::persisted_tiles() const {
    const kvp::KVTileManager* e = engine_of(this);
    return e ? e->persisted_tiles() : 0;
}

bool KVTileManager::is_persisted(long tile_id) const {
    const kvp::KVTileManager* e = engine_of(this);
    return e ? e->is_persisted(tile_id) : false;
}

size_t KVTileManager::query_device_limit() const {
    const kvp::KVTileManager* e = engine_of(this);
    return e ? e->query_device_limit() : 0;
}

bool KVTileManager::arena_init(size_t capacity_bytes, size_t row_stride_floats) {
    KVTM_FORWARD(false, arena_init(capacity_bytes, row_stride_floats));
}

void KVTileManager::arena_begin_step() { KVTM_FORWARD_VOID(arena_begin_step()); }

bool KVTileManager::arena_stage(const void* k_dev, size_t k_bytes, const void* v_dev,
                                size_t v_bytes, long* out_row) {
    KVTM_FORWARD(false, arena_stage(k_dev, k_bytes, v_dev, v_bytes, out_row));
}

bool KVTileManager::arena_apply_window() { KVTM_FORWARD(false, arena_apply_window()); }

void KVTileManager::arena_end_step() { KVTM_FORWARD_VOID(arena_end_step()); }

bool KVTileManager::streaming_begin() { KVTM_FORWARD(false, streaming_begin()); }

bool KVTileManager::streaming_stage(long row_id, const void* k_dev, size_t k_bytes,
                                    const void* v_dev, size_t v_bytes, bool changed,
                                    long* out_slot, bool* restaged) {
    KVTM_FORWARD(false, streaming_stage(row_id, k_dev, k_bytes, v_dev, v_bytes, changed,
                                        out_slot, restaged));
}

bool KVTileManager::streaming_release(long row_id) {
    KVTM_FORWARD(false, streaming_release(row_id));
}

bool KVTileManager::streaming_apply_window() { KVTM_FORWARD(false, streaming_apply_window()); }

void KVTileManager::streaming_end() { KVTM_FORWARD_VOID(streaming_end()); }

#undef KVTM_FORWARD
#undef KVTM_FORWARD_VOID

// ------------------------------------------------------------ policies

void NoPersistencePolicy::select(const float* s, int n, int max_tiles, long* ids, int* count) {
    kvp::NoPersistencePolicy().select(s, n, max_tiles, ids, count);
}
const char* NoPersistencePolicy::name() const { return "none"; }

void UniformWindowPolicy::select(const float* s, int n, int max_tiles, long* ids, int* count) {
    kvp::UniformWindowPolicy().select(s, n, max_tiles, ids, count);
}
const char* UniformWindowPolicy::name() const { return "uniform"; }

void RecencyWindowPolicy::select(const float* s, int n, int max_tiles, long* ids, int* count) {
    kvp::RecencyWindowPolicy().select(s, n, max_tiles, ids, count);
}
const char* RecencyWindowPolicy::name() const { return "recency"; }

ReuseWeightedPolicy::ReuseWeightedPolicy(int tiles_per_frame, int total_frames)
    : tpf_(tiles_per_frame), total_frames_(total_frames) {}
void ReuseWeightedPolicy::select(const float* s, int n, int max_tiles, long* ids, int* count) {
    kvp::ReuseWeightedPolicy(tpf_, total_frames_).select(s, n, max_tiles, ids, count);
}
const char* ReuseWeightedPolicy::name() const { return "reuse_weighted"; }

void MotionGatedPolicy::select(const float* s, int n, int max_tiles, long* ids, int* count) {
    kvp::MotionGatedPolicy().select(s, n, max_tiles, ids, count);
}
const char* MotionGatedPolicy::name() const { return "motion"; }

// ------------------------------------------------------------ attention

void attn_forward_launcher(const float* d_q, const float* d_k, const float* d_v,
                           const float* d_arena, const long* d_kvmap, float* d_out, int frames,
                           int T, int D, int heads, bool remap) {
    kvp::fp32_launcher(d_q, d_k, d_v, d_arena, d_kvmap, d_out, frames, T, D, heads, remap);
}

void attn_forward_single_frame(const float* d_q_f, const float* d_k, const float* d_v,
                               const float* d_arena, const long* d_kvmap_f, float* d_out_f,
                               int T, int D, int heads, int cross, int frame_idx) {
    kvp::fp32_single_frame(d_q_f, d_k, d_v, d_arena, d_kvmap_f, d_out_f, T, D, heads, cross,
                           frame_idx);
}
