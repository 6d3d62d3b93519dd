// KVTileManager implementation (see kv_tile_manager.h).
//
// Accounting follows src/kv_tile_manager.cu:12-219 of the reference rule by
// rule; the per-method comments cite the lines each rule restates.
#include "kv_tile_manager.h"

#include <algorithm>
#include <cstring>
#include <mutex>

#include "kernels.h"
#include "kvp_common.h"

namespace kvp {

namespace {
std::mutex g_registry_mu;
std::vector<KVTileManager*> g_registry;
// The persisting limit seen before the first init(), restored when the last
// initialised manager goes away.
bool g_limit_saved = false;
size_t g_saved_limit = 0;
int g_live_initialised = 0;
}  // namespace

KVTileManager::KVTileManager(size_t budget_bytes, size_t max_window_bytes, unsigned flags)
    : budget_bytes_(budget_bytes), max_window_bytes_(max_window_bytes), flags_(flags) {
    std::lock_guard<std::mutex> g(g_registry_mu);
    g_registry.push_back(this);
}

KVTileManager::~KVTileManager() {
    // A caller may reset the device before destroying its manager (the
    // reference's driver calls cudaDeviceReset() at the end of main(), while
    // its manager is still in scope, src/run_policy_experiment.cu:315).  The
    // handles made in the destroyed context must not reach CUDA again: the
    // reset released them, and an event of a destroyed context faults the
    // driver.  The manager then only forgets them.
    if (!dry_run() && device_ >= 0 && !primary_context_active(device_)) {
        std::lock_guard<std::mutex> g(g_registry_mu);
        g_registry.erase(std::remove(g_registry.begin(), g_registry.end(), this), g_registry.end());
        if (initialized_ && --g_live_initialised == 0) g_limit_saved = false;
        return;
    }
    clear();
    flush();
    if (!dry_run()) {
        if (ops_done_) { cudaEventSynchronize(ops_done_); cudaEventDestroy(ops_done_); }
        if (d_ops_) cudaFree(d_ops_);
        if (h_ops_) cudaFreeHost(h_ops_);
        if (arena_) cudaFree(arena_);
    }
    std::lock_guard<std::mutex> g(g_registry_mu);
    g_registry.erase(std::remove(g_registry.begin(), g_registry.end(), this), g_registry.end());
    if (initialized_ && !dry_run() && --g_live_initialised == 0 && g_limit_saved) {
        cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, g_saved_limit);
        g_limit_saved = false;
    }
}

bool KVTileManager::init() {
    // :23-31 -- carve out the persisting set-aside; the budget is the limit.
    if (dry_run()) {
        saved_limit_ = budget_bytes_;
        initialized_ = true;
        return true;
    }
    {
        std::lock_guard<std::mutex> g(g_registry_mu);
        if (!g_limit_saved) {
            size_t cur = 0;
            if (cudaDeviceGetLimit(&cur, cudaLimitPersistingL2CacheSize) == cudaSuccess) {
                g_saved_limit = cur;
                g_limit_saved = true;
            }
        }
    }
    cudaError_t e = cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, budget_bytes_);
    if (e != cudaSuccess) {
        cuda_status(e, "cudaDeviceSetLimit(PersistingL2CacheSize)");
        return false;
    }
    if (!initialized_) {
        std::lock_guard<std::mutex> g(g_registry_mu);
        ++g_live_initialised;
    }
    initialized_ = true;
    return true;
}

size_t KVTileManager::query_device_limit() const {
    if (dry_run()) return initialized_ ? saved_limit_ : 0;
    size_t v = 0;
    cudaDeviceGetLimit(&v, cudaLimitPersistingL2CacheSize);
    return v;
}

void KVTileManager::apply_window(void* ptr, size_t bytes, cudaAccessProperty prop) {
    // :39-47 -- one access-policy window per stream, hitRatio 1, misses stream.
    if (window_log_.size() >= 4096) window_log_.erase(window_log_.begin());
    window_log_.push_back({ptr, bytes, (int)prop});
    if (dry_run()) return;
    cudaStreamAttrValue attr{};
    attr.accessPolicyWindow.base_ptr = ptr;
    attr.accessPolicyWindow.num_bytes = bytes;
    attr.accessPolicyWindow.hitRatio = 1.0f;
    attr.accessPolicyWindow.hitProp = prop;
    attr.accessPolicyWindow.missProp = cudaAccessPropertyStreaming;
    cudaError_t e = cudaStreamSetAttribute(stream_, cudaStreamAttributeAccessPolicyWindow, &attr);
    if (e != cudaSuccess) cuda_status(e, "cudaStreamSetAttribute(AccessPolicyWindow)");
}

void KVTileManager::reset_persisting() {
    ++reset_calls_;
    if (!dry_run()) cudaCtxResetPersistingL2Cache();
}

KvtmResult KVTileManager::admit(long tile_id, void* ptr, size_t bytes) {
    // :49-60 -- order of the checks decides INVALID vs REFUSED.
    if (!initialized_ || tile_id < 0 || ptr == nullptr || bytes == 0) return KVTM_INVALID;
    if (active_.count(tile_id)) return KVTM_INVALID;
    if (bytes > max_window_bytes_) return KVTM_INVALID;
    if (used_bytes_ + bytes > budget_bytes_) return KVTM_REFUSED_BUDGET;
    apply_window(ptr, bytes, cudaAccessPropertyPersisting);
    active_[tile_id] = {ptr, bytes};
    used_bytes_ += bytes;
    return KVTM_ADMITTED;
}

bool KVTileManager::release(long tile_id) {
    auto it = active_.find(tile_id);
    if (it == active_.end()) return false;
    apply_window(it->second.ptr, it->second.bytes, cudaAccessPropertyNormal);
    used_bytes_ -= it->second.bytes;
    active_.erase(it);
    return true;
}

void KVTileManager::clear() {
    if (active_.empty()) return;
    active_.clear();
    used_bytes_ = 0;
    reset_persisting();
}

// ---- arena mode ----------------------------------------------------------

bool KVTileManager::arena_init(size_t capacity_bytes, size_t row_stride_floats) {
    // :88-97
    if (arena_ready_) return false;
    if (!dry_run() && device_ < 0) cudaGetDevice(&device_);
    if (!dry_run() && cudaMalloc(&arena_, capacity_bytes) != cudaSuccess) {
        arena_ = nullptr;
        set_error("arena cudaMalloc(%zu) failed", capacity_bytes);
        return false;
    }
    arena_ready_ = true;
    arena_cap_ = capacity_bytes;
    arena_row_stride_floats_ = row_stride_floats;
    arena_next_row_ = 0;
    arena_used_ = 0;
    return true;
}

void KVTileManager::arena_begin_step() {
    arena_next_row_ = 0;
    arena_used_ = 0;
}

bool KVTileManager::arena_reserve(size_t total, long* out_row) {
    // :104-121 -- the byte gate against the budget, then against capacity.
    if (arena_used_ + total > budget_bytes_) return false;
    if (arena_used_ + total > arena_cap_) return false;
    *out_row = (long)arena_next_row_;
    ++arena_next_row_;
    arena_used_ += total;
    return true;
}

size_t KVTileManager::arena_reserve_rows(size_t total, size_t n, long* first_row) {
    // arena_reserve n times: each row passes while the bytes used stay within
    // both the budget and the capacity.
    *first_row = (long)arena_next_row_;
    const size_t lim = budget_bytes_ < arena_cap_ ? budget_bytes_ : arena_cap_;
    if (total == 0 || arena_used_ >= lim) return total == 0 ? n : 0;
    size_t k = (lim - arena_used_) / total;
    if (k > n) k = n;
    arena_next_row_ += k;
    arena_used_ += k * total;
    return k;
}

bool KVTileManager::arena_stage(const void* k_dev, size_t k_bytes, const void* v_dev,
                                size_t v_bytes, long* out_row) {
    long row = -1;
    if (!arena_reserve(k_bytes + v_bytes, &row)) return false;
    char* dst = (char*)arena_ + (size_t)row * row_stride_bytes();
    queue_copy(dst, k_dev, k_bytes);
    queue_copy(dst + k_bytes, v_dev, v_bytes);
    *out_row = row;
    return true;
}

size_t KVTileManager::arena_window_span() const {
    if (!initialized_ || arena_used_ == 0 || arena_used_ > max_window_bytes_) return 0;
    return arena_used_;
}

bool KVTileManager::arena_apply_window() {
    // :123-128.  The window is set before the queued copies run, so the
    // arena lines are written with the persisting property.
    const size_t span = arena_window_span();
    if (span) apply_window(arena_, span, cudaAccessPropertyPersisting);
    flush();
    return span != 0;
}

void KVTileManager::arena_end_step() {
    // :130-137
    flush();
    if (arena_used_ > 0) {
        apply_window(arena_, arena_used_, cudaAccessPropertyNormal);
        reset_persisting();
    }
    arena_next_row_ = 0;
    arena_used_ = 0;
}

// ---- streaming mode -------------------------------------------------------

bool KVTileManager::streaming_begin() {
    // :141-151 -- LIFO stack holding [cap-1 .. 0]; the first pop is slot 0.
    if (!arena_ready_) return false;
    row_slot_.clear();
    free_slots_.clear();
    const long cap_rows = (long)(arena_cap_ / row_stride_bytes());
    free_slots_.reserve((size_t)cap_rows);
    for (long s = cap_rows - 1; s >= 0; --s) free_slots_.push_back(s);
    slot_high_water_ = -1;
    staged_bytes_ = 0;
    return true;
}

bool KVTileManager::streaming_reserve(long row_id, size_t bytes_kv, bool changed, long* out_slot,
                                      bool* copy_needed, bool* was_held) {
    // :153-192 -- a sticky hit costs nothing unless the row changed.
    const long* held = row_slot_.find(row_id);
    if (was_held) *was_held = held != nullptr;
    if (held) {
        *out_slot = *held;
        if (!changed) { *copy_needed = false; return true; }
        staged_bytes_ += bytes_kv;
        *copy_needed = true;
        return true;
    }
    if (free_slots_.empty()) return false;
    const long slot = free_slots_.back();
    free_slots_.pop_back();
    row_slot_.put(row_id, slot);
    staged_bytes_ += bytes_kv;
    if (slot > slot_high_water_) slot_high_water_ = slot;
    *out_slot = slot;
    *copy_needed = true;
    return true;
}

bool KVTileManager::streaming_stage(long row_id, const void* k_dev, size_t k_bytes,
                                    const void* v_dev, size_t v_bytes, bool changed,
                                    long* out_slot, bool* restaged) {
    bool copy = false;
    if (!streaming_reserve(row_id, k_bytes + v_bytes, changed, out_slot, &copy)) return false;
    *restaged = copy;
    if (copy) {
        char* dst = (char*)arena_ + (size_t)(*out_slot) * row_stride_bytes();
        queue_copy(dst, k_dev, k_bytes);
        queue_copy(dst + k_bytes, v_dev, v_bytes);
    }
    return true;
}

bool KVTileManager::streaming_release(long row_id) {
    // :194-200 -- the freed slot goes back on top of the stack.
    const long* held = row_slot_.find(row_id);
    if (!held) return false;
    free_slots_.push_back(*held);
    row_slot_.erase(row_id);
    return true;
}

size_t KVTileManager::streaming_window_span() const {
    if (!initialized_ || slot_high_water_ < 0) return 0;
    const size_t span = ((size_t)slot_high_water_ + 1) * row_stride_bytes();
    return span > max_window_bytes_ ? 0 : span;
}

bool KVTileManager::streaming_apply_window() {
    // :202-210 -- the window spans slots [0, high-water].
    const size_t span = streaming_window_span();
    if (span) apply_window(arena_, span, cudaAccessPropertyPersisting);
    flush();
    return span != 0;
}

void KVTileManager::streaming_end() {
    // :212-219
    streaming_apply_window();
    apply_window(arena_, 1, cudaAccessPropertyNormal);
    reset_persisting();
    row_slot_.clear();
    free_slots_.clear();
    slot_high_water_ = -1;
}

// ---- batched staging copies -----------------------------------------------

void KVTileManager::queue_copy(void* dst, const void* src, size_t bytes) {
    // One flush runs its copies in parallel, while the reference's
    // cudaMemcpyAsync calls ran in stream order.  A later copy to the same
    // destination therefore replaces the queued one (the later write wins,
    // as in stream order); a partial overlap with a queued destination
    // issues the queue first.
    if (dry_run() || bytes == 0) return;
    const uintptr_t d0 = (uintptr_t)dst, d1 = d0 + bytes;
    for (CopyOp& op : pending_) {
        const uintptr_t o0 = (uintptr_t)op.dst, o1 = o0 + op.bytes;
        if (d1 <= o0 || o1 <= d0) continue;
        if (o0 == d0 && op.bytes == bytes) {
            op.src = src;
            return;
        }
        flush();
        break;
    }
    pending_.push_back({src, dst, (uint64_t)bytes});
}

int KVTileManager::flush() {
    if (pending_.empty() || dry_run()) return KVP_OK;
    if (device_ < 0) KVP_CUDA(cudaGetDevice(&device_));
    const size_t n = pending_.size();
    if (n > ops_cap_) {
        if (ops_done_) cudaEventSynchronize(ops_done_);
        if (d_ops_) cudaFree(d_ops_);
        if (h_ops_) cudaFreeHost(h_ops_);
        d_ops_ = nullptr;
        h_ops_ = nullptr;
        size_t cap = std::max<size_t>(n, 1024);
        KVP_CUDA(cudaMalloc(&d_ops_, cap * sizeof(CopyOp)));
        KVP_CUDA(cudaMallocHost(&h_ops_, cap * sizeof(CopyOp)));
        ops_cap_ = cap;
    }
    if (!ops_done_) KVP_CUDA(cudaEventCreateWithFlags(&ops_done_, cudaEventDisableTiming));
    // The pinned list may still feed the previous upload.
    KVP_CUDA(cudaEventSynchronize(ops_done_));
    std::memcpy(h_ops_, pending_.data(), n * sizeof(CopyOp));
    KVP_CUDA(cudaMemcpyAsync(d_ops_, h_ops_, n * sizeof(CopyOp), cudaMemcpyHostToDevice, stream_));
    int rc = launch_copy_batch(d_ops_, (int)n, stream_);
    KVP_CUDA(cudaEventRecord(ops_done_, stream_));
    pending_.clear();
    return rc;
}

int flush_all_managers() {
    std::lock_guard<std::mutex> g(g_registry_mu);
    int rc = KVP_OK;
    for (KVTileManager* m : g_registry) {
        int r = m->flush();
        if (r != KVP_OK) rc = r;
    }
    return rc;
}

}  // namespace kvp
