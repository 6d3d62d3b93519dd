// extern "C" boundary of libkvp.so.  Declarations and the reference
// interface each export replaces are in include/kv_tile_manager.h,
// include/attn_kernel.h and include/kvp.h.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>

#include "kernels.h"
#include "kv_tile_manager.h"
#include "kvp_common.h"
#include "motion_sm100.h"
#include "qkv_sm100.h"
#include "session.h"
#include "tile_gating_policy.h"
#include "tile_layout.h"

namespace kvp {

namespace {
thread_local char g_err[512] = "";
}  // namespace

// One device status word per device, allocated on first use.
int* status_word() {
    static int* words[64] = {nullptr};
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> g(mu);
    if (!words[dev]) {
        int* p = nullptr;
        if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
        if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) return nullptr;
        words[dev] = p;
    }
    return words[dev];
}

bool primary_context_active(int device) {
    typedef int (*DeviceGetFn)(int*, int);
    typedef int (*CtxStateFn)(int, unsigned*, int*);
    static DeviceGetFn device_get = nullptr;
    static CtxStateFn ctx_state = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuDeviceGet", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            device_get = reinterpret_cast<DeviceGetFn>(p);
        if (cudaGetDriverEntryPoint("cuDevicePrimaryCtxGetState", &p, cudaEnableDefault, &q) ==
                cudaSuccess && q == cudaDriverEntryPointSuccess)
            ctx_state = reinterpret_cast<CtxStateFn>(p);
    });
    if (!device_get || !ctx_state) return true;
    int dev = 0;
    if (device_get(&dev, device) != 0) return true;
    unsigned flags = 0;
    int active = 1;
    if (ctx_state(dev, &flags, &active) != 0) return true;
    return active != 0;
}

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}

const char* last_error() { return g_err; }

int cuda_status(cudaError_t e, const char* what) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return KVP_ERR_CUDA;
}

}  // namespace kvp

using kvp::KVTileManager;

// ===================================================================== kvtm_*
// Reference facade: src/kv_tile_manager.cu:223-339 (same names, argument
// meaning and return codes).

KVP_API void* kvtm_create(long budget_bytes, long max_window_bytes) {
    try {
        return new KVTileManager((size_t)budget_bytes, (size_t)max_window_bytes);
    } catch (...) {
        return nullptr;
    }
}
KVP_API void kvtm_destroy(void* m) { delete static_cast<KVTileManager*>(m); }
KVP_API int kvtm_init(void* m) { return static_cast<KVTileManager*>(m)->init() ? 1 : 0; }
KVP_API long kvtm_query_limit(void* m) {
    return (long)static_cast<KVTileManager*>(m)->query_device_limit();
}
KVP_API int kvtm_admit(void* m, long tile_id, void* ptr, long bytes) {
    return (int)static_cast<KVTileManager*>(m)->admit(tile_id, ptr, (size_t)bytes);
}
KVP_API int kvtm_release(void* m, long tile_id) {
    return static_cast<KVTileManager*>(m)->release(tile_id) ? 1 : 0;
}
KVP_API void kvtm_clear(void* m) { static_cast<KVTileManager*>(m)->clear(); }
KVP_API long kvtm_persisted_bytes(void* m) {
    return (long)static_cast<KVTileManager*>(m)->persisted_bytes();
}
KVP_API int kvtm_persisted_tiles(void* m) {
    return static_cast<KVTileManager*>(m)->persisted_tiles();
}
KVP_API void* kvtm_dev_alloc(long bytes) {
    void* p = nullptr;
    if (cudaMalloc(&p, (size_t)bytes) != cudaSuccess) return nullptr;
    return p;
}
KVP_API void kvtm_dev_free(void* p) { cudaFree(p); }

KVP_API int kvtm_arena_init(void* m, long cap_bytes, long row_stride_floats) {
    return static_cast<KVTileManager*>(m)->arena_init((size_t)cap_bytes, (size_t)row_stride_floats)
               ? 1 : 0;
}
KVP_API void kvtm_arena_begin(void* m) { static_cast<KVTileManager*>(m)->arena_begin_step(); }
KVP_API int kvtm_arena_stage(void* m, const void* k_dev, long k_bytes, const void* v_dev,
                             long v_bytes, long* out_row) {
    return static_cast<KVTileManager*>(m)->arena_stage(k_dev, (size_t)k_bytes, v_dev,
                                                       (size_t)v_bytes, out_row) ? 1 : 0;
}
KVP_API int kvtm_arena_window(void* m) {
    return static_cast<KVTileManager*>(m)->arena_apply_window() ? 1 : 0;
}
KVP_API void kvtm_arena_end(void* m) { static_cast<KVTileManager*>(m)->arena_end_step(); }
KVP_API long kvtm_arena_used(void* m) {
    return (long)static_cast<KVTileManager*>(m)->arena_used_bytes();
}
KVP_API void* kvtm_arena_ptr(void* m) { return static_cast<KVTileManager*>(m)->arena_device_ptr(); }

KVP_API int kvtm_streaming_begin(void* m) {
    return static_cast<KVTileManager*>(m)->streaming_begin() ? 1 : 0;
}
KVP_API int kvtm_streaming_stage(void* m, long row_id, const void* k_dev, long k_bytes,
                                 const void* v_dev, long v_bytes, int changed, long* out_slot,
                                 int* restaged) {
    bool r = false;
    long slot = -1;
    const int ok = static_cast<KVTileManager*>(m)->streaming_stage(
        row_id, k_dev, (size_t)k_bytes, v_dev, (size_t)v_bytes, changed != 0, &slot, &r);
    if (out_slot) *out_slot = slot;
    if (restaged) *restaged = r ? 1 : 0;
    return ok;
}
KVP_API int kvtm_streaming_release(void* m, long row_id) {
    return static_cast<KVTileManager*>(m)->streaming_release(row_id) ? 1 : 0;
}
KVP_API int kvtm_streaming_window(void* m) {
    return static_cast<KVTileManager*>(m)->streaming_apply_window() ? 1 : 0;
}
KVP_API void kvtm_streaming_end(void* m) { static_cast<KVTileManager*>(m)->streaming_end(); }
KVP_API long kvtm_streaming_staged_bytes(void* m) {
    return (long)static_cast<KVTileManager*>(m)->streaming_staged_bytes();
}

KVP_API long kvtm_layout_tiles_per_frame(int tokens_per_frame, int tile_tokens) {
    return kvp::TileLayout(tokens_per_frame, tile_tokens).tiles_per_frame;
}
KVP_API long kvtm_layout_tile_start(int tpf, int tt, long id) {
    return kvp::TileLayout(tpf, tt).tile_start(id);
}
KVP_API int kvtm_layout_tile_count(int tpf, int tt, long id) {
    return kvp::TileLayout(tpf, tt).tile_count(id);
}

// --- kvtm_* additions (no counterpart in the reference facade)
KVP_API void* kvtm_create_ex(long budget_bytes, long max_window_bytes, unsigned flags) {
    try {
        return new KVTileManager((size_t)budget_bytes, (size_t)max_window_bytes, flags);
    } catch (...) {
        return nullptr;
    }
}
KVP_API void kvtm_set_stream(void* m, void* stream) {
    static_cast<KVTileManager*>(m)->set_stream((cudaStream_t)stream);
}
KVP_API int kvtm_flush(void* m) { return static_cast<KVTileManager*>(m)->flush(); }
KVP_API long kvtm_pending_copies(void* m) {
    return (long)static_cast<KVTileManager*>(m)->pending_copies();
}
KVP_API long kvtm_window_log(void* m, long* bytes_out, int* prop_out, long cap) {
    const auto& log = static_cast<KVTileManager*>(m)->window_log();
    const long n = (long)log.size();
    for (long i = 0; i < n && i < cap; ++i) {
        if (bytes_out) bytes_out[i] = (long)log[(size_t)i].bytes;
        if (prop_out) prop_out[i] = log[(size_t)i].hit_prop;
    }
    return n;
}
KVP_API long kvtm_reset_calls(void* m) { return static_cast<KVTileManager*>(m)->reset_calls(); }

// ============================================================ attn_forward_*
// Reference entry points src/attn_kernel.h:15-29, C linkage here; the C++
// linkage pair the reference's own header declares is in cxx_abi.cpp.  Both
// forward to kvp::fp32_launcher / kvp::fp32_single_frame.

namespace kvp {

void fp32_launcher(const float* d_q, const float* d_k, const float* d_v, const float* d_arena,
                   const long* d_kvmap, float* d_out, int frames, int T, int D, int heads,
                   bool remap) {
    flush_all_managers();
    int* st = status_word();
    if (remap) {
        // Per-frame intra launches with per-frame map slices (legacy path).
        for (int f = 0; f < frames; ++f)
            launch_attn_fp32(d_q + (size_t)f * T * D, d_k + (size_t)f * T * D,
                             d_v + (size_t)f * T * D, d_arena,
                             d_kvmap ? (const int64_t*)d_kvmap + (size_t)f * T : nullptr,
                             d_out + (size_t)f * T * D, T, D, heads, 0, T, INT64_MAX, 1, 0, st,
                             0);
    } else {
        launch_attn_fp32(d_q, d_k, d_v, nullptr, nullptr, d_out, T, D, heads, 0, T, 0, frames,
                         T, st, 0);
    }
}

void fp32_single_frame(const float* d_q_f, const float* d_k, const float* d_v,
                       const float* d_arena, const long* d_kvmap_f, float* d_out_f, int T, int D,
                       int heads, int cross, int frame_idx) {
    flush_all_managers();
    const int64_t span = cross ? (int64_t)(frame_idx + 1) * T : (int64_t)T;
    launch_attn_fp32(d_q_f, d_k, d_v, d_arena, (const int64_t*)d_kvmap_f, d_out_f, T, D, heads,
                     0, span, INT64_MAX, 1, 0, status_word(), 0);
}

}  // namespace kvp

KVP_API void attn_forward_launcher(const float* d_q, const float* d_k, const float* d_v,
                                   const float* d_arena, const long* d_kvmap, float* d_out,
                                   int frames, int T, int D, int heads, bool remap) {
    kvp::fp32_launcher(d_q, d_k, d_v, d_arena, d_kvmap, d_out, frames, T, D, heads, remap);
}

KVP_API void attn_forward_single_frame(const float* d_q_f, const float* d_k, const float* d_v,
                                       const float* d_arena, const long* d_kvmap_f,
                                       float* d_out_f, int T, int D, int heads, int cross,
                                       int frame_idx) {
    kvp::fp32_single_frame(d_q_f, d_k, d_v, d_arena, d_kvmap_f, d_out_f, T, D, heads, cross,
                           frame_idx);
}

// ===================================================================== kvp_*

KVP_API const char* kvp_version(void) { return "kvp-b200 1.0 (sm_100a)"; }
KVP_API const char* kvp_last_error(void) { return kvp::last_error(); }

// Status word the kernels set on a recoverable device error (1 = KVMap entry
// outside the arena).  Reading it clears it.
KVP_API int kvp_read_status(void* stream) {
    int* w = kvp::status_word();
    if (!w) return kvp::KVP_ERR_CUDA;
    int h = 0;
    if (cudaMemcpyAsync(&h, w, sizeof(int), cudaMemcpyDeviceToHost, (cudaStream_t)stream) != cudaSuccess)
        return kvp::KVP_ERR_CUDA;
    if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return kvp::KVP_ERR_CUDA;
    if (h && cudaMemsetAsync(w, 0, sizeof(int), (cudaStream_t)stream) != cudaSuccess)
        return kvp::KVP_ERR_CUDA;
    return h;
}

struct kvp_device_info {
    int device;
    int sm_count;
    int cc_major, cc_minor;
    long long l2_bytes;
    long long max_persisting_l2_bytes;
    long long max_access_policy_window_bytes;
    long long persisting_limit_bytes;
    long long hbm_bytes;
};

KVP_API int kvp_query_device(int device, kvp_device_info* out) {
    if (!out) return kvp::KVP_ERR_ARG;
    std::memset(out, 0, sizeof *out);
    int dev = device;
    if (dev < 0) KVP_CUDA(cudaGetDevice(&dev));
    out->device = dev;
    int v = 0;
    KVP_CUDA(cudaDeviceGetAttribute(&out->sm_count, cudaDevAttrMultiProcessorCount, dev));
    KVP_CUDA(cudaDeviceGetAttribute(&out->cc_major, cudaDevAttrComputeCapabilityMajor, dev));
    KVP_CUDA(cudaDeviceGetAttribute(&out->cc_minor, cudaDevAttrComputeCapabilityMinor, dev));
    KVP_CUDA(cudaDeviceGetAttribute(&v, cudaDevAttrL2CacheSize, dev));
    out->l2_bytes = v;
    KVP_CUDA(cudaDeviceGetAttribute(&v, cudaDevAttrMaxPersistingL2CacheSize, dev));
    out->max_persisting_l2_bytes = v;
    KVP_CUDA(cudaDeviceGetAttribute(&v, cudaDevAttrMaxAccessPolicyWindowSize, dev));
    out->max_access_policy_window_bytes = v;
    size_t lim = 0;
    int cur = -1;
    KVP_CUDA(cudaGetDevice(&cur));
    if (cur == dev) {
        KVP_CUDA(cudaDeviceGetLimit(&lim, cudaLimitPersistingL2CacheSize));
        out->persisting_limit_bytes = (long long)lim;
    }
    size_t free_b = 0, total_b = 0;
    if (cur == dev && cudaMemGetInfo(&free_b, &total_b) == cudaSuccess) out->hbm_bytes = (long long)total_b;
    return kvp::KVP_OK;
}

// Policy selection through the C ABI: the reference's
// TileGatingPolicy::select (src/tile_gating_policy.h:14-15) by policy id
// (0 none, 1 uniform, 2 recency, 3 motion, 4 reuse_weighted).
KVP_API int tgp_select(int policy, const float* scores, int n, int max_tiles, int tiles_per_frame,
                       int total_frames, long* out_ids, int* out_count) {
    if (!out_count || (!out_ids && max_tiles > 0) || (!scores && n > 0 && policy >= 3))
        return kvp::KVP_ERR_ARG;
    kvp::TileGatingPolicy* p = kvp::make_policy(policy, tiles_per_frame > 0 ? tiles_per_frame : 1,
                                                total_frames);
    if (!p) return kvp::KVP_ERR_ARG;
    p->select(scores, n, max_tiles, out_ids, out_count);
    delete p;
    return kvp::KVP_OK;
}

KVP_API int kvp_read_motion_csv(const char* path, int frames, int num_tiles, float* scores,
                                signed char* reuse) {
    if (!path || !scores || frames <= 0 || num_tiles <= 0) return kvp::KVP_ERR_ARG;
    return kvp::read_motion_csv(path, frames, num_tiles, scores, (int8_t*)reuse);
}

// Gather staged rows of one layer: arena[pairs[i].slot] = K[pairs[i].row] || V[...].
KVP_API int kvp_stage_rows(const void* k, const void* v, void* arena, const int* d_pairs, int n,
                           long long row_bytes, void* stream) {
    kvp::GatherLayers L{};
    L.k[0] = k;
    L.v[0] = v;
    L.arena[0] = arena;
    return kvp::launch_gather_rows(L, 1, d_pairs, n, row_bytes, (cudaStream_t)stream);
}

// FP32 remapped attention over an explicit key-row span (intra, cross and
// sliding-window in one form).  Query rows [0, T) of q/out; key rows
// [k_lo, k_hi) of k/v with KVMap indexed by the absolute key row.
KVP_API int kvp_attn_fp32(const float* q, const float* k, const float* v, const float* arena,
                          const long long* kvmap, float* out, int T, int D, int heads,
                          long long k_lo, long long k_hi, long long arena_rows, void* stream) {
    int rc = kvp::flush_all_managers();
    if (rc != kvp::KVP_OK) return rc;
    int* st = kvp::status_word();
    if (!st) return kvp::KVP_ERR_CUDA;
    return kvp::launch_attn_fp32(q, k, v, arena, (const int64_t*)kvmap, out, T, D, heads, k_lo,
                                 k_hi, arena_rows < 0 ? INT64_MAX : arena_rows, 1, 0, st,
                                 (cudaStream_t)stream);
}

// ------------------------------------------------------------------ session

struct kvp_session_config {
    int mode, window, streaming, policy, frames, tokens, hidden, tile_tokens, elem_bytes, layers;
    long long set_aside;
};

struct kvp_step_info {
    int frame, sel_count, staged_tiles, copies;
    long long map_row0, map_rows, window_bytes, staged_bytes;
    int restaged, hits;
};

KVP_API void* kvp_session_create(const kvp_session_config* c) {
    if (!c) return nullptr;
    kvp::SessionConfig sc{c->mode, c->window, c->streaming, c->policy, c->frames, c->tokens,
                          c->hidden, c->tile_tokens, c->elem_bytes, c->layers, c->set_aside};
    kvp::Session* s = new (std::nothrow) kvp::Session(sc);
    if (!s) return nullptr;
    if (s->status() != kvp::KVP_OK) {
        delete s;
        return nullptr;
    }
    return s;
}
KVP_API void kvp_session_destroy(void* s) { delete static_cast<kvp::Session*>(s); }
KVP_API int kvp_session_plan_frame(void* s, int frame, const float* scores_flat) {
    return static_cast<kvp::Session*>(s)->plan_frame(frame, scores_flat);
}
KVP_API int kvp_session_plan_frame_reuse(void* s, int frame, const float* scores_flat,
                                         const signed char* reuse_flat) {
    return static_cast<kvp::Session*>(s)->plan_frame(frame, scores_flat,
                                                     reinterpret_cast<const int8_t*>(reuse_flat));
}
KVP_API int kvp_session_plan_stack(void* s, const float* scores_flat) {
    return static_cast<kvp::Session*>(s)->plan_stack(scores_flat);
}
KVP_API int kvp_session_finish(void* s) { return static_cast<kvp::Session*>(s)->finish(); }
KVP_API int kvp_session_info(void* s, kvp_step_info* out) {
    if (!out) return kvp::KVP_ERR_ARG;
    const kvp::SessionStepInfo& i = static_cast<kvp::Session*>(s)->info();
    out->frame = i.frame;
    out->sel_count = i.sel_count;
    out->staged_tiles = i.staged_tiles;
    out->copies = i.copies;
    out->map_row0 = i.map_row0;
    out->map_rows = i.map_rows;
    out->window_bytes = i.window_bytes;
    out->staged_bytes = i.staged_bytes;
    out->restaged = i.restaged;
    out->hits = i.hits;
    return kvp::KVP_OK;
}
KVP_API long long kvp_session_slots(void* s) { return static_cast<kvp::Session*>(s)->slots(); }
KVP_API long long kvp_session_cap_rows(void* s) { return static_cast<kvp::Session*>(s)->cap_rows(); }
// Copies map rows [row0, row0+n) of the host KVMap.
KVP_API int kvp_session_map(void* s, long long row0, long long n, long long* out) {
    kvp::Session* x = static_cast<kvp::Session*>(s);
    if (!out || row0 < 0 || n < 0 || row0 + n > x->map_len()) return kvp::KVP_ERR_ARG;
    std::memcpy(out, x->host_map() + row0, (size_t)n * sizeof(long long));
    return kvp::KVP_OK;
}
// Copies this step's (source row, arena slot) pairs; returns the count.
KVP_API int kvp_session_copies(void* s, int* pairs_out, int cap) {
    const auto& p = static_cast<kvp::Session*>(s)->pairs();
    const int n = (int)(p.size() / 2);
    if (pairs_out) std::memcpy(pairs_out, p.data(), sizeof(int) * 2 * (size_t)(n < cap ? n : cap));
    return n;
}
KVP_API int kvp_session_selected(void* s, long* ids_out, int cap) {
    const auto& v = static_cast<kvp::Session*>(s)->selected_ids();
    const int n = (int)v.size();
    if (ids_out) for (int i = 0; i < n && i < cap; ++i) ids_out[i] = v[(size_t)i];
    return n;
}
KVP_API long long* kvp_session_device_map(void* s) {
    return (long long*)static_cast<kvp::Session*>(s)->device_map();
}
KVP_API void* kvp_session_arena(void* s, int layer) {
    return static_cast<kvp::Session*>(s)->arena(layer);
}
KVP_API int kvp_session_upload(void* s, void* stream) {
    return static_cast<kvp::Session*>(s)->upload((cudaStream_t)stream);
}
KVP_API int kvp_session_stage(void* s, const void* const* k_layers, const void* const* v_layers,
                              void* stream) {
    return static_cast<kvp::Session*>(s)->stage(k_layers, v_layers, (cudaStream_t)stream);
}
KVP_API int kvp_session_stage_layer(void* s, int layer, const void* k, const void* v, void* stream) {
    return static_cast<kvp::Session*>(s)->stage_layer(layer, k, v, (cudaStream_t)stream);
}
KVP_API int kvp_session_window(void* s, int layer, void* stream) {
    return static_cast<kvp::Session*>(s)->apply_window(layer, (cudaStream_t)stream);
}
KVP_API int kvp_session_step(void* s, int frame, const float* scores_flat,
                             const signed char* reuse_flat, const void* const* k_layers,
                             const void* const* v_layers, int window_layer, void* stream) {
    return static_cast<kvp::Session*>(s)->step(frame, scores_flat,
                                                reinterpret_cast<const int8_t*>(reuse_flat),
                                                k_layers, v_layers, window_layer,
                                                (cudaStream_t)stream);
}
KVP_API int kvp_session_stage_except(void* s, const void* const* k_layers,
                                     const void* const* v_layers, long long skip_row0,
                                     long long skip_rows, void* stream) {
    return static_cast<kvp::Session*>(s)->stage(k_layers, v_layers, (cudaStream_t)stream, skip_row0,
                                                skip_rows);
}
KVP_API int kvp_session_produce(void* s, int layer, const void* x, const void* w, const float* bias,
                                void* q, void* k, void* v, long long row0, long long rows,
                                void* stream) {
    return static_cast<kvp::Session*>(s)->produce(layer, x, w, bias, q, k, v, row0, rows,
                                                  (cudaStream_t)stream);
}
KVP_API int kvp_session_clear_window(void* s, void* stream) {
    return static_cast<kvp::Session*>(s)->clear_window((cudaStream_t)stream);
}

// ------------------------------------------------ QKV producer, LayerNorm
struct kvp_qkv_io {
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
};

KVP_API int kvp_qkv_project_bf16(const kvp_qkv_io* io, void* stream) {
    if (!io) return kvp::KVP_ERR_ARG;
    kvp::QkvIO q{io->x, io->w, io->bias, io->q, io->k, io->v, io->arena, io->kvmap,
                 io->rows, io->map_row0, io->arena_rows, io->D};
    return kvp::launch_qkv_project_bf16(q, nullptr, (cudaStream_t)stream);
}

KVP_API int kvp_layernorm_bf16(const void* x, const float* gamma, const float* beta, void* y,
                               long long rows, int D, float eps, void* stream) {
    return kvp::launch_layernorm_bf16(x, gamma, beta, y, rows, D, eps, (cudaStream_t)stream);
}

// ------------------------------------------------------- motion producer
struct kvp_motion_params {
    int height, width, levels, winsize, iterations, poly_n;
    float poly_sigma, pyr_scale;
    int grid_rows, grid_cols, tile_cells;
};

KVP_API void* kvp_motion_create(const kvp_motion_params* p) {
    if (!p) return nullptr;
    kvp::MotionParams q{p->height, p->width, p->levels, p->winsize, p->iterations, p->poly_n,
                        p->poly_sigma, p->pyr_scale, p->grid_rows, p->grid_cols, p->tile_cells};
    auto* m = new (std::nothrow) kvp::MotionProducer(q);
    if (m && m->status() != kvp::KVP_OK) {
        delete m;
        return nullptr;
    }
    return m;
}
KVP_API void kvp_motion_destroy(void* m) { delete static_cast<kvp::MotionProducer*>(m); }
KVP_API int kvp_motion_tiles(void* m) { return static_cast<kvp::MotionProducer*>(m)->tiles(); }
KVP_API int kvp_motion_flow(void* m, const void* d_prev, const void* d_next, float* d_flow,
                            void* stream) {
    return static_cast<kvp::MotionProducer*>(m)->pair_flow(static_cast<const uint8_t*>(d_prev),
                                                           static_cast<const uint8_t*>(d_next),
                                                           d_flow, (cudaStream_t)stream);
}
KVP_API int kvp_motion_trace(void* m, const void* d_frames, int frames, float* d_change,
                             void* stream) {
    return static_cast<kvp::MotionProducer*>(m)->trace(static_cast<const uint8_t*>(d_frames), frames,
                                                       d_change, (cudaStream_t)stream);
}
KVP_API int kvp_motion_threshold(const float* change, int frames, int tiles, double percentile,
                                 signed char* reuse, signed char* is_static, double* tau) {
    return kvp::motion_threshold(change, frames, tiles, percentile,
                                 reinterpret_cast<int8_t*>(reuse),
                                 reinterpret_cast<int8_t*>(is_static), tau);
}

// --------------------------------------------------------- bf16 attention
// tcgen05 remapped attention for one layer (see include/kvp.h for the
// field meanings).  Staging copies queued by kvtm_* managers are issued
// first, so they precede the kernel as in the reference.
#include "attn_sm100.h"

struct kvp_layer_io {
    const void* q;
    const void* k;
    const void* v;
    void* out;
    const void* arena;
    const long long* kvmap;
    long long q_rows, kv_rows, arena_rows;
};

struct kvp_attn_desc {
    int tokens, frames, q_frame0, mode, window, heads, head_dim, head0, nheads, flat;
};

KVP_API int kvp_probe_bounded_wait(long long limit_ns, void* stream) {
    int* st = kvp::status_word();
    if (!st) return kvp::KVP_ERR_CUDA;
    return kvp::launch_bounded_wait_probe(limit_ns, st, (cudaStream_t)stream);
}

KVP_API int kvp_attn_bf16(const kvp_layer_io* io, const kvp_attn_desc* d, void* stream) {
    if (!io || !d) return kvp::KVP_ERR_ARG;
    kvp::LayerIO L{io->q, io->k, io->v, io->out, io->arena, io->kvmap,
                   io->q_rows, io->kv_rows, io->arena_rows};
    kvp::AttnDesc A{d->tokens, d->frames, d->q_frame0, d->mode, d->window,
                    d->heads, d->head_dim, d->head0, d->nheads, d->flat};
    // Bad arguments are reported before any device state is touched.
    int rc = kvp::check_attn_bf16(L, A);
    if (rc != kvp::KVP_OK) return rc;
    rc = kvp::flush_all_managers();
    if (rc != kvp::KVP_OK) return rc;
    int* st = kvp::status_word();
    if (!st) return kvp::KVP_ERR_CUDA;
    return kvp::launch_attn_bf16(L, A, st, (cudaStream_t)stream);
}

KVP_API int kvp_attn_bf16_multi(const kvp_layer_io* ios, const kvp_attn_desc* ds, int n,
                                void* stream) {
    if (!ios || !ds || n <= 0 || n > 4096) return kvp::KVP_ERR_ARG;
    std::vector<kvp::LayerIO> L((size_t)n);
    std::vector<kvp::AttnDesc> A((size_t)n);
    for (int i = 0; i < n; ++i) {
        const kvp_layer_io& io = ios[i];
        const kvp_attn_desc& d = ds[i];
        L[(size_t)i] = kvp::LayerIO{io.q, io.k, io.v, io.out, io.arena, io.kvmap,
                                    io.q_rows, io.kv_rows, io.arena_rows};
        A[(size_t)i] = kvp::AttnDesc{d.tokens, d.frames, d.q_frame0, d.mode, d.window,
                                     d.heads, d.head_dim, d.head0, d.nheads, d.flat};
        const int rc = kvp::check_attn_bf16(L[(size_t)i], A[(size_t)i]);
        if (rc != kvp::KVP_OK) return rc;
        if (d.tokens != ds[0].tokens || d.frames != ds[0].frames || d.mode != ds[0].mode ||
            d.window != ds[0].window || d.flat != ds[0].flat) {
            kvp::set_error("attn_bf16_multi: layer %d differs from layer 0 in tokens, frames, mode, "
                           "window or tiling", i);
            return kvp::KVP_ERR_ARG;
        }
    }
    // Bad arguments are reported above, before any device work.
    int rc = kvp::flush_all_managers();
    if (rc != kvp::KVP_OK) return rc;
    int* st = kvp::status_word();
    if (!st) return kvp::KVP_ERR_CUDA;
    return kvp::launch_attn_bf16_multi(L.data(), A.data(), n, st, (cudaStream_t)stream);
}

// The per-frame loop (kvp.h); Session::step, then the attention of the frame.
KVP_API int kvp_session_run_frames(void* sp, int f0, int nframes, const float* scores_flat,
                                   const signed char* reuse_flat, const kvp_layer_io* io,
                                   const kvp_attn_desc* d, void* stream) {
    auto* s = static_cast<kvp::Session*>(sp);
    if (!s || !io || !d || nframes <= 0 || f0 < 0) return kvp::KVP_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    kvp::LayerIO L{io->q, io->k, io->v, io->out, nullptr, nullptr, io->q_rows, io->kv_rows, 0};
    kvp::AttnDesc A{d->tokens, 1, f0, d->mode, d->window, d->heads, d->head_dim, d->head0,
                    d->nheads, 0};
    const bool persist = s->persists();
    if (persist) {
        L.kvmap = reinterpret_cast<const long long*>(s->device_map());
        L.arena = s->arena(0);
        L.arena_rows = s->cap_rows();
    }
    // Bad arguments are reported before any device work; the last frame's
    // rows bound every earlier frame's.
    A.q_frame0 = f0 + nframes - 1;
    int rc = kvp::check_attn_bf16(L, A);
    if (rc != kvp::KVP_OK) return rc;
    int* status = kvp::status_word();
    if (!status) return kvp::KVP_ERR_CUDA;
    const void* kl[1] = {io->k};
    const void* vl[1] = {io->v};
    for (int f = f0; f < f0 + nframes; ++f) {
        rc = s->step(f, scores_flat, reinterpret_cast<const int8_t*>(reuse_flat), kl, vl, 0, st);
        if (rc != kvp::KVP_OK) return rc;
        A.q_frame0 = f;
        rc = kvp::launch_attn_bf16(L, A, status, st);
        if (rc != kvp::KVP_OK) return rc;
    }
    return persist ? s->clear_window(st) : kvp::KVP_OK;
}

// The dense-arena per-frame loop with every frame's attention in one grid
// (kvp.h): admission needs nothing from the device, so all frames are
// planned first, frame i staged into arena i with its own KVMap slice.
KVP_API int kvp_session_run_frames_batched(void* sp, int f0, int nframes, const float* scores_flat,
                                           const kvp_layer_io* io, const kvp_attn_desc* d,
                                           long long* maps, void* stream) {
    auto* s = static_cast<kvp::Session*>(sp);
    if (!s || !io || !d || nframes <= 0 || f0 < 0) return kvp::KVP_ERR_ARG;
    const kvp::SessionConfig& c = s->config();
    const bool persist = s->persists();
    if (c.mode != kvp::MODE_INTRA && c.mode != kvp::MODE_CROSS) {
        kvp::set_error("run_frames_batched: needs an intra or cross session");
        return kvp::KVP_ERR_ARG;
    }
    if (f0 + nframes > c.frames) {
        kvp::set_error("run_frames_batched: frames [%d, %d) past the session's %d", f0, f0 + nframes,
                       c.frames);
        return kvp::KVP_ERR_ARG;
    }
    if (persist && (c.streaming || c.layers < nframes || !maps)) {
        kvp::set_error("run_frames_batched: needs dense arenas (streaming 0), one per frame "
                       "(layers %d < %d frames), and a device map buffer", c.layers, nframes);
        return kvp::KVP_ERR_ARG;
    }
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t map_len = s->map_len();
    // With the arenas back to back, every frame's map indexes them as one
    // arena from arena(0) (kvp::Session::stage_batched): all segments then
    // share their tensors, and one gather per chunk stages its frames.
    const int64_t stride = persist ? s->arena_stride_rows() : 0;
    // Frames go in chunks of at most one launch's segments, in frame order:
    // a chunk is planned, staged and launched, and the device runs it while
    // the host plans the next.  Within a chunk the longest key span comes
    // first: entry c0 + j of chunk [c0, c0 + cnt) is frame c0 + cnt - 1 - j.
    const int chunks = (nframes + kvp::kAttnSegsPerLaunch - 1) / kvp::kAttnSegsPerLaunch;
    const int per = (nframes + chunks - 1) / chunks;
    std::vector<kvp::LayerIO> L((size_t)nframes);
    std::vector<kvp::AttnDesc> A((size_t)nframes);
    for (int c0 = 0; c0 < nframes; c0 += per) {
        const int cnt = std::min(per, nframes - c0);
        for (int j = 0; j < cnt; ++j) {
            const int fi = c0 + cnt - 1 - j;   // frame index within the call
            kvp::LayerIO& l = L[(size_t)(c0 + j)];
            l = kvp::LayerIO{io->q, io->k, io->v, io->out, nullptr, nullptr, io->q_rows, io->kv_rows, 0};
            if (persist) {
                l.kvmap = reinterpret_cast<const long long*>(maps + (size_t)fi * (size_t)map_len);
                l.arena = s->arena(stride > 0 ? 0 : fi);
                l.arena_rows = stride > 0 ? (long long)nframes * stride : s->cap_rows();
            }
            kvp::AttnDesc& a = A[(size_t)(c0 + j)];
            a = kvp::AttnDesc{d->tokens, 1, f0 + fi, d->mode, d->window, d->heads, d->head_dim,
                              d->head0, d->nheads, 0};
            const int rc = kvp::check_attn_bf16(l, a);
            if (rc != kvp::KVP_OK) return rc;
        }
    }
    // Bad arguments are reported above, before any device work.
    int* status = kvp::status_word();
    if (!status) return kvp::KVP_ERR_CUDA;
    int rc = kvp::KVP_OK;
    for (int c0 = 0; c0 < nframes; c0 += per) {
        const int cnt = std::min(per, nframes - c0);
        if (stride > 0) {
            rc = s->stage_batched(f0 + c0, cnt, c0, scores_flat, io->k, io->v,
                                  reinterpret_cast<int64_t*>(maps), st);
            if (rc != kvp::KVP_OK) return rc;
        } else {
            for (int i = c0; i < c0 + cnt; ++i) {
                rc = s->plan_frame(f0 + i, scores_flat);
                if (rc != kvp::KVP_OK) return rc;
                if (!persist) continue;
                if ((rc = s->upload_to(reinterpret_cast<int64_t*>(maps) + (size_t)i * (size_t)map_len, st)) !=
                    kvp::KVP_OK)
                    return rc;
                if ((rc = s->stage_layer(i, io->k, io->v, st)) != kvp::KVP_OK) return rc;
            }
        }
        if (persist && (rc = s->apply_window(c0 + cnt - 1, st)) != kvp::KVP_OK) return rc;
        rc = kvp::launch_attn_bf16_multi(L.data() + c0, A.data() + c0, cnt, status, st);
        if (rc != kvp::KVP_OK) return rc;
    }
    return persist ? s->clear_window(st) : kvp::KVP_OK;
}
