// C entry points around the reference's own policy and manager classes,
// compiled together with the reference's unmodified src/tile_gating_policy.cpp
// and src/kv_tile_manager.cu (host-only, see cuda_runtime.h beside this file).
//
// TEST INFRASTRUCTURE ONLY: these shims let ctypes-driven tests call the
// reference's TileGatingPolicy::select (src/tile_gating_policy.h:14-15) and
// run the reference's per-frame admission loop with a sliding frame window,
// which the reference driver (src/run_policy_experiment.cu:156-274) does not
// have.  With window == 0 the loop below is the reference driver's loop and
// its output is checked against the unmodified driver's event log.
#include "cuda_runtime.h"
#include "kv_tile_manager.h"
#include "tile_gating_policy.h"

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <memory>
#include <vector>

static TileGatingPolicy* make_policy(int policy, int tpf, int total_frames) {
    switch (policy) {
        case 0: return new NoPersistencePolicy();
        case 1: return new UniformWindowPolicy();
        case 2: return new RecencyWindowPolicy();
        case 3: return new MotionGatedPolicy();
        case 4: return new ReuseWeightedPolicy(tpf, total_frames);
        default: return nullptr;
    }
}

extern "C" int kvpref_select(int policy, const float* scores, int n, int max_tiles,
                             int tpf, int total_frames, long* out_ids, int* out_count) {
    std::unique_ptr<TileGatingPolicy> p(make_policy(policy, tpf, total_frames));
    if (!p) return -1;
    p->select(scores, n, max_tiles, out_ids, out_count);
    return 0;
}

// Per-frame admission loop with candidates restricted to frames
// [max(0, f-window+1), f].  Writes the uploaded KVMap slice per frame into
// map_out[frames][frames*tokens] (absolute row indexing, -1 elsewhere) and the
// streaming staged-byte counter per frame into staged_out[frames].
extern "C" int kvpref_run_window(int policy, int streaming, int window, int frames,
                                 int tokens, int hidden, int tile_tokens,
                                 long set_aside, const float* scores_flat,
                                 long* map_out, long* staged_out) {
    const long num_tiles = (tokens + tile_tokens - 1) / tile_tokens;
    const size_t elems = (size_t)frames * tokens * hidden;
    float* d_k = nullptr;
    float* d_v = nullptr;
    if (cudaMalloc(&d_k, elems * 4) != cudaSuccess) return -1;
    if (cudaMalloc(&d_v, elems * 4) != cudaSuccess) return -1;
    KVTileManager mgr((size_t)set_aside, (size_t)set_aside);
    cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, (size_t)set_aside);
    const size_t tile_bytes = (size_t)tile_tokens * hidden * 4 * 2;
    const long slots = (long)(set_aside / tile_bytes);
    if (!mgr.init() || !mgr.arena_init((size_t)set_aside, (size_t)hidden * 2)) return -2;
    std::vector<long> h_map((size_t)frames * tokens, -1L);
    std::vector<long> ids((size_t)frames * num_tiles + (size_t)slots + 1);
    std::vector<char> prev_selected;
    if (streaming) mgr.streaming_begin();
    for (long f = 0; f < frames; ++f) {
        const long base = window > 0 ? std::max(0L, f - window + 1) : 0;
        const int n_cand = (int)((f - base + 1) * num_tiles);
        std::unique_ptr<TileGatingPolicy> pol(
            make_policy(policy, (int)num_tiles, (int)(frames - base)));
        int count = 0;
        pol->select(scores_flat + base * num_tiles, n_cand, (int)slots, ids.data(), &count);
        std::vector<char> selected((size_t)((f + 1) * num_tiles), 0);
        std::vector<long> gids;
        for (int i = 0; i < count; ++i) {
            if (ids[i] < 0 || ids[i] >= n_cand) continue;  // Uniform may name ids past the candidates: nothing to stage
            const long gid = base * num_tiles + ids[i];
            selected[(size_t)gid] = 1;
            gids.push_back(gid);
        }
        if (streaming && f > 0) {
            for (long gid = 0; gid < (long)prev_selected.size(); ++gid) {
                if (!prev_selected[gid]) continue;
                if (gid < (long)selected.size() && selected[gid]) continue;
                const long src_f = gid / num_tiles, tile = gid % num_tiles;
                const long t0 = tile * tile_tokens;
                const long c = std::min((long)tile_tokens, (long)tokens - t0);
                for (long r = 0; r < c; ++r) mgr.streaming_release(src_f * tokens + t0 + r);
            }
        }
        mgr.arena_begin_step();
        std::fill(h_map.begin(), h_map.begin() + (f + 1) * tokens, -1L);
        for (long gid : gids) {
            const long src_f = gid / num_tiles, tile = gid % num_tiles;
            const long t0 = tile * tile_tokens;
            const long c = std::min((long)tile_tokens, (long)tokens - t0);
            bool all = true;
            for (long r = 0; r < c && all; ++r) {
                const long row_id = src_f * tokens + t0 + r;
                if (streaming) {
                    long slot = -1;
                    bool restaged = false;
                    all = mgr.streaming_stage(row_id, d_k + (size_t)row_id * hidden,
                                              (size_t)hidden * 4,
                                              d_v + (size_t)row_id * hidden,
                                              (size_t)hidden * 4, false, &slot, &restaged);
                    if (all) h_map[(size_t)row_id] = slot;
                } else {
                    long row = -1;
                    all = mgr.arena_stage(d_k + (size_t)row_id * hidden, (size_t)hidden * 4,
                                          d_v + (size_t)row_id * hidden, (size_t)hidden * 4,
                                          &row);
                    if (all) h_map[(size_t)row_id] = row;
                }
            }
        }
        long* dst = map_out + (size_t)f * frames * tokens;
        for (size_t i = 0; i < (size_t)frames * tokens; ++i) dst[i] = -1;
        for (long r = base * tokens; r < (f + 1) * tokens; ++r) dst[r] = h_map[(size_t)r];
        if (streaming) mgr.streaming_apply_window(); else mgr.arena_apply_window();
        staged_out[f] = streaming ? (long)mgr.streaming_staged_bytes() : (long)mgr.arena_used_bytes();
        if (streaming) prev_selected = selected; else mgr.arena_end_step();
    }
    if (streaming) mgr.streaming_end();
    cudaFree(d_k);
    cudaFree(d_v);
    return 0;
}

// Temporal-reuse streaming loop over the reference's KVTileManager: intra
// candidates (one frame's tiles), slot keys = token position t0+r, and
// streaming_stage(changed = !reuse[f][tile]) -- the reference driver always
// passes false (src/run_policy_experiment.cu:211).  Per frame: map_out
// [frames][tokens], copies (restaged == true), restaged (copies into a slot
// the key already held, tracked here), hits, staged bytes, window bytes
// (-1 when the window was refused).
#include <unordered_set>

extern "C" size_t kvpref_last_window_bytes(void);

extern "C" int kvpref_run_reuse(int policy, int frames, int tokens, int hidden, int tile_tokens,
                                long set_aside, const float* scores_flat,
                                const signed char* reuse_flat, long* map_out, int* copies_out,
                                int* restaged_out, int* hits_out, long* staged_out,
                                long* window_out) {
    const long num_tiles = (tokens + tile_tokens - 1) / tile_tokens;
    const size_t elems = (size_t)frames * tokens * hidden;
    float* d_k = nullptr;
    float* d_v = nullptr;
    if (cudaMalloc(&d_k, elems * 4) != cudaSuccess) return -1;
    if (cudaMalloc(&d_v, elems * 4) != cudaSuccess) return -1;
    KVTileManager mgr((size_t)set_aside, (size_t)set_aside);
    const size_t tile_bytes = (size_t)tile_tokens * hidden * 4 * 2;
    const long slots = (long)(set_aside / tile_bytes);
    if (!mgr.init() || !mgr.arena_init((size_t)set_aside, (size_t)hidden * 2)) return -2;
    std::unique_ptr<TileGatingPolicy> pol(make_policy(policy, (int)num_tiles, frames));
    if (!pol) return -3;
    std::vector<long> ids((size_t)num_tiles + (size_t)slots + 1);
    std::vector<char> prev_selected((size_t)num_tiles, 0);
    std::unordered_set<long> held;
    for (size_t i = 0; i < (size_t)frames * tokens; ++i) map_out[i] = -1;
    const bool persist = policy != 0;
    if (persist) mgr.streaming_begin();
    for (long f = 0; f < frames; ++f) {
        copies_out[f] = restaged_out[f] = hits_out[f] = 0;
        staged_out[f] = 0;
        window_out[f] = -1;
        if (!persist) continue;
        int count = 0;
        pol->select(scores_flat + f * num_tiles, (int)num_tiles, (int)slots, ids.data(), &count);
        std::vector<char> selected((size_t)num_tiles, 0);
        for (int i = 0; i < count; ++i)
            if (ids[i] >= 0 && ids[i] < num_tiles) selected[(size_t)ids[i]] = 1;
        if (f > 0) {
            for (long tile = 0; tile < num_tiles; ++tile) {
                if (!prev_selected[tile] || selected[tile]) continue;
                const long t0 = tile * tile_tokens;
                const long c = std::min((long)tile_tokens, (long)tokens - t0);
                for (long r = c - 1; r >= 0; --r)   // last row first: slots pop ascending
                    if (mgr.streaming_release(t0 + r)) held.erase(t0 + r);
            }
        }
        long* h_map = map_out + f * tokens;
        for (int i = 0; i < count; ++i) {
            if (ids[i] < 0 || ids[i] >= num_tiles) continue;
            const long tile = ids[i];
            const long t0 = tile * tile_tokens;
            const long c = std::min((long)tile_tokens, (long)tokens - t0);
            const bool changed = !(reuse_flat && reuse_flat[f * num_tiles + tile]);
            bool all = true;
            for (long r = 0; r < c && all; ++r) {
                const long row_id = f * tokens + t0 + r;
                long slot = -1;
                bool restaged = false;
                const bool was_held = held.count(t0 + r) != 0;
                all = mgr.streaming_stage(t0 + r, d_k + (size_t)row_id * hidden,
                                          (size_t)hidden * 4, d_v + (size_t)row_id * hidden,
                                          (size_t)hidden * 4, changed, &slot, &restaged);
                if (!all) break;
                held.insert(t0 + r);
                h_map[t0 + r] = slot;
                if (!restaged) { ++hits_out[f]; continue; }
                ++copies_out[f];
                if (was_held) ++restaged_out[f];
            }
        }
        if (mgr.streaming_apply_window())
            window_out[f] = (long)kvpref_last_window_bytes();
        staged_out[f] = (long)mgr.streaming_staged_bytes();
        prev_selected = selected;
    }
    if (persist) mgr.streaming_end();
    cudaFree(d_k);
    cudaFree(d_v);
    return 0;
}
