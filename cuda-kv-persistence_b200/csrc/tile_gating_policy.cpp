// Gating policy selection rules (see tile_gating_policy.h).
//
// Ranking policies use std::partial_sort with a comparator that is a total
// order (score/priority, then id), which yields exactly the first max_tiles
// elements of the reference's std::stable_sort
// (src/tile_gating_policy.cpp:35-81) in O(n log k).
#include "tile_gating_policy.h"

#include <algorithm>
#include <numeric>
#include <vector>

namespace kvp {

void NoPersistencePolicy::select(const float*, int, int, long*, int* out_count) {
    *out_count = 0;
}

void UniformWindowPolicy::select(const float*, int, int max_tiles, long* out_ids,
                                 int* out_count) {
    const int n = max_tiles > 0 ? max_tiles : 0;
    for (int i = 0; i < n; ++i) out_ids[i] = i;
    *out_count = max_tiles;
}

void RecencyWindowPolicy::select(const float*, int num_candidates, int max_tiles,
                                 long* out_ids, int* out_count) {
    const int first = std::max(0, num_candidates - max_tiles);
    int n = 0;
    for (int id = first; id < num_candidates; ++id) out_ids[n++] = id;
    *out_count = n;
}

void ReuseWeightedPolicy::select(const float* scores, int n, int max_tiles, long* out_ids,
                                 int* out_count) {
    if (n <= 0) { *out_count = 0; return; }
    float peak = 1e-6f;
    for (int i = 0; i < n; ++i) peak = std::max(peak, scores[i]);
    const double peak_d = peak;
    std::vector<double> prio((size_t)n);
    for (int i = 0; i < n; ++i) {
        const double sweeps_left = (double)(total_frames_ - (long)i / tpf_);
        const double change = std::min(1.0, (double)scores[i] / peak_d);
        prio[(size_t)i] = sweeps_left * (1.0 - change);
    }
    std::vector<int> order((size_t)n);
    std::iota(order.begin(), order.end(), 0);
    const int k = std::max(0, std::min(max_tiles, n));
    auto before = [&](int a, int b) {
        if (prio[(size_t)a] != prio[(size_t)b]) return prio[(size_t)a] > prio[(size_t)b];
        return a < b;
    };
    std::partial_sort(order.begin(), order.begin() + k, order.end(), before);
    for (int i = 0; i < k; ++i) out_ids[i] = order[(size_t)i];
    *out_count = k;
}

void MotionGatedPolicy::select(const float* scores, int n, int max_tiles, long* out_ids,
                               int* out_count) {
    const int k = std::max(0, std::min(max_tiles, n));
    std::vector<int> order((size_t)std::max(n, 0));
    std::iota(order.begin(), order.end(), 0);
    auto before = [&](int a, int b) {
        if (scores[a] < scores[b]) return true;
        if (scores[b] < scores[a]) return false;
        return a < b;
    };
    std::partial_sort(order.begin(), order.begin() + k, order.end(), before);
    for (int i = 0; i < k; ++i) out_ids[i] = order[(size_t)i];
    *out_count = std::min(max_tiles, n);  // negative max_tiles passes through, as in the reference
}

TileGatingPolicy* make_policy(int policy_id, int tiles_per_frame, int total_frames) {
    switch (policy_id) {
        case POLICY_NONE: return new NoPersistencePolicy();
        case POLICY_UNIFORM: return new UniformWindowPolicy();
        case POLICY_RECENCY: return new RecencyWindowPolicy();
        case POLICY_MOTION: return new MotionGatedPolicy();
        case POLICY_REUSE_WEIGHTED: return new ReuseWeightedPolicy(tiles_per_frame, total_frames);
        default: return nullptr;
    }
}

}  // namespace kvp
