// Gating policy selection rules (see tile_gating_policy.h).
//
// Ranking policies take the first max_tiles records under a comparator that
// is a total order (score/priority, then id) with nth_element + sort, which
// yields exactly the first max_tiles elements of the reference's
// std::stable_sort (src/tile_gating_policy.cpp:35-81) in O(n + k log k).
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

namespace {

// The first k records under `before` (a strict total order), in order:
// nth_element then a sort of the head -- O(n + k log k), and the same ids as
// the reference's full std::stable_sort because ties are broken by id.
template <class Rec, class Less>
void first_k(std::vector<Rec>& recs, int k, Less before) {
    if (k < (int)recs.size())
        std::nth_element(recs.begin(), recs.begin() + k, recs.end(), before);
    std::sort(recs.begin(), recs.begin() + k, before);
}

}  // namespace

void ReuseWeightedPolicy::select(const float* scores, int n, int max_tiles, long* out_ids,
                                 int* out_count) {
    if (n <= 0) { *out_count = 0; return; }
    float peak = 1e-6f;
    for (int i = 0; i < n; ++i) peak = std::max(peak, scores[i]);
    const double peak_d = peak;
    struct Rec { double prio; int id; };
    std::vector<Rec> recs((size_t)n);
    for (int i = 0; i < n; ++i) {
        const double sweeps_left = (double)(total_frames_ - (long)i / tpf_);
        const double change = std::min(1.0, (double)scores[i] / peak_d);
        recs[(size_t)i] = {sweeps_left * (1.0 - change), i};
    }
    const int k = std::max(0, std::min(max_tiles, n));
    first_k(recs, k, [](const Rec& a, const Rec& b) {
        if (a.prio != b.prio) return a.prio > b.prio;
        return a.id < b.id;
    });
    for (int i = 0; i < k; ++i) out_ids[i] = recs[(size_t)i].id;
    *out_count = k;
}

void MotionGatedPolicy::select(const float* scores, int n, int max_tiles, long* out_ids,
                               int* out_count) {
    const int k = std::max(0, std::min(max_tiles, n));
    struct Rec { float score; int id; };
    std::vector<Rec> recs((size_t)std::max(n, 0));
    for (int i = 0; i < n; ++i) recs[(size_t)i] = {scores[i], i};
    // ascending score, ties (and unordered NaN pairs) by id
    first_k(recs, k, [](const Rec& a, const Rec& b) {
        if (a.score < b.score) return true;
        if (b.score < a.score) return false;
        return a.id < b.id;
    });
    for (int i = 0; i < k; ++i) out_ids[i] = recs[(size_t)i].id;
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
