// Tile gating policies: which spatial tiles deserve persisting-L2 residency.
//
// Drop-in for the reference's TileGatingPolicy interface
// (src/tile_gating_policy.h:8-17): the same virtual select()/name() pair and
// the same five policies with the same selection rules.  Candidates are
// tile ids of one frame (intra) or frame-major ids g*tiles_per_frame+t over
// the key frames (cross).  Every rule below defines a total order, so the
// output is deterministic and bit-exact with the reference's stable sorts.
#pragma once

namespace kvp {

class TileGatingPolicy {
public:
    virtual ~TileGatingPolicy() {}
    // Writes at most max_tiles ids (Uniform: exactly max_tiles) and the count.
    virtual void select(const float* motion_scores, int num_tiles, int max_tiles,
                        long* out_ids, int* out_count) = 0;
    virtual const char* name() const = 0;
};

// Persist nothing (the unpinned baseline).
class NoPersistencePolicy : public TileGatingPolicy {
public:
    void select(const float*, int, int, long*, int* out_count) override;
    const char* name() const override { return "none"; }
};

// Ids 0..max_tiles-1 regardless of scores or of num_tiles (not clamped,
// as in the reference, src/tile_gating_policy.cpp:13-17).
class UniformWindowPolicy : public TileGatingPolicy {
public:
    void select(const float*, int, int max_tiles, long* out_ids, int* out_count) override;
    const char* name() const override { return "uniform"; }
};

// The newest max_tiles candidates: ids max(0, n-max_tiles) .. n-1.
class RecencyWindowPolicy : public TileGatingPolicy {
public:
    void select(const float*, int num_candidates, int max_tiles, long* out_ids,
                int* out_count) override;
    const char* name() const override { return "recency"; }
};

// priority = (total_frames - source_frame) * (1 - min(1, score / max_score)),
// max_score = max(1e-6f, max over candidates) in float, priority in double;
// highest priority first, ties by ascending id.
class ReuseWeightedPolicy : public TileGatingPolicy {
public:
    ReuseWeightedPolicy(int tiles_per_frame, int total_frames)
        : tpf_(tiles_per_frame), total_frames_(total_frames) {}
    void select(const float* scores_flat, int num_candidates, int max_tiles, long* out_ids,
                int* out_count) override;
    const char* name() const override { return "reuse_weighted"; }
    // Frames left to sweep, counted from the first candidate frame.
    void set_total_frames(int total_frames) { total_frames_ = total_frames; }

private:
    int tpf_;
    int total_frames_;
};

// Lowest motion first, ties by ascending tile id; min(max_tiles, n) ids.
class MotionGatedPolicy : public TileGatingPolicy {
public:
    void select(const float* motion_scores, int num_tiles, int max_tiles, long* out_ids,
                int* out_count) override;
    const char* name() const override { return "motion"; }
};

enum PolicyId { POLICY_NONE = 0, POLICY_UNIFORM = 1, POLICY_RECENCY = 2, POLICY_MOTION = 3,
                POLICY_REUSE_WEIGHTED = 4 };

// Factory; nullptr for an unknown id.
TileGatingPolicy* make_policy(int policy_id, int tiles_per_frame, int total_frames);

}  // namespace kvp
