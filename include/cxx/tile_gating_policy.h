/* libkvp.so: the C++ tile gating policies, for callers compiled against the
 * reference's C++ interface.
 *
 * Drop-in for GauthamMK-0/cuda-kv-persistence src/tile_gating_policy.h:8-68:
 * the same abstract TileGatingPolicy and the same five classes with the same
 * constructors and layout.  select() and name() are defined in libkvp.so
 * (so are the classes' vtables and type information) and give the ids the C
 * wrapper tgp_select gives, which are bit-exact with the reference's rules.
 */
#ifndef KVP_CXX_TILE_GATING_POLICY_H
#define KVP_CXX_TILE_GATING_POLICY_H

#define KVP_CXX_API __attribute__((visibility("default")))

/* src/tile_gating_policy.h:8-17 */
class KVP_CXX_API TileGatingPolicy {
public:
    virtual ~TileGatingPolicy() {}
    /* Writes up to max_tiles candidate ids and their count. */
    virtual void select(const float* motion_scores, int num_tiles, int max_tiles,
                        long* out_ids, int* out_count) = 0;
    virtual const char* name() const = 0;
};

/* Persists nothing ("none"). */
class KVP_CXX_API NoPersistencePolicy : public TileGatingPolicy {
public:
    void select(const float*, int, int, long*, int* out_count) override;
    const char* name() const override;
};

/* Ids 0 .. max_tiles-1, whatever the scores ("uniform"). */
class KVP_CXX_API UniformWindowPolicy : public TileGatingPolicy {
public:
    void select(const float*, int, int max_tiles, long* out_ids, int* out_count) override;
    const char* name() const override;
};

/* The newest max_tiles of the frame-major candidates ("recency"). */
class KVP_CXX_API RecencyWindowPolicy : public TileGatingPolicy {
public:
    void select(const float*, int num_candidates, int max_tiles, long* out_ids,
                int* out_count) override;
    const char* name() const override;
};

/* Highest (frames left to sweep) x (1 - normalised score) first
 * ("reuse_weighted"). */
class KVP_CXX_API ReuseWeightedPolicy : public TileGatingPolicy {
public:
    ReuseWeightedPolicy(int tiles_per_frame, int total_frames);
    void select(const float* scores_flat, int num_candidates, int max_tiles, long* out_ids,
                int* out_count) override;
    const char* name() const override;

private:
    int tpf_;
    int total_frames_;
};

/* Lowest motion first, ties by id ("motion"). */
class KVP_CXX_API MotionGatedPolicy : public TileGatingPolicy {
public:
    void select(const float* motion_scores, int num_tiles, int max_tiles, long* out_ids,
                int* out_count) override;
    const char* name() const override;
};

#endif
