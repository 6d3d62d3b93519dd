/* CPU oracle: plain-C restatement of the reference's admission path.
 *
 * TEST INFRASTRUCTURE ONLY (see kvp_oracle.h).  Byte quantities use uint64_t
 * arithmetic because the reference keeps them in size_t.  Floating point is
 * plain IEEE single/double with no contraction, as in the reference's
 * host code.
 */
#include "kvp_oracle.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ layout */
/* src/tile_layout.h:19-29 */
int64_t orc_tiles_per_frame(int tpf, int tt) { return (int64_t)((tpf + tt - 1) / tt); }
int64_t orc_tile_start(int tpf, int tt, int64_t id) { (void)tpf; return id * tt; }
int orc_tile_count(int tpf, int tt, int64_t id) {
    int64_t s = id * tt;
    int64_t rem = (int64_t)tpf - s;
    return (int)(rem < tt ? rem : tt);
}

/* ---------------------------------------------------------------- policies */
typedef struct { int64_t id; double prio; } orc_cand;

static int cmp_reuse(const void* a, const void* b) {
    /* src/tile_gating_policy.cpp:56-60: priority descending, then id ascending */
    const orc_cand* x = (const orc_cand*)a;
    const orc_cand* y = (const orc_cand*)b;
    if (x->prio > y->prio) return -1;
    if (x->prio < y->prio) return 1;
    return (x->id < y->id) ? -1 : (x->id > y->id);
}

typedef struct { int idx; float score; } orc_scored;

static int cmp_motion(const void* a, const void* b) {
    /* src/tile_gating_policy.cpp:72-76: stable sort by score ascending, so
     * equal scores keep index order */
    const orc_scored* x = (const orc_scored*)a;
    const orc_scored* y = (const orc_scored*)b;
    if (x->score < y->score) return -1;
    if (y->score < x->score) return 1;
    return (x->idx < y->idx) ? -1 : (x->idx > y->idx);
}

int orc_select(int policy, const float* scores, int n, int max_tiles, int tpf,
               int total_frames, int64_t* out_ids, int* out_count) {
    switch (policy) {
    case ORC_NONE: /* :6-9 */
        *out_count = 0;
        return 0;
    case ORC_UNIFORM: /* :13-17, ids are not clamped to n */
        for (int i = 0; i < max_tiles; ++i) out_ids[i] = i;
        *out_count = max_tiles;
        return 0;
    case ORC_RECENCY: { /* :21-28 */
        int c = 0;
        for (int i = (n - max_tiles > 0 ? n - max_tiles : 0); i < n; ++i) out_ids[c++] = i;
        *out_count = c;
        return 0;
    }
    case ORC_REUSE: { /* :35-66 */
        float max_rate = 1e-6f;
        for (int i = 0; i < n; ++i)
            if (max_rate < scores[i]) max_rate = scores[i];
        const double max_rate_d = (double)max_rate;
        orc_cand* c = (orc_cand*)malloc(sizeof(orc_cand) * (size_t)(n > 0 ? n : 1));
        if (!c) return -1;
        for (int i = 0; i < n; ++i) {
            const int64_t src_f = (int64_t)i / tpf;
            const double remaining = (double)(total_frames - src_f);
            const double q = (double)scores[i] / max_rate_d;
            const double rate = (q < 1.0) ? q : 1.0; /* std::min(1.0, q) */
            c[i].id = i;
            c[i].prio = remaining * (1.0 - rate);
        }
        qsort(c, (size_t)n, sizeof(orc_cand), cmp_reuse);
        int k = 0;
        for (int i = 0; i < n && k < max_tiles; ++i) out_ids[k++] = c[i].id;
        *out_count = k;
        free(c);
        return 0;
    }
    case ORC_MOTION: { /* :70-81 */
        orc_scored* o = (orc_scored*)malloc(sizeof(orc_scored) * (size_t)(n > 0 ? n : 1));
        if (!o) return -1;
        for (int i = 0; i < n; ++i) { o[i].idx = i; o[i].score = scores[i]; }
        qsort(o, (size_t)n, sizeof(orc_scored), cmp_motion);
        const int k = max_tiles < n ? max_tiles : n;
        for (int i = 0; i < k; ++i) out_ids[i] = o[i].idx;
        *out_count = k > 0 ? k : 0;
        free(o);
        return 0;
    }
    default:
        return -1;
    }
}

/* ------------------------------------------------------ int64 -> int64 map */
typedef struct { int64_t* keys; int64_t* vals; uint8_t* used; size_t cap, n, tombs; } orc_hmap;

static size_t hm_hash(int64_t k, size_t cap) {
    uint64_t x = (uint64_t)k * 0x9E3779B97F4A7C15ull;
    return (size_t)(x >> 17) & (cap - 1);
}
static void hm_free(orc_hmap* h) { free(h->keys); free(h->vals); free(h->used); memset(h, 0, sizeof *h); }
static int hm_init(orc_hmap* h, size_t cap) {
    size_t c = 16;
    while (c < cap * 2) c <<= 1;
    h->keys = (int64_t*)calloc(c, sizeof(int64_t));
    h->vals = (int64_t*)calloc(c, sizeof(int64_t));
    h->used = (uint8_t*)calloc(c, 1);
    h->cap = c; h->n = 0; h->tombs = 0;
    return (h->keys && h->vals && h->used) ? 0 : -1;
}
static int hm_find(const orc_hmap* h, int64_t k, int64_t* v) {
    if (!h->cap) return 0;
    for (size_t i = hm_hash(k, h->cap);; i = (i + 1) & (h->cap - 1)) {
        if (!h->used[i]) return 0;
        if (h->used[i] == 1 && h->keys[i] == k) { if (v) *v = h->vals[i]; return 1; }
    }
}
static int hm_put(orc_hmap* h, int64_t k, int64_t v);
static int hm_grow(orc_hmap* h) {
    orc_hmap old = *h;
    if (hm_init(h, 2 * (old.n + 1)) != 0) return -1;
    for (size_t i = 0; i < old.cap; ++i)
        if (old.used[i] == 1) hm_put(h, old.keys[i], old.vals[i]);
    hm_free(&old);
    return 0;
}
static int hm_put(orc_hmap* h, int64_t k, int64_t v) {
    if (!h->cap && hm_init(h, 64) != 0) return -1;
    /* rehash when live entries plus tombstones fill half the table, so a
     * probe always reaches an empty slot */
    if ((h->n + h->tombs + 1) * 2 > h->cap && hm_grow(h) != 0) return -1;
    size_t tomb = (size_t)-1;
    for (size_t i = hm_hash(k, h->cap);; i = (i + 1) & (h->cap - 1)) {
        if (h->used[i] == 1 && h->keys[i] == k) { h->vals[i] = v; return 0; }
        if (h->used[i] == 2 && tomb == (size_t)-1) tomb = i;
        if (!h->used[i]) {
            size_t j = tomb != (size_t)-1 ? tomb : i;
            if (j == tomb) --h->tombs;
            h->used[j] = 1; h->keys[j] = k; h->vals[j] = v; ++h->n;
            return 0;
        }
    }
}
static int hm_erase(orc_hmap* h, int64_t k) {
    if (!h->cap) return 0;
    for (size_t i = hm_hash(k, h->cap);; i = (i + 1) & (h->cap - 1)) {
        if (!h->used[i]) return 0;
        if (h->used[i] == 1 && h->keys[i] == k) { h->used[i] = 2; --h->n; ++h->tombs; return 1; }
    }
}
static void hm_clear(orc_hmap* h) { if (h->cap) memset(h->used, 0, h->cap); h->n = 0; h->tombs = 0; }

/* ----------------------------------------------------------------- manager */
struct orc_mgr {
    uint64_t budget, max_window, used, limit;
    int initialized;
    orc_hmap active_bytes; /* tile id -> bytes (src/kv_tile_manager.h:69-74) */
    int has_arena;
    uint64_t arena_cap, stride_floats, next_row, arena_used;
    orc_hmap row_slot;
    int64_t* free_slots; size_t n_free, cap_free;
    int64_t high_water;
    uint64_t staged;
    int64_t last_win_bytes; int last_win_prop;
    int64_t win_calls, reset_calls;
};

static void apply_window(orc_mgr* m, uint64_t bytes, int prop) {
    /* src/kv_tile_manager.cu:39-47 (one window per stream) */
    m->last_win_bytes = (int64_t)bytes;
    m->last_win_prop = prop;
    ++m->win_calls;
}

orc_mgr* orc_mgr_create(int64_t budget, int64_t max_window) {
    orc_mgr* m = (orc_mgr*)calloc(1, sizeof(orc_mgr));
    if (!m) return NULL;
    m->budget = (uint64_t)budget;
    m->max_window = (uint64_t)max_window;
    m->high_water = -1;
    m->last_win_bytes = -1;
    return m;
}
void orc_mgr_destroy(orc_mgr* m) {
    if (!m) return;
    hm_free(&m->active_bytes); hm_free(&m->row_slot); free(m->free_slots); free(m);
}
int orc_mgr_init(orc_mgr* m) { m->limit = m->budget; m->initialized = 1; return 1; }
int64_t orc_mgr_query_limit(orc_mgr* m) { return (int64_t)m->limit; }

int orc_mgr_admit(orc_mgr* m, int64_t tile_id, uint64_t ptr, int64_t bytes) {
    /* src/kv_tile_manager.cu:49-60 */
    const uint64_t b = (uint64_t)bytes;
    if (!m->initialized || tile_id < 0 || ptr == 0 || b == 0) return -1;
    if (hm_find(&m->active_bytes, tile_id, NULL)) return -1;
    if (b > m->max_window) return -1;
    if (m->used + b > m->budget) return 0;
    apply_window(m, b, 2);
    hm_put(&m->active_bytes, tile_id, (int64_t)b);
    m->used += b;
    return 1;
}
int orc_mgr_release(orc_mgr* m, int64_t tile_id) {
    int64_t b;
    if (!hm_find(&m->active_bytes, tile_id, &b)) return 0;
    apply_window(m, (uint64_t)b, 0);
    m->used -= (uint64_t)b;
    hm_erase(&m->active_bytes, tile_id);
    return 1;
}
void orc_mgr_clear(orc_mgr* m) {
    if (m->active_bytes.n == 0) return;
    hm_clear(&m->active_bytes);
    m->used = 0;
    ++m->reset_calls;
}
int64_t orc_mgr_persisted_bytes(orc_mgr* m) { return (int64_t)m->used; }
int orc_mgr_persisted_tiles(orc_mgr* m) { return (int)m->active_bytes.n; }

int orc_mgr_arena_init(orc_mgr* m, int64_t cap_bytes, int64_t row_stride_floats) {
    /* :88-97 */
    if (m->has_arena) return 0;
    m->has_arena = 1;
    m->arena_cap = (uint64_t)cap_bytes;
    m->stride_floats = (uint64_t)row_stride_floats;
    m->next_row = 0;
    m->arena_used = 0;
    return 1;
}
void orc_mgr_arena_begin(orc_mgr* m) { m->next_row = 0; m->arena_used = 0; }
int orc_mgr_arena_stage(orc_mgr* m, int64_t kb, int64_t vb, int64_t* out_row) {
    /* :104-121 */
    const uint64_t total = (uint64_t)kb + (uint64_t)vb;
    if (m->arena_used + total > m->budget) return 0;
    if (m->arena_used + total > m->arena_cap) return 0;
    *out_row = (int64_t)m->next_row;
    ++m->next_row;
    m->arena_used += total;
    return 1;
}
int orc_mgr_arena_window(orc_mgr* m) {
    if (!m->initialized || m->arena_used == 0 || m->arena_used > m->max_window) return 0;
    apply_window(m, m->arena_used, 2);
    return 1;
}
void orc_mgr_arena_end(orc_mgr* m) {
    if (m->arena_used > 0) { apply_window(m, m->arena_used, 0); ++m->reset_calls; }
    m->next_row = 0;
    m->arena_used = 0;
}
int64_t orc_mgr_arena_used(orc_mgr* m) { return (int64_t)m->arena_used; }

int orc_mgr_streaming_begin(orc_mgr* m) {
    /* :141-151: LIFO stack [cap-1 .. 0], so the first pop is slot 0 */
    if (!m->has_arena) return 0;
    hm_clear(&m->row_slot);
    const uint64_t row_bytes = m->stride_floats * 4u;
    const int64_t cap_rows = row_bytes ? (int64_t)(m->arena_cap / row_bytes) : 0;
    if ((size_t)cap_rows > m->cap_free) {
        free(m->free_slots);
        m->free_slots = (int64_t*)malloc(sizeof(int64_t) * (size_t)(cap_rows + 1));
        m->cap_free = (size_t)cap_rows;
    }
    m->n_free = 0;
    for (int64_t s = cap_rows - 1; s >= 0; --s) m->free_slots[m->n_free++] = s;
    m->high_water = -1;
    m->staged = 0;
    return 1;
}
int orc_mgr_streaming_stage(orc_mgr* m, int64_t row_id, int64_t kb, int64_t vb, int changed,
                            int64_t* out_slot, int* restaged) {
    /* :153-192 */
    int64_t slot;
    *out_slot = -1;
    *restaged = 0;
    if (hm_find(&m->row_slot, row_id, &slot)) {
        *out_slot = slot;
        if (!changed) return 1; /* sticky hit: no copy */
        m->staged += (uint64_t)kb + (uint64_t)vb;
        *restaged = 1;
        return 1;
    }
    if (m->n_free == 0) return 0;
    slot = m->free_slots[--m->n_free];
    hm_put(&m->row_slot, row_id, slot);
    m->staged += (uint64_t)kb + (uint64_t)vb;
    if (slot > m->high_water) m->high_water = slot;
    *out_slot = slot;
    *restaged = 1;
    return 1;
}
int orc_mgr_streaming_release(orc_mgr* m, int64_t row_id) {
    /* :194-200: freed slot goes back on top of the stack */
    int64_t slot;
    if (!hm_find(&m->row_slot, row_id, &slot)) return 0;
    if (m->n_free >= m->cap_free) {
        size_t nc = m->cap_free ? m->cap_free * 2 : 16;
        int64_t* p = (int64_t*)realloc(m->free_slots, sizeof(int64_t) * nc);
        if (!p) return 0;
        m->free_slots = p; m->cap_free = nc;
    }
    m->free_slots[m->n_free++] = slot;
    hm_erase(&m->row_slot, row_id);
    return 1;
}
int orc_mgr_streaming_window(orc_mgr* m) {
    /* :202-210 */
    if (!m->initialized || m->high_water < 0) return 0;
    const uint64_t span = ((uint64_t)m->high_water + 1) * m->stride_floats * 4u;
    if (span > m->max_window) return 0;
    apply_window(m, span, 2);
    return 1;
}
void orc_mgr_streaming_end(orc_mgr* m) {
    /* :212-219 */
    orc_mgr_streaming_window(m);
    apply_window(m, 1, 0);
    ++m->reset_calls;
    hm_clear(&m->row_slot);
    m->n_free = 0;
    m->high_water = -1;
}
int64_t orc_mgr_streaming_staged_bytes(orc_mgr* m) { return (int64_t)m->staged; }
int64_t orc_mgr_last_window_bytes(orc_mgr* m) { return m->last_win_bytes; }
int orc_mgr_last_window_prop(orc_mgr* m) { return m->last_win_prop; }
int64_t orc_mgr_window_calls(orc_mgr* m) { return m->win_calls; }
int64_t orc_mgr_reset_calls(orc_mgr* m) { return m->reset_calls; }

/* ---------------------------------------------------------------- CSV read */
int orc_read_motion_csv(const char* path, int frames, int num_tiles, float* scores_out,
                        int8_t* reuse_out) {
    /* src/run_policy_experiment.cu:45-69 (scores are sscanf "%f" of the text) */
    FILE* f = fopen(path, "r");
    if (!f) return -1;
    memset(scores_out, 0, sizeof(float) * (size_t)frames * (size_t)num_tiles);
    if (reuse_out) memset(reuse_out, 0, (size_t)frames * (size_t)num_tiles);
    char line[256];
    int accepted = 0;
    if (!fgets(line, sizeof line, f)) { fclose(f); return 0; }
    while (fgets(line, sizeof line, f)) {
        int fr, tid, is_static, start, count, reuse = 0;
        float score;
        int got = sscanf(line, "%d,%d,%f,%d,%d,%d,%d", &fr, &tid, &score, &is_static, &start,
                         &count, &reuse);
        if ((got == 6 || got == 7) && fr >= 0 && fr < frames && tid >= 0 && tid < num_tiles) {
            scores_out[(size_t)fr * num_tiles + tid] = score;
            if (got == 7 && reuse_out) reuse_out[(size_t)fr * num_tiles + tid] = (int8_t)reuse;
            ++accepted;
        }
    }
    fclose(f);
    return accepted;
}

/* --------------------------------------------------------- per-frame loop */
int orc_run_trace(const orc_params* p, const float* scores_flat, int64_t* map_out,
                  int* sel_count, int64_t* sel_ids, int sel_cap, int* copy_count,
                  int64_t* copy_rows, int64_t* copy_slots, int64_t copy_cap,
                  int64_t* window_bytes, int64_t* staged_bytes, int* staged_tiles) {
    /* src/run_policy_experiment.cu:98-276 */
    if (!p || p->frames <= 0 || p->tokens <= 0 || p->hidden <= 0 || p->tile_tokens <= 0 ||
        p->elem_bytes <= 0 || (2 * p->hidden * p->elem_bytes) % 4 != 0)
        return -1;
    const int F = p->frames, T = p->tokens, tt = p->tile_tokens;
    const int64_t nt = orc_tiles_per_frame(T, tt);
    const size_t map_len = (size_t)F * (size_t)T;
    for (int f = 0; f < F; ++f) {
        sel_count[f] = 0; copy_count[f] = 0; window_bytes[f] = -1;
        staged_bytes[f] = 0; staged_tiles[f] = 0;
    }
    for (size_t i = 0; i < (size_t)F * map_len; ++i) map_out[i] = -1;
    if (p->policy == ORC_NONE) return 0; /* no map, kernel reads base K/V (:290-302) */

    const uint64_t row_kv_bytes = (uint64_t)p->hidden * (uint64_t)p->elem_bytes;
    const uint64_t tile_bytes = (uint64_t)tt * row_kv_bytes * 2u;
    const int64_t slots = (int64_t)((uint64_t)p->set_aside / tile_bytes);
    if (slots > sel_cap) return -2;
    orc_mgr* m = orc_mgr_create(p->set_aside, p->set_aside);
    if (!m) return -3;
    orc_mgr_init(m);
    orc_mgr_arena_init(m, p->set_aside, (int64_t)(2u * row_kv_bytes / 4u));
    int64_t* h_map = (int64_t*)malloc(sizeof(int64_t) * map_len);
    int64_t* ids = (int64_t*)malloc(sizeof(int64_t) * (size_t)(slots + (int64_t)F * nt + 1));
    char* selected = (char*)calloc((size_t)F * (size_t)nt + 1, 1);
    char* prev_sel = (char*)calloc((size_t)F * (size_t)nt + 1, 1);
    int64_t prev_len = 0;
    int rc = 0;
    int64_t n_copies = 0;
    for (size_t i = 0; i < map_len; ++i) h_map[i] = -1;
    if (p->streaming) orc_mgr_streaming_begin(m);

    for (int f = 0; f < F && rc == 0; ++f) {
        const int64_t base = (p->cross && p->window > 0 && f - p->window + 1 > 0)
                                 ? (int64_t)(f - p->window + 1) : 0;
        const int n_cand = p->cross ? (int)(((int64_t)f - base + 1) * nt) : (int)nt;
        const float* cand_scores = p->cross ? scores_flat + base * nt : scores_flat + (int64_t)f * nt;
        int count = 0;
        orc_select(p->policy, cand_scores, n_cand, (int)slots, (int)nt, (int)(F - base), ids, &count);
        sel_count[f] = count;
        for (int i = 0; i < count && i < sel_cap; ++i) sel_ids[(size_t)f * sel_cap + i] = ids[i];

        /* selected[] over absolute ids [0, (f+1)*nt).  Ids outside the
         * candidate range (Uniform with more slots than candidates) are not
         * staged; the reference writes them out of bounds (:170-172). */
        const int64_t sel_len = ((int64_t)f + 1) * nt;
        memset(selected, 0, (size_t)sel_len);
        for (int i = 0; i < count; ++i)
            if (ids[i] >= 0 && ids[i] < n_cand)
                selected[(p->cross ? base * nt : 0) + ids[i]] = 1;

        if (p->streaming && f > 0) { /* :173-187 */
            for (int64_t gid = 0; gid < prev_len; ++gid) {
                if (!prev_sel[gid]) continue;
                if (gid < sel_len && selected[gid]) continue;
                const int64_t src_f = p->cross ? gid / nt : f; /* intra uses the current frame */
                const int64_t tile = p->cross ? gid % nt : gid;
                const int64_t t0 = tile * tt;
                const int64_t c = (T - t0) < tt ? (T - t0) : tt;
                for (int64_t r = 0; r < c; ++r)
                    orc_mgr_streaming_release(m, src_f * T + t0 + r);
            }
        }
        orc_mgr_arena_begin(m);
        for (int64_t i = 0; i < ((int64_t)f + 1) * T; ++i) h_map[i] = -1;
        int tiles_ok = 0;
        for (int i = 0; i < count; ++i) { /* :197-232, policy order */
            if (ids[i] < 0 || ids[i] >= n_cand) continue;
            const int64_t gid = (p->cross ? base * nt : 0) + ids[i];
            const int64_t src_f = p->cross ? gid / nt : f;
            const int64_t tile = p->cross ? gid % nt : gid;
            const int64_t t0 = tile * tt;
            const int64_t c = (T - t0) < tt ? (T - t0) : tt;
            int all = 1;
            for (int64_t r = 0; r < c && all; ++r) {
                const int64_t row_id = src_f * T + t0 + r;
                int64_t slot = -1;
                int copied = 0;
                if (p->streaming) {
                    all = orc_mgr_streaming_stage(m, row_id, (int64_t)row_kv_bytes,
                                                  (int64_t)row_kv_bytes, 0, &slot, &copied);
                } else {
                    all = orc_mgr_arena_stage(m, (int64_t)row_kv_bytes, (int64_t)row_kv_bytes, &slot);
                    copied = all;
                }
                if (all) {
                    h_map[row_id] = slot;
                    if (copied) {
                        if (n_copies >= copy_cap) { rc = -4; break; }
                        copy_rows[n_copies] = row_id;
                        copy_slots[n_copies] = slot;
                        ++n_copies;
                        ++copy_count[f];
                    }
                }
            }
            if (rc) break;
            if (all) ++tiles_ok;
        }
        staged_tiles[f] = tiles_ok;
        memcpy(map_out + (size_t)f * map_len, h_map, sizeof(int64_t) * map_len);
        const int ok = p->streaming ? orc_mgr_streaming_window(m) : orc_mgr_arena_window(m);
        window_bytes[f] = ok ? orc_mgr_last_window_bytes(m) : -1;
        staged_bytes[f] = p->streaming ? orc_mgr_streaming_staged_bytes(m) : orc_mgr_arena_used(m);
        if (p->streaming) {
            memcpy(prev_sel, selected, (size_t)sel_len);
            prev_len = sel_len;
        } else {
            orc_mgr_arena_end(m);
        }
    }
    if (p->streaming) orc_mgr_streaming_end(m);
    free(h_map); free(ids); free(selected); free(prev_sel);
    orc_mgr_destroy(m);
    return rc;
}

/* ------------------------------------------------- temporal-reuse streaming */
int orc_run_reuse(const orc_params* p, const float* scores_flat, const int8_t* reuse_flat,
                  int64_t* map_out, int* copy_count, int* restage_count, int* hit_count,
                  int64_t* copy_rows, int64_t* copy_slots, int64_t copy_cap,
                  int64_t* window_bytes, int64_t* staged_bytes, int* staged_tiles) {
    /* src/run_policy_experiment.cu:156-274 (intra, streaming) with position
     * keys and changed = !reuse; src/kv_tile_manager.cu:153-200 */
    if (!p || !p->streaming || p->cross || p->frames <= 0 || p->tokens <= 0 || p->hidden <= 0 ||
        p->tile_tokens <= 0 || p->elem_bytes <= 0 || (2 * p->hidden * p->elem_bytes) % 4 != 0)
        return -1;
    const int F = p->frames, T = p->tokens, tt = p->tile_tokens;
    const int64_t nt = orc_tiles_per_frame(T, tt);
    for (int f = 0; f < F; ++f) {
        copy_count[f] = restage_count[f] = hit_count[f] = 0;
        window_bytes[f] = -1; staged_bytes[f] = 0; staged_tiles[f] = 0;
    }
    for (size_t i = 0; i < (size_t)F * (size_t)T; ++i) map_out[i] = -1;
    if (p->policy == ORC_NONE) return 0;

    const uint64_t row_kv_bytes = (uint64_t)p->hidden * (uint64_t)p->elem_bytes;
    const uint64_t tile_bytes = (uint64_t)tt * row_kv_bytes * 2u;
    const int64_t slots = (int64_t)((uint64_t)p->set_aside / tile_bytes);
    orc_mgr* m = orc_mgr_create(p->set_aside, p->set_aside);
    if (!m) return -3;
    orc_mgr_init(m);
    orc_mgr_arena_init(m, p->set_aside, (int64_t)(2u * row_kv_bytes / 4u));
    int64_t* ids = (int64_t*)malloc(sizeof(int64_t) * (size_t)(slots + nt + 1));
    char* selected = (char*)calloc((size_t)nt + 1, 1);
    char* prev_sel = (char*)calloc((size_t)nt + 1, 1);
    int rc = 0;
    int64_t n_copies = 0;
    orc_mgr_streaming_begin(m);

    for (int f = 0; f < F && rc == 0; ++f) {
        int count = 0;
        orc_select(p->policy, scores_flat + (int64_t)f * nt, (int)nt, (int)slots, (int)nt, F, ids,
                   &count);
        memset(selected, 0, (size_t)nt);
        for (int i = 0; i < count; ++i)
            if (ids[i] >= 0 && ids[i] < nt) selected[ids[i]] = 1;
        if (f > 0) {
            for (int64_t tile = 0; tile < nt; ++tile) {
                if (!prev_sel[tile] || selected[tile]) continue;
                const int64_t t0 = tile * tt;
                const int64_t c = (T - t0) < tt ? (T - t0) : tt;
                /* last row first: the LIFO free stack then hands the
                 * tile's slots back in ascending order */
                for (int64_t r = c - 1; r >= 0; --r) orc_mgr_streaming_release(m, t0 + r);
            }
        }
        int64_t* h_map = map_out + (size_t)f * (size_t)T;
        int tiles_ok = 0;
        for (int i = 0; i < count; ++i) {
            if (ids[i] < 0 || ids[i] >= nt) continue;
            const int64_t tile = ids[i];
            const int64_t t0 = tile * tt;
            const int64_t c = (T - t0) < tt ? (T - t0) : tt;
            const int changed = !(reuse_flat && reuse_flat[(size_t)f * (size_t)nt + (size_t)tile]);
            int all = 1;
            for (int64_t r = 0; r < c && all; ++r) {
                int64_t slot = -1, had = -1;
                int copied = 0;
                const int held = hm_find(&m->row_slot, t0 + r, &had);
                all = orc_mgr_streaming_stage(m, t0 + r, (int64_t)row_kv_bytes,
                                              (int64_t)row_kv_bytes, changed, &slot, &copied);
                if (!all) break;
                h_map[t0 + r] = slot;
                if (!copied) { ++hit_count[f]; continue; }
                if (held) ++restage_count[f];
                if (n_copies >= copy_cap) { rc = -4; break; }
                copy_rows[n_copies] = (int64_t)f * T + t0 + r;
                copy_slots[n_copies] = slot;
                ++n_copies;
                ++copy_count[f];
            }
            if (rc) break;
            if (all) ++tiles_ok;
        }
        staged_tiles[f] = tiles_ok;
        window_bytes[f] = orc_mgr_streaming_window(m) ? orc_mgr_last_window_bytes(m) : -1;
        staged_bytes[f] = orc_mgr_streaming_staged_bytes(m);
        memcpy(prev_sel, selected, (size_t)nt);
    }
    orc_mgr_streaming_end(m);
    free(ids); free(selected); free(prev_sel);
    orc_mgr_destroy(m);
    return rc;
}
