// Session implementation (see session.h).
#include "session.h"

#include <algorithm>
#include <cstdio>
#include <cstring>

#include "kvp_common.h"
#include "qkv_sm100.h"

namespace kvp {

Session::Session(const SessionConfig& c)
    : c_(c), layout_(c.tokens > 0 ? c.tokens : 1, c.tile_tokens > 0 ? c.tile_tokens : 1) {
    if (c.frames <= 0 || c.tokens <= 0 || c.hidden <= 0 || c.tile_tokens <= 0 ||
        (c.elem_bytes != 2 && c.elem_bytes != 4) || c.set_aside < 0 || c.layers < 0 ||
        c.layers > kMaxLayers || c.mode < MODE_INTRA || c.mode > MODE_REUSE || c.window < 0 ||
        (c.mode == MODE_REUSE && !c.streaming) ||
        (2 * (int64_t)c.hidden * c.elem_bytes) % 16 != 0) {
        set_error("session: invalid configuration");
        status_ = KVP_ERR_ARG;
        return;
    }
    nt_ = layout_.tiles_per_frame;
    row_kv_bytes_ = (int64_t)c.hidden * c.elem_bytes;
    // src/run_policy_experiment.cu:143-144, with the element size as a
    // parameter (4 reproduces the reference's fp32 formula).
    const int64_t tile_bytes = (int64_t)c.tile_tokens * row_kv_bytes_ * 2;
    slots_ = c.set_aside / tile_bytes;
    cap_rows_ = c.set_aside / (2 * row_kv_bytes_);
    policy_.reset(make_policy(c.policy, (int)nt_, c.frames));
    if (!policy_) {
        set_error("session: unknown policy %d", c.policy);
        status_ = KVP_ERR_ARG;
        return;
    }
    mgr_.reset(new KVTileManager((size_t)c.set_aside, (size_t)c.set_aside, KVTM_FLAG_DRY_RUN));
    mgr_->init();
    mgr_->arena_init((size_t)c.set_aside, (size_t)(2 * row_kv_bytes_ / 4));
    if (c.streaming) mgr_->streaming_begin();
    map_.assign((size_t)c.frames * c.tokens, -1);
    ids_.resize((size_t)(slots_ + (int64_t)c.frames * nt_ + 1));
    selected_.assign((size_t)(c.frames * nt_ + 1), 0);
    prev_selected_.assign((size_t)(c.frames * nt_ + 1), 0);

    if (c.layers > 0) {
        arena_layer_bytes_ = ((int64_t)cap_rows_ * 2 * row_kv_bytes_ + 255) / 256 * 256;
        const size_t map_bytes = map_.size() * sizeof(int64_t);
        const size_t pair_bytes = (size_t)std::max<int64_t>(cap_rows_, 1) * 2 * sizeof(int32_t);
        cudaError_t e = cudaMalloc(&d_map_, map_bytes);
        if (e == cudaSuccess) e = cudaMalloc(&d_pairs_, pair_bytes);
        if (e == cudaSuccess && arena_layer_bytes_ > 0)
            e = cudaMalloc(&d_arena_, (size_t)arena_layer_bytes_ * c.layers);
        for (int i = 0; i < kUploadSlots && e == cudaSuccess; ++i) {
            e = cudaMallocHost(&h_map_pinned_[i], map_bytes);
            if (e == cudaSuccess) e = cudaMallocHost(&h_pairs_pinned_[i], pair_bytes);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&upload_done_[i], cudaEventDisableTiming);
        }
        if (e == cudaSuccess) e = cudaMemset(d_map_, 0xff, map_bytes);  // all -1
        if (e == cudaSuccess && d_arena_)
            e = cudaMemset(d_arena_, 0, (size_t)arena_layer_bytes_ * c.layers);
        if (e != cudaSuccess) status_ = cuda_status(e, "session device buffers");
    }
}

Session::~Session() {
    for (int i = 0; i < kUploadSlots; ++i)
        if (upload_done_[i]) { cudaEventSynchronize(upload_done_[i]); cudaEventDestroy(upload_done_[i]); }
    if (d_map_) cudaFree(d_map_);
    if (d_pairs_) cudaFree(d_pairs_);
    if (d_arena_) cudaFree(d_arena_);
    for (int i = 0; i < kUploadSlots; ++i) {
        if (h_map_pinned_[i]) cudaFreeHost(h_map_pinned_[i]);
        if (h_pairs_pinned_[i]) cudaFreeHost(h_pairs_pinned_[i]);
    }
}

void* Session::arena(int layer) const {
    if (!d_arena_ || layer < 0 || layer >= c_.layers) return nullptr;
    return static_cast<char*>(d_arena_) + (size_t)arena_layer_bytes_ * layer;
}

int Session::stage_rows_of(int64_t gid, int64_t src_f, int64_t tile) {
    // One tile's rows in order; a refused row stops the tile and the rows
    // already staged stay mapped (src/run_policy_experiment.cu:197-232).
    (void)gid;
    const int64_t t0 = layout_.tile_start(tile);
    const int64_t cnt = layout_.tile_count(tile);
    if (!c_.streaming) {
        // dense arena: consecutive slots, every row a copy
        long first = -1;
        const int64_t k = (int64_t)mgr_->arena_reserve_rows((size_t)(2 * row_kv_bytes_), (size_t)cnt, &first);
        const int64_t row0 = src_f * c_.tokens + t0;
        const size_t p0 = pairs_.size();
        pairs_.resize(p0 + 2 * (size_t)k);
        for (int64_t r = 0; r < k; ++r) {
            map_[(size_t)(row0 + r)] = first + r;
            pairs_[p0 + 2 * (size_t)r] = (int32_t)(row0 + r);
            pairs_[p0 + 2 * (size_t)r + 1] = (int32_t)(first + r);
        }
        return k == cnt ? 1 : 0;
    }
    // streaming: a held row is a sticky hit, mapped without a copy
    bool all = true;
    for (int64_t r = 0; r < cnt && all; ++r) {
        const int64_t row_id = src_f * c_.tokens + t0 + r;
        long slot = -1;
        bool copy = false;
        all = mgr_->streaming_reserve((long)row_id, (size_t)(2 * row_kv_bytes_), false, &slot, &copy);
        if (all) {
            map_[(size_t)row_id] = slot;
            if (copy) {
                pairs_.push_back((int32_t)row_id);
                pairs_.push_back((int32_t)slot);
            } else {
                ++info_.hits;
            }
        }
    }
    return all ? 1 : 0;
}

int Session::plan_frame(int f, const float* scores_flat, const int8_t* reuse_flat) {
    if (status_ != KVP_OK) return status_;
    if (c_.mode == MODE_REUSE && f >= 0 && f < c_.frames && scores_flat && f == last_frame_ + 1 &&
        !finished_)
        return plan_reuse(f, scores_flat, reuse_flat);
    if (c_.mode == MODE_STACK || c_.mode == MODE_REUSE || f < 0 || f >= c_.frames || !scores_flat || f != last_frame_ + 1 ||
        finished_) {
        set_error("plan_frame: frame %d out of order (expected %d) or wrong mode", f, last_frame_ + 1);
        return KVP_ERR_ARG;
    }
    const bool cross = c_.mode == MODE_CROSS;
    const int64_t base = (cross && c_.window > 0) ? std::max<int64_t>(0, f - c_.window + 1) : 0;
    const int n_cand = cross ? (int)((f - base + 1) * nt_) : (int)nt_;
    const float* cand = cross ? scores_flat + base * nt_ : scores_flat + (int64_t)f * nt_;
    if (c_.policy == POLICY_REUSE_WEIGHTED)
        static_cast<ReuseWeightedPolicy*>(policy_.get())->set_total_frames((int)(c_.frames - base));
    int count = 0;
    info_ = SessionStepInfo{};
    info_.frame = f;
    pairs_.clear();
    sel_ids_.clear();
    const bool persist = c_.policy != POLICY_NONE;
    if (persist) {
        policy_->select(cand, n_cand, (int)slots_, ids_.data(), &count);
        sel_ids_.assign(ids_.begin(), ids_.begin() + std::max(0, count));
    }
    info_.sel_count = count;
    const int64_t gid0 = cross ? base * nt_ : 0;
    const int64_t sel_len = ((int64_t)f + 1) * nt_;
    std::fill(selected_.begin(), selected_.begin() + sel_len, 0);
    // Ids beyond the candidates (Uniform with more slots than tiles) stage
    // nothing; the reference writes them past the end of its selection
    // vector (src/run_policy_experiment.cu:170-172).
    for (int i = 0; i < count; ++i)
        if (ids_[i] >= 0 && ids_[i] < n_cand) selected_[(size_t)(gid0 + ids_[i])] = 1;

    if (persist && c_.streaming && f > 0) {
        // :173-187 -- intra mode releases with the current frame index (the
        // reference's rows of the previous frame stay held), kept as is.
        for (int64_t gid = 0; gid < prev_len_; ++gid) {
            if (!prev_selected_[(size_t)gid]) continue;
            if (gid < sel_len && selected_[(size_t)gid]) continue;
            const int64_t src_f = cross ? gid / nt_ : f;
            const int64_t tile = cross ? gid % nt_ : gid;
            const int64_t t0 = layout_.tile_start(tile);
            const int64_t cnt = layout_.tile_count(tile);
            for (int64_t r = 0; r < cnt; ++r) mgr_->streaming_release((long)(src_f * c_.tokens + t0 + r));
        }
    }
    mgr_->arena_begin_step();
    std::fill(map_.begin(), map_.begin() + ((int64_t)f + 1) * c_.tokens, -1);
    int tiles_ok = 0;
    if (persist) {
        for (int i = 0; i < count; ++i) {
            if (ids_[i] < 0 || ids_[i] >= n_cand) continue;
            const int64_t gid = gid0 + ids_[i];
            const int64_t src_f = cross ? gid / nt_ : f;
            const int64_t tile = cross ? gid % nt_ : gid;
            tiles_ok += stage_rows_of(gid, src_f, tile);
        }
    }
    info_.staged_tiles = tiles_ok;
    info_.copies = (int)(pairs_.size() / 2);
    info_.map_row0 = cross ? base * c_.tokens : (int64_t)f * c_.tokens;
    info_.map_rows = cross ? ((int64_t)f + 1 - base) * c_.tokens : c_.tokens;
    if (persist) {
        info_.window_bytes = (int64_t)(c_.streaming ? mgr_->streaming_window_span()
                                                    : mgr_->arena_window_span());
        info_.staged_bytes = (int64_t)(c_.streaming ? mgr_->streaming_staged_bytes()
                                                    : mgr_->arena_used_bytes());
        if (c_.streaming) {
            std::copy(selected_.begin(), selected_.begin() + sel_len, prev_selected_.begin());
            prev_len_ = sel_len;
        } else {
            mgr_->arena_end_step();
        }
    }
    last_frame_ = f;
    return KVP_OK;
}

int Session::plan_reuse(int f, const float* scores_flat, const int8_t* reuse_flat) {
    // The intra streaming loop of src/run_policy_experiment.cu:156-274 with
    // position keys and changed = !reuse[f][tile] in streaming_stage
    // (src/kv_tile_manager.cu:153-175).
    int count = 0;
    info_ = SessionStepInfo{};
    info_.frame = f;
    pairs_.clear();
    sel_ids_.clear();
    const bool persist = c_.policy != POLICY_NONE;
    if (persist) {
        policy_->select(scores_flat + (int64_t)f * nt_, (int)nt_, (int)slots_, ids_.data(), &count);
        sel_ids_.assign(ids_.begin(), ids_.begin() + std::max(0, count));
    }
    info_.sel_count = count;
    std::fill(selected_.begin(), selected_.begin() + nt_, 0);
    for (int i = 0; i < count; ++i)
        if (ids_[i] >= 0 && ids_[i] < nt_) selected_[(size_t)ids_[i]] = 1;
    if (tile_full_.size() != (size_t)nt_) {
        tile_full_.assign((size_t)nt_, 0);
        tile_slots_.assign((size_t)(nt_ * c_.tile_tokens), -1);
    }
    if (persist && f > 0) {
        for (int64_t tile = 0; tile < nt_; ++tile) {
            if (!prev_selected_[(size_t)tile] || selected_[(size_t)tile]) continue;
            const int64_t t0 = layout_.tile_start(tile);
            const int64_t cnt = layout_.tile_count(tile);
            // Last row first: the LIFO free stack then hands these slots to
            // the next admitted tile in ascending order, so its 8-row groups
            // stay single ascending runs the kernel stages with TMA boxes.
            for (int64_t r = cnt - 1; r >= 0; --r) mgr_->streaming_release((long)(t0 + r));
            tile_full_[(size_t)tile] = 0;
        }
    }
    int64_t* map = map_.data() + (int64_t)f * c_.tokens;
    std::fill(map, map + c_.tokens, -1);
    int tiles_ok = 0;
    for (int i = 0; persist && i < count; ++i) {
        if (ids_[i] < 0 || ids_[i] >= nt_) continue;
        const int64_t tile = ids_[i];
        const int64_t t0 = layout_.tile_start(tile);
        const int64_t cnt = layout_.tile_count(tile);
        const bool changed = !(reuse_flat && reuse_flat[(int64_t)f * nt_ + tile]);
        int64_t* cached = tile_slots_.data() + tile * c_.tile_tokens;
        if (tile_full_[(size_t)tile]) {
            // Every row holds its slot: a sticky hit changes no manager
            // state, a re-copy only counts its bytes (streaming_reserve with
            // a held row), so neither needs the per-row lookup.
            for (int64_t r = 0; r < cnt; ++r) map[t0 + r] = cached[r];
            if (!changed) {
                info_.hits += (int)cnt;
            } else {
                mgr_->streaming_count_restage((size_t)(cnt * 2 * row_kv_bytes_));
                info_.restaged += (int)cnt;
                for (int64_t r = 0; r < cnt; ++r) {
                    pairs_.push_back((int32_t)((int64_t)f * c_.tokens + t0 + r));
                    pairs_.push_back((int32_t)cached[r]);
                }
            }
            ++tiles_ok;
            continue;
        }
        bool all = true;
        for (int64_t r = 0; r < cnt && all; ++r) {
            long slot = -1;
            bool copy = false, held = false;
            all = mgr_->streaming_reserve((long)(t0 + r), (size_t)(2 * row_kv_bytes_), changed, &slot,
                                          &copy, &held);
            if (!all) break;
            map[t0 + r] = slot;
            cached[r] = slot;
            if (!copy) { ++info_.hits; continue; }
            if (held) ++info_.restaged;
            pairs_.push_back((int32_t)((int64_t)f * c_.tokens + t0 + r));
            pairs_.push_back((int32_t)slot);
        }
        if (all) {
            ++tiles_ok;
            tile_full_[(size_t)tile] = 1;
        }
    }
    info_.staged_tiles = tiles_ok;
    info_.copies = (int)(pairs_.size() / 2);
    info_.map_row0 = (int64_t)f * c_.tokens;
    info_.map_rows = c_.tokens;
    if (persist) {
        info_.window_bytes = (int64_t)mgr_->streaming_window_span();
        info_.staged_bytes = (int64_t)mgr_->streaming_staged_bytes();
        std::copy(selected_.begin(), selected_.begin() + nt_, prev_selected_.begin());
    }
    last_frame_ = f;
    return KVP_OK;
}

int Session::plan_stack(const float* scores_flat) {
    if (status_ != KVP_OK) return status_;
    if (c_.mode != MODE_STACK || !scores_flat || finished_) {
        set_error("plan_stack: session is not in stack mode");
        return KVP_ERR_ARG;
    }
    // Candidates are every frame's tiles, whatever the attention window.
    const int64_t F = c_.frames;
    const int64_t base = 0;
    const int n_cand = (int)(F * nt_);
    if (c_.policy == POLICY_REUSE_WEIGHTED)
        static_cast<ReuseWeightedPolicy*>(policy_.get())->set_total_frames((int)(F - base));
    int count = 0;
    info_ = SessionStepInfo{};
    info_.frame = -1;
    pairs_.clear();
    sel_ids_.clear();
    const bool persist = c_.policy != POLICY_NONE;
    if (persist) {
        policy_->select(scores_flat + base * nt_, n_cand, (int)slots_, ids_.data(), &count);
        sel_ids_.assign(ids_.begin(), ids_.begin() + std::max(0, count));
    }
    info_.sel_count = count;
    const int64_t sel_len = F * nt_;
    std::fill(selected_.begin(), selected_.begin() + sel_len, 0);
    for (int i = 0; i < count; ++i)
        if (ids_[i] >= 0 && ids_[i] < n_cand) selected_[(size_t)(base * nt_ + ids_[i])] = 1;
    if (persist && c_.streaming && prev_len_ > 0) {
        for (int64_t gid = 0; gid < prev_len_; ++gid) {
            if (!prev_selected_[(size_t)gid] || selected_[(size_t)gid]) continue;
            const int64_t t0 = layout_.tile_start(gid % nt_);
            const int64_t cnt = layout_.tile_count(gid % nt_);
            for (int64_t r = 0; r < cnt; ++r)
                mgr_->streaming_release((long)((gid / nt_) * c_.tokens + t0 + r));
        }
    }
    mgr_->arena_begin_step();
    std::fill(map_.begin(), map_.end(), -1);
    int tiles_ok = 0;
    if (persist) {
        for (int i = 0; i < count; ++i) {
            if (ids_[i] < 0 || ids_[i] >= n_cand) continue;
            const int64_t gid = base * nt_ + ids_[i];
            tiles_ok += stage_rows_of(gid, gid / nt_, gid % nt_);
        }
    }
    info_.staged_tiles = tiles_ok;
    info_.copies = (int)(pairs_.size() / 2);
    info_.map_row0 = 0;
    info_.map_rows = F * c_.tokens;
    if (persist) {
        info_.window_bytes = (int64_t)(c_.streaming ? mgr_->streaming_window_span()
                                                    : mgr_->arena_window_span());
        info_.staged_bytes = (int64_t)(c_.streaming ? mgr_->streaming_staged_bytes()
                                                    : mgr_->arena_used_bytes());
        if (c_.streaming) {
            std::copy(selected_.begin(), selected_.begin() + sel_len, prev_selected_.begin());
            prev_len_ = sel_len;
        } else {
            mgr_->arena_end_step();
        }
    }
    return KVP_OK;
}

int Session::finish() {
    if (status_ != KVP_OK) return status_;
    if (!finished_ && c_.streaming && c_.policy != POLICY_NONE) mgr_->streaming_end();
    finished_ = true;
    return KVP_OK;
}

int Session::upload(cudaStream_t s) { return upload_to(d_map_, s); }

int Session::upload_to(int64_t* dmap, cudaStream_t s, int64_t slot_offset) {
    if (!d_map_ || !dmap) return KVP_ERR_ARG;
    const int64_t r0 = info_.map_row0, n = info_.map_rows;
    if (r0 < 0 || n < 0 || r0 + n > (int64_t)map_.size()) return KVP_ERR_ARG;
    // This slot's pinned buffers may still feed the upload made
    // kUploadSlots uploads ago.
    const int k = upload_slot_;
    upload_slot_ = (upload_slot_ + 1) % kUploadSlots;
    KVP_CUDA(cudaEventSynchronize(upload_done_[k]));
    if (slot_offset == 0) {
        std::memcpy(h_map_pinned_[k] + r0, map_.data() + r0, (size_t)n * sizeof(int64_t));
    } else {
        for (int64_t r = r0; r < r0 + n; ++r)
            h_map_pinned_[k][r] = map_[(size_t)r] >= 0 ? map_[(size_t)r] + slot_offset : map_[(size_t)r];
    }
    KVP_CUDA(cudaMemcpyAsync(dmap + r0, h_map_pinned_[k] + r0, (size_t)n * sizeof(int64_t),
                             cudaMemcpyHostToDevice, s));
    if (!pairs_.empty()) {
        if (slot_offset == 0) {
            std::memcpy(h_pairs_pinned_[k], pairs_.data(), pairs_.size() * sizeof(int32_t));
        } else {
            for (size_t p = 0; p < pairs_.size(); p += 2) {
                h_pairs_pinned_[k][p] = pairs_[p];
                h_pairs_pinned_[k][p + 1] = pairs_[p + 1] + (int32_t)slot_offset;
            }
        }
        KVP_CUDA(cudaMemcpyAsync(d_pairs_, h_pairs_pinned_[k], pairs_.size() * sizeof(int32_t),
                                 cudaMemcpyHostToDevice, s));
    }
    KVP_CUDA(cudaEventRecord(upload_done_[k], s));
    return KVP_OK;
}

int Session::stage(const void* const* k_layers, const void* const* v_layers, cudaStream_t s,
                   int64_t skip_row0, int64_t skip_rows) {
    const int64_t lo = skip_row0, hi = skip_row0 + (skip_rows > 0 ? skip_rows : 0);
    bool any = false;
    for (size_t i = 0; i < pairs_.size() && !any; i += 2) any = pairs_[i] < lo || pairs_[i] >= hi;
    if (!any) return KVP_OK;   // nothing to copy (or every row was produced in place)
    if (!d_arena_ || !k_layers || !v_layers) return KVP_ERR_ARG;
    GatherLayers L{};
    for (int l = 0; l < c_.layers; ++l) {
        L.k[l] = k_layers[l];
        L.v[l] = v_layers[l];
        L.arena[l] = arena(l);
    }
    return launch_gather_rows(L, c_.layers, d_pairs_, (int)(pairs_.size() / 2), row_kv_bytes_, s,
                              lo, hi);
}

int Session::produce(int layer, const void* x, const void* w, const float* bias, void* q, void* k,
                     void* v, int64_t row0, int64_t rows, cudaStream_t s) {
    void* a = arena(layer);
    if (c_.mode == MODE_REUSE || c_.elem_bytes != 2 || !d_map_ || rows <= 0 ||
        row0 < info_.map_row0 || row0 + rows > info_.map_row0 + info_.map_rows) {
        set_error("session produce: needs a bf16 session with device buffers, a mode other than "
                  "reuse, and rows inside this step's map slice [%lld, %lld)",
                  (long long)info_.map_row0, (long long)(info_.map_row0 + info_.map_rows));
        return KVP_ERR_ARG;
    }
    int* st = status_word();
    if (!st) return KVP_ERR_CUDA;
    QkvIO io{};
    io.x = x;
    io.w = w;
    io.bias = bias;
    io.q = q;
    io.k = k;
    io.v = v;
    const bool persist = c_.policy != POLICY_NONE && a;
    io.arena = persist ? a : nullptr;
    io.kvmap = persist ? reinterpret_cast<const long long*>(d_map_) : nullptr;
    io.rows = rows;
    io.map_row0 = row0;
    io.arena_rows = cap_rows_;
    io.D = c_.hidden;
    return launch_qkv_project_bf16(io, st, s);
}

int64_t Session::arena_stride_rows() const {
    const int64_t row = 2 * row_kv_bytes_;
    return (row > 0 && arena_layer_bytes_ > 0 && arena_layer_bytes_ % row == 0) ? arena_layer_bytes_ / row
                                                                               : 0;
}

int Session::stage_batched(int f0, int n, int arena0, const float* scores_flat, const void* k,
                           const void* v, int64_t* maps, cudaStream_t s) {
    const int64_t stride = arena_stride_rows();
    if (status_ != KVP_OK) return status_;
    if (c_.streaming || (c_.mode != MODE_INTRA && c_.mode != MODE_CROSS) || c_.policy == POLICY_NONE ||
        n <= 0 || arena0 < 0 || arena0 + n > c_.layers || stride <= 0 || !maps || !k || !v || !d_arena_) {
        set_error("session stage_batched: needs a dense intra/cross session with a policy, one "
                  "back-to-back arena per frame (%d frames, %d layers) and device buffers", n, c_.layers);
        return KVP_ERR_ARG;
    }
    // Per frame: plan, upload its map slice and copy list with the slots
    // moved to its arena (through the pinned ring), gather its rows.
    const int64_t map_len = (int64_t)map_.size();
    for (int i = 0; i < n; ++i) {
        int rc = plan_frame(f0 + i, scores_flat);
        if (rc != KVP_OK) return rc;
        const int64_t off = (int64_t)(arena0 + i) * stride;
        if (off + stride > INT32_MAX) return KVP_ERR_ARG;
        if ((rc = upload_to(maps + (size_t)(arena0 + i) * (size_t)map_len, s, off)) != KVP_OK) return rc;
        if ((rc = stage_layer(0, k, v, s)) != KVP_OK) return rc;
    }
    return KVP_OK;
}

int Session::stage_layer(int layer, const void* k, const void* v, cudaStream_t s) {
    if (!d_arena_ || layer < 0 || layer >= c_.layers || !k || !v) return KVP_ERR_ARG;
    if (pairs_.empty()) return KVP_OK;
    GatherLayers L{};
    L.k[0] = k;
    L.v[0] = v;
    L.arena[0] = arena(layer);
    return launch_gather_rows(L, 1, d_pairs_, (int)(pairs_.size() / 2), row_kv_bytes_, s);
}

int Session::apply_window(int layer, cudaStream_t s) {
    void* a = arena(layer);
    if (!a) return KVP_ERR_ARG;
    cudaStreamAttrValue attr{};
    attr.accessPolicyWindow.base_ptr = a;
    attr.accessPolicyWindow.num_bytes = (size_t)info_.window_bytes;
    attr.accessPolicyWindow.hitRatio = info_.window_bytes > 0 ? 1.0f : 0.0f;
    attr.accessPolicyWindow.hitProp =
        info_.window_bytes > 0 ? cudaAccessPropertyPersisting : cudaAccessPropertyNormal;
    attr.accessPolicyWindow.missProp = cudaAccessPropertyStreaming;
    if (info_.window_bytes <= 0) attr.accessPolicyWindow.missProp = cudaAccessPropertyNormal;
    KVP_CUDA(cudaStreamSetAttribute(s, cudaStreamAttributeAccessPolicyWindow, &attr));
    return KVP_OK;
}

int Session::clear_window(cudaStream_t s) {
    cudaStreamAttrValue attr{};
    attr.accessPolicyWindow.base_ptr = nullptr;
    attr.accessPolicyWindow.num_bytes = 0;
    attr.accessPolicyWindow.hitRatio = 0.f;
    attr.accessPolicyWindow.hitProp = cudaAccessPropertyNormal;
    attr.accessPolicyWindow.missProp = cudaAccessPropertyNormal;
    KVP_CUDA(cudaStreamSetAttribute(s, cudaStreamAttributeAccessPolicyWindow, &attr));
    return KVP_OK;
}

int Session::step(int f, const float* scores_flat, const int8_t* reuse_flat,
                  const void* const* k_layers, const void* const* v_layers, int window_layer,
                  cudaStream_t s) {
    int rc = plan_frame(f, scores_flat, reuse_flat);
    if (rc != KVP_OK || c_.policy == POLICY_NONE) return rc;
    if ((rc = upload(s)) != KVP_OK) return rc;
    if ((rc = stage(k_layers, v_layers, s)) != KVP_OK) return rc;
    return window_layer >= 0 ? apply_window(window_layer, s) : KVP_OK;
}

int read_motion_csv(const char* path, int frames, int num_tiles, float* scores, int8_t* reuse) {
    FILE* f = std::fopen(path, "r");
    if (!f) return -1;
    std::memset(scores, 0, sizeof(float) * (size_t)frames * (size_t)num_tiles);
    if (reuse) std::memset(reuse, 0, (size_t)frames * (size_t)num_tiles);
    char line[256];
    int accepted = 0;
    if (std::fgets(line, sizeof line, f)) {  // header
        while (std::fgets(line, sizeof line, f)) {
            int fr = 0, tid = 0, is_static = 0, start = 0, count = 0, rz = 0;
            float score = 0.f;
            const int got = std::sscanf(line, "%d,%d,%f,%d,%d,%d,%d", &fr, &tid, &score, &is_static,
                                        &start, &count, &rz);
            if ((got == 6 || got == 7) && fr >= 0 && fr < frames && tid >= 0 && tid < num_tiles) {
                scores[(size_t)fr * num_tiles + tid] = score;
                if (got == 7 && reuse) reuse[(size_t)fr * num_tiles + tid] = (int8_t)rz;
                ++accepted;
            }
        }
    }
    std::fclose(f);
    return accepted;
}

}  // namespace kvp
