// Open-addressing map from a row id to its streaming slot (linear probing,
// backward-shift deletion, no tombstones).  The streaming manager looks up
// every admitted row every step; a flat table keeps those lookups to one or
// two cache lines instead of a node walk.
#pragma once

#include <climits>
#include <cstddef>
#include <cstdint>
#include <algorithm>
#include <vector>

namespace kvp {

class SlotMap {
public:
    SlotMap() { rehash(64); }

    // Pointer to key's value, or nullptr.
    long* find(long key) {
        if (key == kEmpty) return has_min_ ? &min_val_ : nullptr;
        for (size_t i = home(key);; i = (i + 1) & mask_) {
            if (keys_[i] == key) return &vals_[i];
            if (keys_[i] == kEmpty) return nullptr;
        }
    }
    // Inserts or overwrites.
    void put(long key, long val) {
        if (key == kEmpty) { n_ += has_min_ ? 0 : 1; has_min_ = true; min_val_ = val; return; }
        if ((n_ + 1) * 4 > (mask_ + 1) * 3) rehash((mask_ + 1) * 2);
        for (size_t i = home(key);; i = (i + 1) & mask_) {
            if (keys_[i] == key) { vals_[i] = val; return; }
            if (keys_[i] == kEmpty) { keys_[i] = key; vals_[i] = val; ++n_; return; }
        }
    }
    // Removes key; false if absent.
    bool erase(long key) {
        if (key == kEmpty) {
            if (!has_min_) return false;
            has_min_ = false;
            --n_;
            return true;
        }
        size_t i = home(key);
        for (;; i = (i + 1) & mask_) {
            if (keys_[i] == key) break;
            if (keys_[i] == kEmpty) return false;
        }
        // Backward shift: move later members of the probe run into the hole
        // when their home position does not lie in (hole, their slot].
        size_t j = i;
        for (;;) {
            j = (j + 1) & mask_;
            if (keys_[j] == kEmpty) break;
            const size_t h = home(keys_[j]);
            const bool stays = i <= j ? (i < h && h <= j) : (i < h || h <= j);
            if (stays) continue;
            keys_[i] = keys_[j];
            vals_[i] = vals_[j];
            i = j;
        }
        keys_[i] = kEmpty;
        --n_;
        return true;
    }
    void clear() {
        std::fill(keys_.begin(), keys_.end(), kEmpty);
        n_ = 0;
        has_min_ = false;
    }
    size_t size() const { return n_; }

private:
    static constexpr long kEmpty = LONG_MIN;   // empty-cell marker; that key itself lives in min_val_
    size_t home(long key) const {
        return (size_t)(((uint64_t)key * 0x9E3779B97F4A7C15ull) >> shift_) & mask_;
    }
    void rehash(size_t cap) {
        std::vector<long> ok, ov;
        ok.swap(keys_);
        ov.swap(vals_);
        keys_.assign(cap, kEmpty);
        vals_.assign(cap, 0);
        mask_ = cap - 1;
        shift_ = 64;
        for (size_t c = cap; c > 1; c >>= 1) --shift_;
        n_ = has_min_ ? 1 : 0;
        for (size_t i = 0; i < ok.size(); ++i)
            if (ok[i] != kEmpty) put(ok[i], ov[i]);
    }

    std::vector<long> keys_, vals_;
    size_t mask_ = 0, n_ = 0;
    int shift_ = 64;
    bool has_min_ = false;
    long min_val_ = 0;
};

}  // namespace kvp
