// Host side of the expert cache: which (layer, expert) pairs hold a slot of the HBM pool.
//
// Experts live in pinned host memory; a step copies the experts a layer selected into slots of
// a device pool before the expert kernels run. The unit is one expert of one layer (its gate,
// up and down matrices together: the three are always selected together, so per-slice and
// per-expert hit rates are the same). Two policies:
//   LRU  -- a miss takes a free slot, else evicts the least recently used entry;
//   FREQ -- the reference's frequency-gated admission (core/arch/src/stream.rs:1314-1379,
//           1400-1475; core/arch/src/expert_cache.rs): every selection counts one use of the
//           expert, hit or miss; a miss with the cache full samples 8 resident entries
//           (xorshift64 over the list of admitted keys, stale keys dropped as they are met),
//           takes the one with the fewest uses (the first met on ties) and replaces it only if
//           the newcomer has strictly more uses; otherwise the expert is served from a
//           transient bounce slot and not cached.
// Entries the current layer uses are never evicted while it runs (their slots are being read).
// The list of admitted keys holds at most 4 * n_layer * n_expert entries: a push onto a full
// list first drops its stale keys, keeping the order. xcache.cu makes the same decisions on the
// device.
#pragma once

#include <stdint.h>

#include <vector>

namespace bt {

struct XCacheStats {
    uint64_t hits = 0, misses = 0, evictions = 0, admissions = 0, bypasses = 0, bytes_copied = 0;
};

class ExpertCachePolicy {
   public:
    enum { LRU = 0, FREQ = 1 };
    ExpertCachePolicy() = default;
    ExpertCachePolicy(int policy, int capacity, int n_layer, int n_expert)
        : policy_(policy), cap_(capacity), NE_(n_expert), slot_of_((size_t)n_layer * n_expert, -1),
          freq_((size_t)n_layer * n_expert, 0), key_of_(capacity, -1), last_(capacity, 0), inuse_(capacity, 0),
          keycap_((size_t)4 * n_layer * n_expert) {
        for (int s = capacity - 1; s >= 0; s--) free_.push_back(s);
    }

    // One layer's distinct selected experts (any order). For each: its cache slot in out_slot
    // (copy_needed set when the slot must be filled first), or -1 when the expert is served
    // from a bounce slot (always copied). Updates the statistics.
    void lookup(int layer, const int *experts, int n, int *out_slot, bool *copy_needed, XCacheStats &st) {
        tick_++;
        for (int i = 0; i < n; i++) {  // this layer's resident entries are pinned for the step
            const int s = slot_of_[(size_t)layer * NE_ + experts[i]];
            if (s >= 0) inuse_[s] = tick_;
        }
        for (int i = 0; i < n; i++) {
            const int key = layer * NE_ + experts[i];
            freq_[key]++;
            int s = slot_of_[key];
            copy_needed[i] = false;
            if (s >= 0) {
                st.hits++;
                last_[s] = tick_;
                out_slot[i] = s;
                continue;
            }
            st.misses++;
            s = take_slot(key, st);
            if (s < 0) {
                st.bypasses++;
                out_slot[i] = -1;
                continue;
            }
            slot_of_[key] = s;
            key_of_[s] = key;
            last_[s] = tick_;
            inuse_[s] = tick_;
            if (policy_ == FREQ) {  // (only the admission sample reads the list)
                if (keys_.size() == keycap_) {  // full: drop the stale keys, in order
                    size_t m = 0;
                    for (size_t q = 0; q < keys_.size(); q++)
                        if (slot_of_[keys_[q]] >= 0) keys_[m++] = keys_[q];
                    keys_.resize(m);
                }
                keys_.push_back(key);
            }
            st.admissions++;
            out_slot[i] = s;
            copy_needed[i] = true;
        }
    }
    int slot(int layer, int expert) const { return slot_of_[(size_t)layer * NE_ + expert]; }
    int capacity() const { return cap_; }

   private:
    int take_slot(int key, XCacheStats &st) {
        if (!free_.empty()) {
            const int s = free_.back();
            free_.pop_back();
            return s;
        }
        int victim = -1;
        if (policy_ == LRU) {
            uint64_t best = UINT64_MAX;
            for (int s = 0; s < cap_; s++)
                if (inuse_[s] != tick_ && last_[s] < best) {
                    best = last_[s];
                    victim = s;
                }
        } else {
            victim = weakest(8);
            if (victim >= 0 && freq_[key] <= freq_[key_of_[victim]]) victim = -1;  // the incumbent stays
        }
        if (victim < 0) return -1;
        slot_of_[key_of_[victim]] = -1;
        key_of_[victim] = -1;
        st.evictions++;
        return victim;
    }
    // the least-used of a sample of admitted entries (fewest uses, the first met on ties);
    // entries the current layer uses are skipped
    int weakest(int sample) {
        int best = -1;
        uint32_t best_uses = 0;
        int tries = 0;
        while (tries < sample * 2 && !keys_.empty()) {
            tries++;
            const size_t i = (size_t)(next_rand() % keys_.size());
            const int key = keys_[i];
            const int s = slot_of_[key];
            if (s < 0) {  // stale: evicted earlier
                keys_[i] = keys_.back();
                keys_.pop_back();
                continue;
            }
            if (inuse_[s] == tick_) continue;
            const uint32_t uses = freq_[key];
            if (best < 0 || uses < best_uses) {
                best = s;
                best_uses = uses;
            }
        }
        return best;
    }
    uint64_t next_rand() {  // xorshift64
        uint64_t x = rng_;
        x ^= x << 13;
        x ^= x >> 7;
        x ^= x << 17;
        rng_ = x;
        return x;
    }

    int policy_ = LRU, cap_ = 0, NE_ = 0;
    std::vector<int> slot_of_;    // [layer * NE + expert] -> slot, or -1
    std::vector<uint32_t> freq_;  // selections per (layer, expert)
    std::vector<int> key_of_;     // slot -> key, or -1
    std::vector<uint64_t> last_;  // slot -> tick of its last use
    std::vector<uint64_t> inuse_; // slot -> tick of the layer using it
    std::vector<int> free_;       // never-used slots
    std::vector<int> keys_;       // admitted keys (may hold stale ones), at most keycap_
    size_t keycap_ = 0;
    uint64_t tick_ = 0, rng_ = 0x9E3779B97F4A7C15ull;
};

}  // namespace bt
