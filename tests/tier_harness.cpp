// C entry points over hale_tier::Book so tests/test_tier_book.py can drive
// the tiered pool's bookkeeping on the CPU (built by the test with g++).
#include <cstdint>
#include <vector>

#include "../hale-token_b200/csrc/hale_tier.h"

extern "C" {

void* tier_create(uint64_t n_keys, const int64_t* pinned, uint64_t n_pinned, uint64_t lru_bytes,
                  uint64_t record_bytes, uint64_t per_request) {
    auto* b = new hale_tier::Book();
    std::vector<int64_t> pk(pinned, pinned + n_pinned);
    std::vector<uint8_t> seen(n_keys, 0);
    uint64_t distinct = 0;
    for (int64_t k : pk)
        if (!seen[k]) {
            seen[k] = 1;
            distinct++;
        }
    b->init(n_keys, pk, lru_bytes, record_bytes,
            hale_tier::Book::slots_needed(n_keys, distinct, lru_bytes, record_bytes, per_request));
    return b;
}

void tier_destroy(void* h) { delete static_cast<hale_tier::Book*>(h); }

uint32_t tier_slots(void* h) { return static_cast<hale_tier::Book*>(h)->n_slots; }

// Returns the number of (slot, key) copies written to out, or -1 when no slot
// was free.
int64_t tier_request(void* h, const int64_t* keys, uint64_t n, int64_t* out, uint64_t cap) {
    std::vector<std::pair<int32_t, int64_t>> loads;
    if (!static_cast<hale_tier::Book*>(h)->request(keys, n, loads)) return -1;
    if (loads.size() > cap) return -2;
    for (size_t i = 0; i < loads.size(); i++) {
        out[2 * i] = loads[i].first;
        out[2 * i + 1] = loads[i].second;
    }
    return (int64_t)loads.size();
}

void tier_release(void* h) { static_cast<hale_tier::Book*>(h)->release(); }

void tier_counters(void* h, uint64_t* out) {
    const auto* b = static_cast<hale_tier::Book*>(h);
    out[0] = b->c.pinned_hits;
    out[1] = b->c.lru_hits;
    out[2] = b->c.misses;
    out[3] = b->c.bytes_loaded;
    out[4] = b->lru.count;
    out[5] = b->lru.used;
}

int32_t tier_slot_of(void* h, int64_t key) { return static_cast<hale_tier::Book*>(h)->slot_of[key]; }

uint64_t tier_routing(void* h, int64_t key) { return static_cast<hale_tier::Book*>(h)->routing[key]; }
}
