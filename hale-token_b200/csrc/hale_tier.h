// hale_tier.h -- host bookkeeping of a tiered expert pool (plain C++, no CUDA).
//
// Expert keys are 0 .. n_keys-1 (pool layer * experts + expert). HBM holds
// n_slots experts: the pinned keys (their slots fixed for the pool's life),
// the keys an LRU with the reference's byte budget keeps, and the keys the
// current request still needs. `request` applies ExpertCache::fetch
// (src/expert/cache.rs:124-194) to one request and returns the copies to
// issue (slot <- key); `release` ends the previous request, after its
// kernels have completed, and frees the slots no tier keeps. hale_cuda.cu
// drives this for hale_pool_create_tiered pools; tests/ drive it on the CPU.
#pragma once

#include <cstddef>
#include <cstdint>
#include <utility>
#include <vector>

namespace hale_tier {

// LruCache (src/expert/lru.rs:40-160) over keys 0 .. n-1: a doubly linked
// recency list in index arrays, every entry of the same weight (one expert
// record).
struct KeyLru {
    std::vector<int64_t> prev, next;
    std::vector<uint8_t> in;
    int64_t head = -1, tail = -1;
    uint64_t used = 0, cap = 0, weight = 0;
    size_t count = 0;

    void init(size_t n, uint64_t cap_bytes, uint64_t w) {
        prev.assign(n, -1);
        next.assign(n, -1);
        in.assign(n, 0);
        head = tail = -1;
        used = 0;
        cap = cap_bytes;
        weight = w;
        count = 0;
    }
    void unlink(int64_t k) {
        if (prev[k] >= 0) next[prev[k]] = next[k]; else head = next[k];
        if (next[k] >= 0) prev[next[k]] = prev[k]; else tail = prev[k];
        prev[k] = next[k] = -1;
    }
    void push_front(int64_t k) {
        prev[k] = -1;
        next[k] = head;
        if (head >= 0) prev[head] = k;
        head = k;
        if (tail < 0) tail = k;
    }
    void remove(int64_t k) {
        unlink(k);
        in[k] = 0;
        used -= weight;
        count--;
    }
    // get(): a hit becomes the most recently used entry
    bool get(int64_t k) {
        if (!in[k]) return false;
        unlink(k);
        push_front(k);
        return true;
    }
    // insert(): evicts from the tail until the entry fits; an entry heavier
    // than the whole budget is not stored and comes back as evicted
    void insert(int64_t k, std::vector<int64_t>& evicted) {
        if (in[k]) remove(k);
        if (weight > cap) {
            evicted.push_back(k);
            return;
        }
        while (used + weight > cap) {
            const int64_t t = tail;
            remove(t);
            evicted.push_back(t);
        }
        push_front(k);
        in[k] = 1;
        used += weight;
        count++;
    }
};

// CacheStats counters the book maintains (cache.rs:15-33).
struct Counters {
    uint64_t pinned_hits = 0, lru_hits = 0, misses = 0, bytes_loaded = 0;
};

struct Book {
    uint64_t record_bytes = 0;
    uint32_t n_slots = 0;
    uint64_t n_pinned = 0;
    std::vector<uint8_t> pinned_key;   // [n_keys]
    std::vector<int32_t> slot_of;      // [n_keys] HBM slot or -1
    std::vector<int64_t> slot_key;     // [n_slots] key or -1
    std::vector<int32_t> free_slots;
    std::vector<int64_t> held;         // unpinned keys of the request in flight
    std::vector<uint8_t> held_mark;    // [n_keys]
    std::vector<uint64_t> routing;     // [n_keys] requests per key
    KeyLru lru;
    Counters c;

    // The slot count that always suffices: pinned + LRU capacity + the most
    // distinct keys one request can name (at most n_keys in all).
    static uint32_t slots_needed(size_t n_keys, uint64_t n_pinned, uint64_t lru_bytes, uint64_t record_bytes,
                                 uint64_t per_request) {
        const uint64_t want = n_pinned + lru_bytes / record_bytes + per_request;
        return (uint32_t)(want < n_keys ? want : n_keys);
    }

    // pinned: keys kept in HBM for good (duplicates allowed; keys < n_keys).
    void init(size_t n_keys, const std::vector<int64_t>& pinned, uint64_t lru_bytes, uint64_t rec_bytes,
              uint32_t slots) {
        record_bytes = rec_bytes;
        n_slots = slots;
        pinned_key.assign(n_keys, 0);
        n_pinned = 0;
        for (int64_t k : pinned)
            if (!pinned_key[k]) {
                pinned_key[k] = 1;
                n_pinned++;
            }
        slot_of.assign(n_keys, -1);
        slot_key.assign(slots, -1);
        held.clear();
        held_mark.assign(n_keys, 0);
        routing.assign(n_keys, 0);
        lru.init(n_keys, lru_bytes, rec_bytes);
        c = Counters{};
        // pinned keys take the first slots
        uint32_t next = 0;
        for (size_t k = 0; k < n_keys; k++)
            if (pinned_key[k]) {
                slot_of[k] = (int32_t)next;
                slot_key[next] = (int64_t)k;
                next++;
            }
        free_slots.clear();
        for (int32_t s = (int32_t)slots - 1; s >= (int32_t)next; s--) free_slots.push_back(s);
    }

    void free_slot(int64_t key) {
        const int32_t s = slot_of[key];
        if (s < 0) return;
        slot_of[key] = -1;
        slot_key[s] = -1;
        free_slots.push_back(s);
    }

    // The previous request's kernels have completed: slots of its experts
    // that no tier keeps become free.
    void release() {
        for (int64_t key : held) {
            held_mark[key] = 0;
            if (!pinned_key[key] && !lru.in[key]) free_slot(key);
        }
        held.clear();
    }

    // One request (keys in request order): routing recorded, pass 1 serves
    // pinned and LRU hits (a hit refreshes recency), pass 2 loads the misses
    // in request order and inserts them into the LRU. Every expert of the
    // request keeps its slot until the next release, even if a later insert
    // evicts it from the LRU; a miss whose bytes are still in a held slot
    // needs no copy (it counts as a miss all the same). Several requests may
    // run between releases (one per token of a forward). Returns false when
    // no slot is free, which the slot count above rules out.
    bool request(const int64_t* keys, size_t n, std::vector<std::pair<int32_t, int64_t>>& loads) {
        for (size_t i = 0; i < n; i++) routing[keys[i]]++;
        uint64_t pinned_hits = 0, lru_hits = 0;
        std::vector<int64_t> missing;
        for (size_t i = 0; i < n; i++) {
            const int64_t key = keys[i];
            if (pinned_key[key]) {
                pinned_hits++;
                continue;
            }
            if (!held_mark[key]) {
                held_mark[key] = 1;
                held.push_back(key);
            }
            if (lru.get(key)) lru_hits++;
            else missing.push_back(key);
        }
        std::vector<int64_t> evicted;
        for (int64_t key : missing) {
            if (slot_of[key] < 0) {
                if (free_slots.empty()) return false;
                const int32_t s = free_slots.back();
                free_slots.pop_back();
                slot_of[key] = s;
                slot_key[s] = key;
                loads.emplace_back(s, key);
            }
            evicted.clear();
            lru.insert(key, evicted);
            for (int64_t ev : evicted)
                if (!held_mark[ev]) free_slot(ev);
        }
        c.pinned_hits += pinned_hits;
        c.lru_hits += lru_hits;
        c.misses += missing.size();
        c.bytes_loaded += (uint64_t)missing.size() * record_bytes;
        return true;
    }
};

}  // namespace hale_tier
