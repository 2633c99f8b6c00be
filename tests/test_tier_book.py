"""The tiered pool's host bookkeeping (hale-token_b200/csrc/hale_tier.h) on
the CPU: random forwards of per-token requests checked against a host
restatement of ExpertCache::fetch + LruCache (src/expert/cache.rs:124-194,
src/expert/lru.rs:97-125), and against the invariants the GPU path relies
on -- every expert a forward names sits in a slot holding its bytes until
the forward ends, pinned slots never move, and no slot serves two experts.
The same header drives hale_pool_create_tiered pools.
"""
import ctypes as C
import os
import shutil
import subprocess
from collections import OrderedDict

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def lib(tmp_path_factory):
    gxx = shutil.which("g++")
    if not gxx:
        pytest.skip("g++ not available")
    out = str(tmp_path_factory.mktemp("tier") / "libtier.so")
    subprocess.check_call([gxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-o", out,
                           os.path.join(HERE, "tier_harness.cpp")])
    L = C.CDLL(out)
    P, I64, U64 = C.c_void_p, C.c_int64, C.c_uint64
    L.tier_create.restype = P
    L.tier_create.argtypes = [U64, P, U64, U64, U64, U64]
    L.tier_destroy.argtypes = [P]
    L.tier_slots.restype = C.c_uint32
    L.tier_slots.argtypes = [P]
    L.tier_request.restype = I64
    L.tier_request.argtypes = [P, P, U64, P, U64]
    L.tier_release.argtypes = [P]
    L.tier_counters.argtypes = [P, P]
    L.tier_slot_of.restype = C.c_int32
    L.tier_slot_of.argtypes = [P, I64]
    L.tier_routing.restype = U64
    L.tier_routing.argtypes = [P, I64]
    return L


class RefCache:
    """ExpertCache::fetch over LruCache (byte budget, equal weights)."""

    def __init__(self, pinned, lru_bytes, w):
        self.pinned, self.cap, self.w = set(pinned), lru_bytes, w
        self.lru = OrderedDict()
        self.c = [0, 0, 0]

    def fetch(self, keys):
        missing = []
        for k in keys:
            if k in self.pinned:
                self.c[0] += 1
            elif k in self.lru:
                self.lru.move_to_end(k)
                self.c[1] += 1
            else:
                missing.append(k)
        for k in missing:
            self.lru.pop(k, None)
            if self.w > self.cap:
                continue
            while (len(self.lru) + 1) * self.w > self.cap:
                self.lru.popitem(last=False)
            self.lru[k] = True
        self.c[2] += len(missing)


@pytest.mark.parametrize("seed", range(6))
@pytest.mark.parametrize("shape", [(3, 16, 4, 0, 1), (2, 8, 2, 2, 3), (4, 32, 8, 5, 0), (1, 8, 3, 1, 20)])
def test_book_matches_the_reference_cache_and_keeps_slots_safe(lib, seed, shape):
    layers, E, k, n_pinned, lru_experts = shape
    rng = np.random.default_rng([seed, layers, E])
    n_keys, w = layers * E, 1000
    pinned = sorted({int(x) for x in rng.choice(n_keys, size=n_pinned, replace=False)}) if n_pinned else []
    parr = (C.c_int64 * max(1, len(pinned)))(*pinned)
    h = lib.tier_create(n_keys, C.cast(parr, C.c_void_p), len(pinned), lru_experts * w, w, E)
    try:
        n_slots = lib.tier_slots(h)
        assert n_slots == min(n_keys, len(pinned) + lru_experts + E)
        pinned_slot = {p: lib.tier_slot_of(h, p) for p in pinned}
        ref = RefCache(pinned, lru_experts * w, w)
        content = {}  # slot -> key whose bytes it holds (pinned slots uploaded at creation)
        for p, s in pinned_slot.items():
            content[s] = p
        out = (C.c_int64 * (2 * n_keys + 2))()
        routed = np.zeros(n_keys, np.int64)
        for fwd in range(40):
            lib.tier_release(h)
            layer = int(rng.integers(layers))
            m = int(rng.integers(1, 7))
            named = set()
            for _ in range(m):
                experts = rng.choice(E, size=k, replace=False)
                keys = [layer * E + int(e) for e in experts]
                karr = (C.c_int64 * k)(*keys)
                got = lib.tier_request(h, C.cast(karr, C.c_void_p), k, C.cast(out, C.c_void_p), n_keys + 1)
                assert got >= 0, "ran out of slots"
                for i in range(got):
                    s, key = out[2 * i], out[2 * i + 1]
                    assert 0 <= s < n_slots and s not in pinned_slot.values()
                    content[s] = key
                ref.fetch(keys)
                for key in keys:
                    routed[key] += 1
                named.update(keys)
            # every expert the forward named is resident with its own bytes at
            # the end of the forward (so no copy overwrote a slot still in use)
            slots = {key: lib.tier_slot_of(h, key) for key in named}
            for key, s in slots.items():
                assert s >= 0 and content[s] == key, f"forward {fwd}: key {key}"
            assert len(set(slots.values())) == len(slots)
            for p, s in pinned_slot.items():
                assert lib.tier_slot_of(h, p) == s
        c = (C.c_uint64 * 6)()
        lib.tier_counters(h, C.cast(c, C.c_void_p))
        assert list(c[:3]) == ref.c
        assert c[3] == ref.c[2] * w
        assert (c[4], c[5]) == (len(ref.lru), len(ref.lru) * w)
        assert all(lib.tier_routing(h, key) == routed[key] for key in range(n_keys))
    finally:
        lib.tier_destroy(h)


def test_a_request_beyond_the_slots_is_refused(lib):
    # 2 layers x 4 experts, no pinned, no LRU: slots = one layer's 4 experts
    h = lib.tier_create(8, None, 0, 0, 1000, 4)
    try:
        out = (C.c_int64 * 20)()
        keys = (C.c_int64 * 6)(0, 1, 2, 3, 4, 5)   # 6 distinct experts of two layers in one request
        assert lib.tier_request(h, C.cast(keys, C.c_void_p), 6, C.cast(out, C.c_void_p), 10) == -1
    finally:
        lib.tier_destroy(h)
