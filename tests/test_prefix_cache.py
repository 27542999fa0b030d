"""PrefixCache (host logic) against the reference's own tests,
prefix_cache.rs:116-226: misses, exact and prefix matches, the longest
prefix winning, non-prefix entries ignored, refreshing a key, LRU eviction,
capacity at least one.  (The stored logits of CachedPrefix are not kept:
speculative_generate does not read them, generate.rs:617-627.)"""
import modelc_b200 as mb


class Dummy:
    def __init__(self, n):
        self.n = n
        self.closed = False

    def close(self):
        self.closed = True


def test_lookup_miss_returns_none():
    pc = mb.PrefixCache(4)
    assert pc.lookup([1, 2, 3]) is None
    assert pc.is_empty()


def test_exact_match():
    pc = mb.PrefixCache(4)
    pc.insert([1, 2, 3], Dummy(3))
    look = pc.lookup([1, 2, 3])
    assert look.matched_len == 3 and look.kv.n == 3


def test_prefix_match_returns_the_entry():
    pc = mb.PrefixCache(4)
    pc.insert([1, 2], Dummy(2))
    look = pc.lookup([1, 2, 3, 4])
    assert look.matched_len == 2 and look.kv.n == 2


def test_longest_prefix_wins():
    pc = mb.PrefixCache(4)
    pc.insert([1], Dummy(1))
    pc.insert([1, 2, 3], Dummy(3))
    assert pc.lookup([1, 2, 3, 4]).matched_len == 3


def test_tie_goes_to_the_most_recent_entry():
    pc = mb.PrefixCache(4)
    a, b = Dummy(2), Dummy(2)
    pc.insert([1, 2], a)
    pc.insert([1, 2], b)  # same key: refreshed, the old value closed
    assert pc.lookup([1, 2, 3]).kv is b and a.closed


def test_non_prefix_entry_is_ignored():
    pc = mb.PrefixCache(4)
    pc.insert([9, 9], Dummy(2))
    assert pc.lookup([1, 2, 9, 9]) is None


def test_insert_refreshes_existing_key():
    pc = mb.PrefixCache(4)
    pc.insert([1, 2], Dummy(2))
    new = Dummy(2)
    pc.insert([1, 2], new)
    assert len(pc) == 1
    assert pc.lookup([1, 2]).kv is new


def test_lru_eviction_drops_oldest():
    pc = mb.PrefixCache(2)
    first = Dummy(1)
    pc.insert([1], first)
    pc.insert([2], Dummy(1))
    pc.insert([3], Dummy(1))
    assert len(pc) == 2
    assert pc.lookup([1, 2]) is None and first.closed
    assert pc.lookup([2]) is not None
    assert pc.lookup([3]) is not None


def test_capacity_minimum_is_one():
    assert mb.PrefixCache(0).capacity() == 1
