"""PrefixCache rules, restating the reference's model-free prefix-cache tests
(tests/test_prefix_cache.py:64-189: LCP, reuse eligibility, LRU slots, the min-reuse gate,
the all-but-last-token bookkeeping, the reuse cap below the prompt length, reset) on the same
inputs with the same fake caches."""
from mlx_dspark_b200.prefix_cache import PrefixCache, _lcp, target_cache_reusable


class KVCache:
    def __init__(self, offset=0):
        self.offset = offset

    def trim(self, n):
        n = min(n, self.offset)
        self.offset -= n
        return n


class RotatingKVCache:
    offset = 0

    def trim(self, n):
        return 0


class RealRotatingKVCache:
    def __init__(self, offset=0, max_size=512):
        self.offset = offset
        self.max_size = max_size

    def is_trimmable(self):
        return self.offset < self.max_size

    def trim(self, n):
        n = min(self.offset, n)
        self.offset -= n
        return n


RealRotatingKVCache.__name__ = "RotatingKVCache"


class FakeCtx:
    def __init__(self):
        self.k = self.v = None
        self.trimmed_to = None

    def trim_to(self, length):
        self.trimmed_to = length


def _mk_cache():
    return [KVCache(), KVCache()]


def _mk_ctx():
    return [FakeCtx(), FakeCtx()]


def test_lcp():
    assert _lcp([1, 2, 3], [1, 2, 9]) == 2
    assert _lcp([1, 2, 3], [1, 2, 3, 4]) == 3
    assert _lcp([], [1]) == 0
    assert _lcp([5], [6]) == 0


def test_reusable_detection():
    assert target_cache_reusable([KVCache(), KVCache()]) is True
    assert target_cache_reusable([KVCache(), RotatingKVCache()]) is False
    assert target_cache_reusable([KVCache(), RealRotatingKVCache()]) is True


def test_wrapped_rotating_cache_is_not_stored():
    pc = PrefixCache(_mk_cache, _mk_ctx, min_reuse=1)
    prompt = list(range(20))
    cache = [RealRotatingKVCache(max_size=16), KVCache()]
    ctx = _mk_ctx()
    cache[0].offset = 16
    cache[1].offset = 21
    pc.store(cache, ctx, prompt, [99, 100])
    assert pc.info()["cached_tokens"] == 0
    cache[0].offset = 10
    pc.store(cache, ctx, prompt, [99, 100])
    assert pc.info()["cached_tokens"] == 21


def test_lru_two_slots_dont_evict_each_other():
    pc = PrefixCache(_mk_cache, _mk_ctx, min_reuse=4, slots=2)
    conv_a, conv_b = list(range(100, 120)), list(range(200, 220))
    ca, xa, _ = pc.acquire(conv_a)
    for c in ca:
        c.offset = len(conv_a)
    pc.store(ca, xa, conv_a, [1, 2])
    cb, xb, _ = pc.acquire(conv_b)
    assert cb is not ca
    for c in cb:
        c.offset = len(conv_b)
    pc.store(cb, xb, conv_b, [3, 4])
    got_a, _, reuse_a = pc.acquire(conv_a + [1, 130])
    assert got_a is ca and reuse_a == len(conv_a) + 1
    pc.store(got_a, xa, conv_a + [1, 130], [5, 6])
    got_b, _, reuse_b = pc.acquire(conv_b + [3, 230])
    assert got_b is cb and reuse_b == len(conv_b) + 1
    assert pc.hits == 2


def test_lru_eviction_beyond_capacity():
    pc = PrefixCache(_mk_cache, _mk_ctx, min_reuse=4, slots=2)
    convs = [list(range(i * 100, i * 100 + 20)) for i in (1, 2, 3)]
    for conv in convs:
        c, x, _ = pc.acquire(conv)
        for layer in c:
            layer.offset = len(conv)
        pc.store(c, x, conv, [7, 8])
    assert len(pc.info()["slots"]) == 2
    assert pc.acquire(convs[0] + [9])[2] == 0
    assert pc.acquire(convs[2] + [9])[2] > 0


def test_acquire_empty_is_fresh():
    pc = PrefixCache(_mk_cache, _mk_ctx, min_reuse=4)
    cache, ctx, reuse_len = pc.acquire([1, 2, 3, 4, 5])
    assert reuse_len == 0 and len(cache) == 2 and len(ctx) == 2


def test_store_bookkeeping_and_reuse():
    pc = PrefixCache(_mk_cache, _mk_ctx, min_reuse=4)
    prompt, gen = list(range(1, 11)), [11, 12, 13]
    cache, ctx, _ = pc.acquire(prompt)
    for c in cache:
        c.offset = len(prompt) + len(gen) - 1
    pc.store(cache, ctx, prompt, gen)
    assert pc.info()["cached_tokens"] == 12
    cache2, ctx2, reuse_len = pc.acquire([1, 2, 3, 4, 5, 6, 50, 51])
    assert reuse_len == 6
    assert cache2 is cache and all(c.offset == 6 for c in cache2)
    assert all(c.trimmed_to == 6 for c in ctx2)
    assert pc.hits == 1 and pc.reused_tokens == 6


def test_min_reuse_gate():
    pc = PrefixCache(_mk_cache, _mk_ctx, min_reuse=8)
    prompt = list(range(1, 11))
    cache, ctx, _ = pc.acquire(prompt)
    for c in cache:
        c.offset = len(prompt) - 1
    pc.store(cache, ctx, prompt, [99])
    assert pc.acquire([1, 2, 3, 500, 501, 502])[2] == 0 and pc.hits == 0


def test_reuse_len_capped_below_prompt_len():
    pc = PrefixCache(_mk_cache, _mk_ctx, min_reuse=1)
    prompt = [1, 2, 3, 4, 5]
    cache, ctx, _ = pc.acquire(prompt)
    for c in cache:
        c.offset = len(prompt) - 1
    pc.store(cache, ctx, prompt, [6])
    assert pc.acquire([1, 2, 3, 4, 5])[2] == 4


def test_reset_invalidates():
    pc = PrefixCache(_mk_cache, _mk_ctx, min_reuse=1)
    cache, ctx, _ = pc.acquire([1, 2, 3])
    for c in cache:
        c.offset = 2
    pc.store(cache, ctx, [1, 2, 3], [4])
    pc.reset()
    assert pc.info()["cached_tokens"] == 0
    assert pc.acquire([1, 2, 3])[2] == 0
