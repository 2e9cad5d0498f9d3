"""Prefix KV reuse.

PrefixCache — the conversation cache of src/mlx_dspark/prefix_cache.py:111-249 with the same
rules: a small LRU of finished generations (token record = prompt + generated[:-1], since the
last generated token is the pending one, never fed through the target); a request reuses the
slot with the longest common prefix, reuse = min(lcp, len(cached), len(prompt) - 1), only if
reuse >= min_reuse (16); the chosen slot is checked out until store() re-validates it. On the
paged caches here, trimming a slot to the shared prefix is a length update (O(1)).

PrefixBlocks — block reuse across concurrent rows, the B200 form the batch engine uses: the
whole 64-token pages of a stored prompt prefix are mapped into a new row's block table with a
reference count (the row never writes below its own length, so shared pages stay read-only),
the partially covered last page is copied, and only the rest of the prompt is prefilled. The
reference has no cross-row reuse (its batch engine skips the prefix cache for batched rows,
server.py:388-390); this is what makes the shared 2048-token prefix of BASELINE's C4
workload one prefill instead of 32.
"""
from __future__ import annotations

from .kvcache import PAGE, CacheState


def _lcp(a: list[int], b: list[int]) -> int:
    n = min(len(a), len(b))
    i = 0
    while i < n and a[i] == b[i]:
        i += 1
    return i


def _trim_target(cache, to_len: int) -> None:
    for c in cache:
        off = getattr(c, "offset", None)
        if off is None or not hasattr(c, "trim"):
            continue
        n = int(off) - to_len
        if n > 0:
            c.trim(n)


def target_cache_reusable(cache) -> bool:
    """Whether a target cache can be cut back to any earlier length exactly, which reuse of a
    stored conversation needs (the reference's rule, prefix_cache.py:62-79, restated for the
    caches here). The caches this build makes are paged (kvcache.TargetCache over a
    CacheState), where a trim is a length update, so they always can. A cache object handed in
    by a caller qualifies when every layer view offers offset and trim; a sliding-window view
    (mlx-lm's RotatingKVCache) also has to report its window (max_size) and whether it has
    wrapped (is_trimmable), which store() checks before keeping it."""
    if isinstance(getattr(cache, "state", None), CacheState):
        return True

    def view_ok(c) -> bool:
        if not (hasattr(c, "offset") and callable(getattr(c, "trim", None))):
            return False
        if type(c).__name__ == "RotatingKVCache" or getattr(c, "max_size", None) is not None:
            return hasattr(c, "max_size") and callable(getattr(c, "is_trimmable", None))
        return True

    return all(view_ok(c) for c in cache)


def _storable(cache) -> bool:
    for c in cache:
        fn = getattr(c, "is_trimmable", None)
        if callable(fn) and not fn():
            return False
    return True


class _Slot:
    __slots__ = ("tokens", "cache", "ctx", "sid")

    def __init__(self, tokens, cache, ctx, sid: int):
        self.tokens: list[int] = tokens
        self.cache = cache
        self.ctx = ctx
        self.sid = sid


class PrefixCache:
    def __init__(self, make_cache, make_ctx=None, *, min_reuse: int = 16,
                 l2_dir: str | None = None, max_ram_bytes: int = 0, slots: int = 2):
        if l2_dir:
            raise NotImplementedError("the SSD spill of cached conversations is not built")
        self.make_cache = make_cache
        self.make_ctx = make_ctx
        self.min_reuse = max(1, min_reuse)
        self.l2_dir = None
        self.max_ram_bytes = max_ram_bytes
        self.max_slots = max(1, slots)
        self.hits = 0
        self.reused_tokens = 0
        self._slots: list[_Slot] = []     # most recently used first
        self._next_sid = 0

    def acquire(self, prompt_ids: list[int]):
        """(cache, ctx, reuse_len): the best-matching slot's caches trimmed to the shared prefix
        (checked out until store()), or fresh caches."""
        best, best_len = None, 0
        for slot in self._slots:
            lcp = _lcp(slot.tokens, prompt_ids)
            reuse = max(0, min(lcp, len(slot.tokens), len(prompt_ids) - 1))
            if reuse > best_len:
                best, best_len = slot, reuse
        if best is not None and best_len >= self.min_reuse:
            self._slots.remove(best)
            _trim_target(best.cache, best_len)
            if best.ctx is not None:
                for c in best.ctx:
                    c.trim_to(best_len)
            self.hits += 1
            self.reused_tokens += best_len
            return best.cache, best.ctx, best_len
        return self.make_cache(), (self.make_ctx() if self.make_ctx else None), 0

    def store(self, cache, ctx, prompt_ids: list[int], token_ids: list[int]) -> None:
        if not _storable(cache):
            return
        slot = _Slot(list(prompt_ids) + list(token_ids[:-1]), cache, ctx, self._next_sid)
        self._next_sid += 1
        self._slots.insert(0, slot)
        while len(self._slots) > self.max_slots:
            self._evict(self._slots.pop())

    def reset(self) -> None:
        for s in self._slots:
            self._evict(s)
        self._slots = []

    def info(self) -> dict:
        newest = self._slots[0] if self._slots else None
        return {"enabled": True,
                "cached_tokens": len(newest.tokens) if newest else 0,
                "slots": [{"tokens": len(s.tokens), "spilled": False} for s in self._slots],
                "hits": self.hits, "reused_tokens": self.reused_tokens, "l2": False}

    @staticmethod
    def _evict(slot: _Slot) -> None:
        for obj in (slot.cache, slot.ctx):
            rel = getattr(obj, "release", None)
            if callable(rel):
                rel()


class PrefixBlocks:
    """Shared prompt prefixes as refcounted page lists for the rows of a batch engine."""

    def __init__(self, tstate: CacheState, cstate: CacheState | None, *, min_reuse: int = 16,
                 entries: int = 4):
        self.tstate, self.cstate = tstate, cstate
        self.min_reuse = max(1, min_reuse)
        self.max_entries = max(1, entries)
        self._entries: list[tuple[list[int], list[int], list[int]]] = []  # MRU first
        self.hits = 0
        self.reused_tokens = 0

    def lookup(self, prompt_ids: list[int]):
        """Longest stored prefix usable for this prompt: (entry, reuse_len) or (None, 0).
        reuse_len never reaches the whole prompt (the last token must be prefilled)."""
        best, best_len = None, 0
        for e in self._entries:
            n = min(_lcp(e[0], prompt_ids), len(prompt_ids) - 1)
            if n > best_len:
                best, best_len = e, n
        if best is None or best_len < self.min_reuse:
            return None, 0
        return best, best_len

    def map_row(self, row: int, prompt_ids: list[int]) -> int:
        """Map the longest stored prefix of `prompt_ids` into `row` of both caches; returns
        the number of prompt tokens now cached in the row (0 on a miss)."""
        entry, n = self.lookup(prompt_ids)
        if entry is None:
            return 0
        tokens, tpages, cpages = entry
        self._entries.remove(entry)
        self._entries.insert(0, entry)
        self.tstate.share_prefix(row, tpages, n)
        if self.cstate is not None:
            self.cstate.share_prefix(row, cpages, n)
        self.hits += 1
        self.reused_tokens += n
        return n

    def store_row(self, row: int, prompt_ids: list[int]) -> None:
        """Keep the whole pages of `row`'s prompt (its first len(prompt) positions) for later
        rows; the entry holds a reference so the pages outlive the row."""
        full = len(prompt_ids) // PAGE
        if full * PAGE < self.min_reuse:
            return
        for e in self._entries:
            if len(e[0]) >= full * PAGE and e[0][:full * PAGE] == prompt_ids[:full * PAGE]:
                return  # already covered by an entry at least as long
        tp = list(self.tstate.pages[row][:full])
        cp = list(self.cstate.pages[row][:full]) if self.cstate is not None else []
        self.tstate.pool.retain(tp)
        if self.cstate is not None:
            self.cstate.pool.retain(cp)
        self._entries.insert(0, (list(prompt_ids[:full * PAGE]), tp, cp))
        while len(self._entries) > self.max_entries:
            _, tp, cp = self._entries.pop()
            self.tstate.pool.release(tp)
            if self.cstate is not None:
                self.cstate.pool.release(cp)

    def reset(self) -> None:
        for _, tp, cp in self._entries:
            self.tstate.pool.release(tp)
            if self.cstate is not None:
                self.cstate.pool.release(cp)
        self._entries = []
