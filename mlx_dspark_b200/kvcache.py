"""Paged KV cache: page pools in HBM, per-row block tables and device-resident lengths.

Layout (one pool per model, all layers): ``data[layer, page, page_bytes]`` uint8 with the
page format of include/dspark_b200.h (bf16 or 8-bit affine group-64 pages of 64 tokens).
A row's logical position p lives in page ``block_table[row, p // 64]``. The lengths that
kernels read (``seq_len``) live on the device, so commit / rollback (``seq_len += n + 1``)
happens inside a captured round without a host round trip.

Reference semantics kept (mlx-lm KVCache as used by src/mlx_dspark/target.py:36-48 and the
per-row BatchCache of src/mlx_dspark/batch_engine.py:61-163):
  * ``offset`` is the logical length; ``trim(n)`` only moves it back (the stale tail is
    overwritten by the next write), clamped at zero;
  * a multi-token update writes at the current offset and advances it;
  * every layer of a cache has its own ``offset``/``trim`` (generate.py:929-933 trims each
    layer; prefix_cache._trim_target trims each layer to a target length).
"""
from __future__ import annotations

import torch

from . import ops

PAGE = 64


class PagePool:
    """Physical pages of one model (all layers share the page numbering)."""

    def __init__(self, n_layers: int, num_pages: int, num_kv_heads: int, head_dim: int,
                 kv8: bool, device="cuda"):
        self.n_layers = n_layers
        self.num_pages = num_pages
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.kv8 = bool(kv8)
        self.page_bytes = ops.kv_page_bytes(PAGE, num_kv_heads, head_dim, kv8)
        # zero-filled: masked attention reads stale-but-finite tails only
        self.data = torch.zeros(n_layers, num_pages, self.page_bytes, dtype=torch.uint8,
                                device=device)
        self.free = list(range(num_pages - 1, -1, -1))
        self.refs = [0] * num_pages
        self.version = 0          # bumped when `data` moves (layouts hold its address)
        self.growable = True

    def grow(self, num_pages: int) -> None:
        """Reallocate to `num_pages` pages, copying the old ones (page ids stay valid)."""
        if num_pages <= self.num_pages:
            return
        data = torch.zeros(self.n_layers, num_pages, self.page_bytes, dtype=torch.uint8,
                           device=self.data.device)
        data[:, :self.num_pages].copy_(self.data)
        self.data = data
        self.free = list(range(num_pages - 1, self.num_pages - 1, -1)) + self.free
        self.refs += [0] * (num_pages - self.num_pages)
        self.num_pages = num_pages
        self.version += 1

    def alloc(self, n: int) -> list[int]:
        if n > len(self.free) and self.growable:
            self.grow(self.num_pages + max(n - len(self.free), self.num_pages // 2))
        if n > len(self.free):
            raise MemoryError(f"KV page pool exhausted ({n} pages wanted, {len(self.free)} free)")
        out = [self.free.pop() for _ in range(n)]
        for p in out:
            self.refs[p] = 1
        return out

    def retain(self, pages) -> None:
        for p in pages:
            self.refs[p] += 1

    def release(self, pages) -> None:
        for p in pages:
            self.refs[p] -= 1
            if self.refs[p] == 0:
                self.free.append(p)

    def layout(self, layer: int, block_table: torch.Tensor) -> ops.KvLayout:
        return ops.kv_layout(self.data[layer], block_table, PAGE, self.num_kv_heads,
                             self.head_dim, self.kv8)

    def nbytes(self) -> int:
        return self.data.numel()


class CacheState:
    """Rows x pages bookkeeping for one batch of sequences over a PagePool."""

    def __init__(self, pool: PagePool, rows: int, max_tokens: int, device="cuda"):
        self.pool = pool
        self.rows = rows
        self.max_pages = (max_tokens + PAGE - 1) // PAGE
        self.block_table = torch.zeros(rows, self.max_pages, dtype=torch.int32, device=device)
        self.seq_len = torch.zeros(rows, dtype=torch.int32, device=device)
        self.pages: list[list[int]] = [[] for _ in range(rows)]
        self.host_len = [0] * rows
        self._layouts = None
        self._layout_version = -1

    # -- pages --
    def grow(self, max_tokens: int) -> None:
        """Widen the block table so rows can hold `max_tokens` positions (pages stay put)."""
        need = (max_tokens + PAGE - 1) // PAGE
        if need <= self.max_pages:
            return
        bt = torch.zeros(self.rows, need, dtype=torch.int32, device=self.block_table.device)
        bt[:, :self.max_pages] = self.block_table
        self.block_table = bt
        self.max_pages = need
        self._layouts = None

    def ensure(self, row: int, tokens: int) -> None:
        """Make sure positions [0, tokens) of `row` have pages."""
        need = (tokens + PAGE - 1) // PAGE
        if need > self.max_pages:
            raise ValueError(f"row {row}: {tokens} tokens exceed the cache capacity "
                             f"({self.max_pages * PAGE})")
        have = len(self.pages[row])
        if need > have:
            new = self.pool.alloc(need - have)
            self.pages[row].extend(new)
            self.block_table[row, have:need] = torch.tensor(new, dtype=torch.int32)

    def share_prefix(self, row: int, src_pages: list[int], tokens: int) -> None:
        """Map the first `tokens` positions of `row` onto existing pages (prefix reuse).
        Only whole pages are shared; a partially covered last page is copied."""
        self.release_row(row)
        full = tokens // PAGE
        shared = list(src_pages[:full])
        self.pool.retain(shared)
        self.pages[row] = shared
        if shared:
            self.block_table[row, :full] = torch.tensor(shared, dtype=torch.int32)
        rem = tokens - full * PAGE
        if rem:
            (p,) = self.pool.alloc(1)
            self.pool.data[:, p].copy_(self.pool.data[:, src_pages[full]])
            self.pages[row].append(p)
            self.block_table[row, full] = p
        self.set_len(row, tokens)

    def release_row(self, row: int) -> None:
        self.pool.release(self.pages[row])
        self.pages[row] = []
        self.set_len(row, 0)

    def release(self) -> None:
        for r in range(self.rows):
            self.release_row(r)

    # -- lengths --
    def set_len(self, row: int, n: int) -> None:
        self.host_len[row] = n
        self.seq_len[row] = n

    def sync_from_device(self) -> list[int]:
        self.host_len = [int(x) for x in self.seq_len.tolist()]
        return self.host_len

    def move_row(self, src: int, dst: int) -> None:
        """Row dst takes over row src's pages and length (batch compaction: a block-table row
        copy, no KV bytes move); row src is left empty. dst's old pages must be released."""
        assert not self.pages[dst], "move_row: release the destination row first"
        self.pages[dst] = self.pages[src]
        self.pages[src] = []
        self.block_table[dst].copy_(self.block_table[src])
        self.seq_len[dst] = self.seq_len[src]
        self.host_len[dst] = self.host_len[src]
        self.set_len(src, 0)

    def layout(self, layer: int) -> ops.KvLayout:
        if self._layouts is None or self._layout_version != self.pool.version:
            self._layouts = [self.pool.layout(l, self.block_table) for l in range(self.pool.n_layers)]
            self._layout_version = self.pool.version
        return self._layouts[layer]


class RowView:
    """One row of a CacheState seen as a one-row state (slices share storage), so a row can
    be prefilled alone while the batch's buffers stay in place."""

    def __init__(self, state: CacheState, row: int):
        self.pool = state.pool
        self.rows = 1
        self.max_pages = state.max_pages
        self.block_table = state.block_table[row:row + 1]
        self.seq_len = state.seq_len[row:row + 1]
        self._layouts = None
        self._layout_version = -1

    def layout(self, layer: int) -> ops.KvLayout:
        if self._layouts is None or self._layout_version != self.pool.version:
            self._layouts = [self.pool.layout(l, self.block_table) for l in range(self.pool.n_layers)]
            self._layout_version = self.pool.version
        return self._layouts[layer]


class LayerCache:
    """One layer's view of a single-row cache: the mlx-lm KVCache duck type."""

    def __init__(self, parent: "TargetCache", layer: int):
        self._parent = parent
        self.layer = layer
        self.offset = 0

    def trim(self, n: int) -> int:
        n = max(0, min(int(n), self.offset))
        self.offset -= n
        return n

    def is_trimmable(self) -> bool:
        return True

    @property
    def state(self):
        """Bytes held for RAM accounting (prefix_cache._cache_ram_bytes duck type)."""
        s = self._parent.state
        return [_Bytes(s.pool.page_bytes * len(s.pages[0]))]


class _Bytes:
    def __init__(self, n):
        self.nbytes = n


class TargetCache(list):
    """make_cache() result for one sequence: a list of per-layer LayerCache views over one
    CacheState. The device length follows the layers' common offset before each forward."""

    def __init__(self, state: CacheState, n_layers: int, kind: str = "KVCache"):
        super().__init__(LayerCache(self, l) for l in range(n_layers))
        self.state = state
        self.kind = kind

    @property
    def offset(self) -> int:
        return self[0].offset

    def common_offset(self) -> int:
        offs = {c.offset for c in self}
        if len(offs) != 1:
            raise ValueError(f"layers of one cache disagree on the offset: {sorted(offs)}")
        return offs.pop()

    def sync_to_device(self) -> int:
        off = self.common_offset()
        if self.state.host_len[0] != off:
            self.state.set_len(0, off)
        return off

    def advance(self, n: int) -> None:
        for c in self:
            c.offset += n
        self.state.host_len[0] += n

    def set_offset(self, n: int) -> None:
        for c in self:
            c.offset = n
        self.state.host_len[0] = n

    def release(self) -> None:
        self.state.release()


class _CtxLayer:
    """One layer's view of a drafter context cache (reference CtxCache duck type,
    src/mlx_dspark/model.py:48-80): every layer shares the cache's single length."""

    def __init__(self, parent: "CtxCaches"):
        self._parent = parent

    @property
    def length(self) -> int:
        return self._parent.state.host_len[0]

    def trim_to(self, length: int) -> None:
        st = self._parent.state
        if length < st.host_len[0]:
            st.set_len(0, max(0, int(length)))


class CtxCaches(list):
    """make_ctx_cache() result for one sequence: per-layer views over one CacheState."""

    def __init__(self, state: CacheState, n_layers: int):
        super().__init__(_CtxLayer(self) for _ in range(n_layers))
        self.state = state

    @property
    def length(self) -> int:
        return self.state.host_len[0]

    def release(self) -> None:
        self.state.release()
