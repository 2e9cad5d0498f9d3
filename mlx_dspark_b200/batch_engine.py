"""Continuous batching of speculative decoding on the device (src/mlx_dspark/batch_engine.py).

SpecSlots keeps the reference's slot engine (batch_engine.py:431-598): `capacity` slots, a
request is admitted into the next free slot (single-row prefill seeding its drafter context),
step() runs one speculative round over the active rows, a finished row retires at once and the
last active row is compacted into its place, so every round runs at the active width.

What changes on B200:
  * All rows live in one paged KV cache per model (kvcache.CacheState); a row's rope offset,
    write position and attention length are its device seq_len, so ragged rows need no padding
    mask (build_batch_mask / _ctx_block_mask, batch_engine.py:170-178,401-411, become
    per-row lengths inside the attention kernel) and rollback is the length update alone.
  * Compaction moves a block-table row and a length (CacheState.move_row), not KV bytes
    (BatchCache.move_row copies the row, batch_engine.py:116-126).
  * Admission maps the whole pages of a stored prompt prefix into the new row with a
    reference count (prefix_cache.PrefixBlocks) and prefills only the rest.
  * The round at each active width is one CUDA graph (draft, batched verify, fused greedy
    accept, context update, commit) with one plan read per round.
  * 8-bit KV (QuantizedKVCache(64, 8)) works in the batch: the reference refuses batching with
    kv_bits (batch_engine.py:55); here the KV8 pages are just another page format.
"""
from __future__ import annotations

import time
from collections import deque

import torch

from .generate import (GenResult, GreedySession, SpecSession, _decode, _pick_first,
                       eos_token_ids, prefill_rows)
from .model import Sampling
from .kvcache import PAGE, CacheState, RowView
from .prefix_cache import PrefixBlocks
from .streaming import TextStream


def batchable(target) -> bool:
    """Every target here can batch (paged caches, KV8 included) (batch_engine.py:43-58)."""
    return True


class _RowTracker:
    """One row's committed tokens, its text stream (on_text, stop strings), its eos / length /
    stop-string end and its result (batch_engine.py:254-319)."""

    def __init__(self, tokenizer, first: int, max_new_tokens: int, on_text=None, stop=None):
        self.tok = tokenizer
        self.eos = eos_token_ids(tokenizer)
        self.mnt = int(max_new_tokens)
        self.stream = TextStream(tokenizer, self.eos, on_text, stop)
        self.out_ids = [int(first)]
        self.accept_lengths: list[int] = []
        self.finished = False
        self.stream.update(self.out_ids)
        self._check()

    def _check(self):
        ids = self.out_ids
        if ids[-1] in self.eos or len(ids) >= self.mnt or self.stream.stopped:
            self.finished = True
            self.stream.flush()   # the rest of the text goes out as the row finishes

    def commit(self, tokens, accept_len=None):
        if self.finished:
            return
        if accept_len is not None:
            self.accept_lengths.append(accept_len)
        for t in tokens:
            self.out_ids.append(int(t))
            if t in self.eos:
                break
        self.stream.update(self.out_ids)
        self._check()

    def result(self, secs: float) -> GenResult:
        ids = self.out_ids
        reason = "stop" if (ids[-1] in self.eos or self.stream.stopped) else "length"
        spec = bool(self.accept_lengths)
        al = self.accept_lengths if spec else [1] * len(ids)
        return GenResult(text=self.stream.final_text(self.tok, ids, _decode),
                         token_ids=ids, num_tokens=len(ids), num_rounds=len(al),
                         accept_lengths=al, target_forwards=(len(al) + 1) if spec else len(ids),
                         seconds=secs, finish_reason=reason)


class SpecSlots:
    def __init__(self, target, tokenizer, drafter, *, capacity: int, max_draft_tokens: int = 2,
                 batched_drafter: bool = True, cap_controller=None, max_tokens: int = 4096,
                 prefix_reuse: bool = True, min_reuse: int = 16, use_graph: bool = True):
        if not batched_drafter:
            raise NotImplementedError("the per-row drafter mode (Stage A) is not built; the "
                                      "batched drafter covers it")
        if getattr(drafter, "target", None) is not target:
            drafter.bind(target)
        cfg = drafter.config
        # optional CapController: the cap of a round at batch width B is cap_for(B) (the live
        # cap at B = 1), and every row's outcome feeds its acceptance estimate
        # (batch_engine.py:535-538,595-596); a cap change switches the session's round buffers
        self.ctrl = cap_controller
        self.target, self.tokenizer, self.drafter = target, tokenizer, drafter
        self.tap = list(cfg.target_layer_ids)
        self.k = int(cfg.block_size)
        self.cap = max(1, min(int(max_draft_tokens), self.k))
        self.capacity = int(capacity)
        self.max_tokens = int(max_tokens)
        self.use_graph = use_graph
        C = self.capacity
        # one paged cache per model for all slots; pools are sized up front (captured rounds
        # hold their addresses) with room for the shared prefix entries
        row_pages = (self.max_tokens + PAGE - 1) // PAGE
        extra = 4 * row_pages
        dev = target.device
        self.tstate = CacheState(target.new_pool(self.max_tokens, C, extra_pages=extra), C,
                                 self.max_tokens, dev)
        cpool = drafter.new_pool(self.max_tokens, C + 4)
        self.cstate = CacheState(cpool, C, self.max_tokens, dev)
        self.tstate.pool.growable = False
        self.cstate.pool.growable = False
        self.blocks = PrefixBlocks(self.tstate, self.cstate, min_reuse=min_reuse) if prefix_reuse else None
        self.sessions: dict[int, SpecSession] = {}
        self.n_active = 0
        self.pending = [0] * C
        self.trk: list[_RowTracker | None] = [None] * C
        self.meta = [None] * C
        self.t0 = [0.0] * C
        self.prefill_tokens = 0   # prompt tokens actually prefilled (reuse skips the rest)

    @property
    def has_free_slot(self) -> bool:
        return self.n_active < self.capacity

    def _session(self, B: int) -> SpecSession:
        s = self.sessions.get(B)
        if s is None:
            s = SpecSession(self.target, self.drafter, B, self.cap, self.max_tokens,
                            states=(self.tstate, self.cstate),
                            max_cap=self.k if self.ctrl is not None else None)
            self.sessions[B] = s
        return s

    def admit(self, prompt_ids: list[int], *, max_new_tokens: int, on_text=None, stop=None,
              meta=None) -> None:
        """Prefill one request into the next free slot (reusing a stored prefix's pages)."""
        if not self.has_free_slot:
            raise RuntimeError("SpecSlots.admit: no free slot")
        ids = list(prompt_ids)
        need = len(ids) + int(max_new_tokens) + self.cap + self.k + 2
        if need > self.max_tokens:
            raise ValueError(f"request needs {need} positions > max_tokens {self.max_tokens}")
        b = self.n_active
        reuse = self.blocks.map_row(b, ids) if self.blocks is not None else 0
        if not reuse:
            self.tstate.release_row(b)
            self.cstate.release_row(b)
        self.tstate.ensure(b, need)
        self.cstate.ensure(b, need)
        last = prefill_rows(self.target, ids[reuse:], RowView(self.tstate, b), self.tap,
                            self.drafter, RowView(self.cstate, b))
        self.prefill_tokens += len(ids) - reuse
        first = int(last.float().argmax())
        if self.blocks is not None:
            self.blocks.store_row(b, ids)
        self.pending[b] = first
        self.trk[b] = _RowTracker(self.tokenizer, first, max_new_tokens, on_text, stop)
        self.meta[b] = meta
        self.t0[b] = time.time()
        self.n_active += 1

    def _retire(self, b: int):
        meta, res = self.meta[b], self.trk[b].result(time.time() - self.t0[b])
        last = self.n_active - 1
        self.tstate.release_row(b)
        self.cstate.release_row(b)
        if b != last:
            self.tstate.move_row(last, b)
            self.cstate.move_row(last, b)
            for st in (self.pending, self.trk, self.meta, self.t0):
                st[b] = st[last]
        self.trk[last], self.meta[last] = None, None
        self.pending[last], self.t0[last] = 0, 0.0
        self.n_active = last
        return meta, res

    def _sweep_finished(self) -> list:
        out = []
        b = 0
        while b < self.n_active:
            if self.trk[b].finished:
                out.append(self._retire(b))
            else:
                b += 1
        return out

    def step(self) -> list:
        """One speculative round over the active rows; returns [(meta, GenResult)] of the
        requests that finished (already retired)."""
        finished = self._sweep_finished()
        B = self.n_active
        if B == 0:
            return finished
        sess = self._session(B)
        if self.ctrl is not None:
            want = self.ctrl.cap_for(B) if B > 1 else self.ctrl.cap
            sess.set_cap(max(1, min(int(want), self.k)))
        sess.pending_host[:B] = torch.tensor(self.pending[:B], dtype=torch.int32)
        plans = sess.step(self.use_graph, feed_pending=True)
        if self.use_graph and sess.graph is None:
            sess.capture()
        for b in range(B):
            n = plans[b][0]
            committed = plans[b][2:3 + n]
            self.trk[b].commit(committed, accept_len=len(committed))
            self.pending[b] = self.trk[b].out_ids[-1]
            if self.ctrl is not None:
                self.ctrl.update(n, sess.cap)
        finished += self._sweep_finished()
        return finished

    def release(self) -> None:
        for s in self.sessions.values():
            s.release()
        self.sessions = {}
        if self.blocks is not None:
            self.blocks.reset()
        self.tstate.release()
        self.cstate.release()


def batch_spec_generate(target, tokenizer, drafter, prompts_ids: list[list[int]], *,
                        max_new_tokens=128, max_draft_tokens: int = 2,
                        batched_drafter: bool = True, on_texts=None, stops=None,
                        seed: int | None = None, prefix_reuse: bool = True,
                        max_tokens: int | None = None) -> list[GenResult]:
    """Static batched DSpark speculative decode (greedy) of B prompts (batch_engine.py:601-636):
    all rows admitted into SpecSlots of capacity B, stepped until every row is done."""
    B = len(prompts_ids)
    if B == 0:
        return []
    mnt = list(max_new_tokens) if isinstance(max_new_tokens, (list, tuple)) else [max_new_tokens] * B
    mt = max_tokens or (max(len(p) for p in prompts_ids) + max(mnt) + 2 * drafter.block_size + 64)
    slots = SpecSlots(target, tokenizer, drafter, capacity=B, max_draft_tokens=max_draft_tokens,
                      batched_drafter=batched_drafter, max_tokens=mt, prefix_reuse=prefix_reuse)
    try:
        ot = list(on_texts) if on_texts is not None else [None] * B
        sp = list(stops) if stops is not None else [None] * B
        for i, ids in enumerate(prompts_ids):
            slots.admit(ids, max_new_tokens=mnt[i], on_text=ot[i], stop=sp[i], meta=i)
        results: list[GenResult | None] = [None] * B
        while slots.n_active:
            for meta, res in slots.step():
                results[meta] = res
        return results
    finally:
        slots.release()


def batch_generate_baseline(target, tokenizer, prompts_ids: list[list[int]], *,
                            max_new_tokens=128, temperature: float = 0.0, top_p: float = 1.0,
                            top_k: int = 0, seed: int | None = None, use_graph: bool = True,
                            on_texts=None, stops=None) -> list[GenResult]:
    """Batched plain decode (batch_engine.py:322-362): per-row prefill, then one batched target
    forward per token until every row is done; greedy, or with temperature > 0 a draw from
    top-p/top-k(softmax(logits / T)) per row, row b on its own Philox stream seeded with
    seed + b (seed 0 when None)."""
    B = len(prompts_ids)
    mnt = list(max_new_tokens) if isinstance(max_new_tokens, (list, tuple)) else [max_new_tokens] * B
    base_seed = 0 if seed is None else int(seed)
    sess = GreedySession(target, B, max(len(p) for p in prompts_ids) + max(mnt) + 2,
                         Sampling(temperature, top_p, top_k), [base_seed + b for b in range(B)])
    try:
        t0 = time.time()
        first = []
        for b, ids in enumerate(prompts_ids):
            last = prefill_rows(target, list(ids), RowView(sess.tstate, b), ())
            first.append(_pick_first(target, last, sess.sampling, sess.rng[b:b + 1]))
        sess.buf.ids.copy_(torch.tensor(first, dtype=torch.int32))
        ot = list(on_texts) if on_texts is not None else [None] * B
        sp = list(stops) if stops is not None else [None] * B
        trk = [_RowTracker(tokenizer, first[b], mnt[b], ot[b], sp[b]) for b in range(B)]
        while not all(t.finished for t in trk):
            plans = sess.step(use_graph)
            if use_graph and sess.graph is None:
                sess.capture()
            for b in range(B):
                trk[b].commit([plans[b][2]])
        secs = time.time() - t0
        return [t.result(secs) for t in trk]
    finally:
        sess.release()


def serve_requests(target, tokenizer, drafter, requests, *, capacity: int = 4,
                   max_draft_tokens: int = 8, prefix_reuse: bool = True,
                   max_tokens: int | None = None):
    """Drive SpecSlots over a queue of (prompt_ids, max_new_tokens) requests, admitting one
    whenever a slot is free (the scheduling of BatchEngine._run_session, server.py:505-563).
    Returns (results in request order, stats)."""
    q = deque(enumerate(requests))
    mt = max_tokens or (max(len(p) + n for p, n in requests) + 2 * drafter.block_size + 64)
    slots = SpecSlots(target, tokenizer, drafter, capacity=capacity,
                      max_draft_tokens=max_draft_tokens, max_tokens=mt, prefix_reuse=prefix_reuse)
    results = [None] * len(requests)
    rounds = 0
    t0 = time.time()
    try:
        while q or slots.n_active:
            while q and slots.has_free_slot:
                i, (ids, n) = q.popleft()
                slots.admit(ids, max_new_tokens=n, meta=i)
            for meta, res in slots.step():
                results[meta] = res
            rounds += 1
        torch.cuda.synchronize()
        secs = time.time() - t0
        stats = {"rounds": rounds, "seconds": secs,
                 "tokens": sum(r.num_tokens for r in results),
                 "prefill_tokens": slots.prefill_tokens,
                 "prefix_hits": slots.blocks.hits if slots.blocks else 0,
                 "prefix_reused_tokens": slots.blocks.reused_tokens if slots.blocks else 0}
        return results, stats
    finally:
        slots.release()


__all__ = ["SpecSlots", "batch_spec_generate", "batch_generate_baseline", "serve_requests",
           "batchable"]
