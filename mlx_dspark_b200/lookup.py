"""Prompt-lookup (n-gram) drafts: the drafter-free proposals of src/mlx_dspark/lookup.py.

NGramIndex keeps, for every n-gram of the growing token sequence (min_n <= n <= max_n), the
end positions of its two most recent occurrences; propose() continues the latest occurrence
that is not the current suffix itself, longest n first (lookup.py:44-89). The verify of a
lookup draft runs on the device like a drafter round: exact argmax match when greedy, and at
temperature > 0 the one-hot proposal of the rejection sampler (dspark_accept_sample with
q_onehot), so the output stays an exact sample of the target.

lookup_generate is the pure prompt-lookup loop (lookup.py:92-202): a plain 1-token step when
nothing matches, a wider verify of [pending] + draft when something does.
"""
from __future__ import annotations

import time

import torch

from . import ops
from .generate import (GenResult, _decode, _finish_reason, _pick_first, eos_token_ids,
                       prefill_rows)
from .kvcache import CacheState
from .model import Sampling
from .streaming import TextStream


class NGramIndex:
    """Incremental n-gram -> (previous end, latest end) index over a token sequence."""

    def __init__(self, min_n: int = 3, max_n: int = 4, max_draft: int = 6):
        self.min_n = max(1, int(min_n))
        self.max_n = max(self.min_n, int(max_n))
        self.max_draft = max(1, int(max_draft))
        self.tokens: list[int] = []
        self._ends: dict[tuple, tuple[int | None, int]] = {}

    def extend(self, new_tokens) -> None:
        toks = self.tokens
        for t in new_tokens:
            toks.append(int(t))
            end = len(toks)
            for n in range(self.min_n, min(self.max_n, end) + 1):
                key = tuple(toks[end - n:end])
                old = self._ends.get(key)
                self._ends[key] = (None if old is None else old[1], end)

    def propose(self) -> list[int]:
        """Continuation of the latest earlier occurrence of the current suffix (longest n
        first); [] when nothing matches."""
        toks = self.tokens
        end = len(toks)
        for n in range(min(self.max_n, end), self.min_n - 1, -1):
            hit = self._ends.get(tuple(toks[end - n:end]))
            if hit is None:
                continue
            prev, latest = hit
            start = prev if latest == end else latest
            if start is None:
                continue
            draft = toks[start:start + self.max_draft]
            if draft:
                return draft
        return []


class BlockVerifier:
    """Eager verify of a variable-width block [pending] + draft for one row: the target forward
    (optionally with the hidden-state tap), penalties, and greedy or one-hot-proposal
    acceptance. Returns the plan row {n, n + 1, committed...}; commits the target KV length
    itself unless `commit` is False (the hybrid loop commits after the drafter context)."""

    def __init__(self, target, tstate: CacheState, tap=(), sampling: Sampling | None = None,
                 rng: torch.Tensor | None = None, counts: torch.Tensor | None = None,
                 penalties=(0.0, 0.0), pending: torch.Tensor | None = None):
        self.target, self.tstate, self.tap = target, tstate, list(tap)
        self.sampling = sampling if (sampling is not None and sampling.active) else None
        self.rng, self.counts, self.penalties = rng, counts, penalties
        dev = target.device
        self.pending = pending if pending is not None else torch.zeros(1, dtype=torch.int32, device=dev)
        self.ids_host = torch.zeros(64, dtype=torch.int32, pin_memory=True)
        self.lp = None  # a LogprobRows of the decode, when per-token logprobs are requested
        self._plans: dict[int, tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = {}
        self.done = torch.cuda.Event()

    def _plan(self, T):
        p = self._plans.get(T)
        if p is None:
            dev = self.target.device
            p = (torch.zeros(1, T + 2, dtype=torch.int32, device=dev),
                 torch.zeros(1, T + 2, dtype=torch.int32, pin_memory=True),
                 torch.zeros(T, dtype=torch.int32, device=dev))
            self._plans[T] = p
        return p

    def launch(self, pending: int, draft: list[int], commit: bool = True):
        t = self.target
        T = len(draft) + 1
        buf = t.buffers(1, T, len(self.tap))
        self.ids_host[:T] = torch.tensor([pending] + list(draft), dtype=torch.int32)
        buf.ids.copy_(self.ids_host[:T], non_blocking=True)
        t.forward(buf, self.tstate, self.tap)
        if self.lp is not None and self.counts is not None:
            self.lp.snapshot(buf.logits, T)
        if self.counts is not None:
            ops.apply_penalties(buf.logits, 1, T, self.counts, buf.ids, *self.penalties)
        plan, plan_host, argmax = self._plan(T)
        kv = self.tstate.seq_len if commit else None
        sm = self.sampling
        if sm is None:
            ops.accept_greedy(buf.logits, 1, T, buf.ids, argmax, kv, commit, self.pending, plan,
                              t.scratch)
        else:
            ops.accept_sample(buf.logits, 1, T, buf.ids, None, sm.temperature, sm.top_p, sm.top_k,
                              self.rng, kv, commit, self.pending, plan, t.scratch, q_onehot=True)
        if self.counts is not None:
            ops.penalty_counts_add(self.counts, plan, 1)
        if self.lp is not None:
            self.lp.launch(buf.logits, T, plan[:, 2:], T + 2, T)
        return buf, plan, plan_host

    def finish(self, plan, plan_host) -> list[int]:
        plan_host.copy_(plan, non_blocking=True)
        self.target.scratch.read_status_async()
        self.done.record()
        self.done.synchronize()
        self.target.scratch.raise_on_status()
        return plan_host[0].tolist()

    def run(self, pending: int, draft: list[int]) -> list[int]:
        _, plan, plan_host = self.launch(pending, draft, commit=True)
        return self.finish(plan, plan_host)


def lookup_generate(target_model, tokenizer, prompt: str = "", *,
                    prompt_ids: list[int] | None = None, cache=None, reuse_len: int = 0,
                    max_new_tokens: int = 128, max_draft_tokens: int = 6, ngram_min: int = 3,
                    ngram_max: int = 4, temperature: float = 0.0, top_p: float = 1.0,
                    top_k: int = 0, seed: int | None = None, apply_chat_template: bool = True,
                    stop: list[str] | None = None, on_text=None) -> GenResult:
    """Prompt-lookup speculative decoding, batch 1, no drafter model (lookup.py:92-202)."""
    eos_ids = eos_token_ids(tokenizer)
    st = TextStream(tokenizer, eos_ids, on_text, stop)
    if prompt_ids is None:
        prompt_ids = list(tokenizer.encode(prompt))
    ids = list(prompt_ids)
    t = target_model
    budget = len(ids) + max_new_tokens + max_draft_tokens + 2
    tstate = CacheState(t.new_pool(budget + 64, 1), 1, budget + 64, t.device)
    tstate.ensure(0, budget + 64)
    sampling = Sampling(temperature, top_p, top_k)
    rng = ops.rng_state(0 if seed is None else int(seed), t.device)
    ver = BlockVerifier(t, tstate, (), sampling, rng)
    index = NGramIndex(ngram_min, ngram_max, max(1, max_draft_tokens))
    index.extend(ids)
    try:
        t0 = time.time()
        last = prefill_rows(t, ids, tstate, ())
        pending = _pick_first(t, last, ver.sampling, rng)
        out = [pending]
        index.extend([pending])
        st.update(out)
        accept = []
        while len(out) < max_new_tokens and pending not in eos_ids and not st.stopped:
            draft = index.propose()
            plan = ver.run(pending, draft)
            n = plan[0]
            committed = plan[2:3 + n]
            accept.append(len(committed))
            appended = []
            for tok in committed:
                out.append(tok)
                appended.append(tok)
                if tok in eos_ids:
                    break
            index.extend(appended)
            pending = out[-1]
            st.update(out)
        st.flush()
        secs = time.time() - t0
        return GenResult(text=st.final_text(tokenizer, out, _decode),
                         token_ids=out, num_tokens=len(out), num_rounds=len(accept),
                         accept_lengths=accept, target_forwards=len(accept) + 1, seconds=secs,
                         finish_reason=_finish_reason(out, max_new_tokens, pending, eos_ids,
                                                      st.stopped))
    finally:
        tstate.release()


__all__ = ["NGramIndex", "BlockVerifier", "lookup_generate"]
