"""Decode loops on the device: speculative (DSpark or DFlash drafter; greedy or sampled) and
plain decoding.

Reference: src/mlx_dspark/generate.py — GenResult (:27-46), greedy_generate (:373-465),
dflash_generate (:468-601), _prefill_tapped (:632-656), _spec_sample_accept (:659-688),
speculative_generate (:691-978).

One speculative round is a fixed sequence of launches on one stream, with every varying
quantity (positions, lengths, pending token, draft ids) in device memory:

  draft  : block embed -> drafter layer(s) over [ctx; block] -> head on cap rows -> Markov argmax
           (writes verify_ids = [pending, d_1..d_cap])
  verify : target forward over verify_ids with the hidden-state tap
  accept : fused argmax + accepted prefix + bonus token -> plan, pending (greedy), or the
           rejection-sampling acceptance with residual draw (temperature > 0; the drafts and
           their q distributions come from the drafter's draw kernels, all randomness from a
           per-request Philox stream on the device whose offset the acceptance advances)
  context: fc + hidden_norm + k/v of the verified rows written at the drafter's context length
  commit : seq_len += n + 1 for the target KV and the drafter context (rollback = not counting)

so it is captured once into a CUDA graph and replayed; the host reads one small plan per
round (the reference also synchronises once per round, generate.py:917).
"""
from __future__ import annotations

import time
from dataclasses import dataclass

import torch

from . import ops
from .kvcache import CacheState, RowView
from .logprobs import LogprobRows
from .model import Sampling
from .streaming import StopStreaming, TextStream
from .target import PREFILL_CHUNK



@dataclass
class GenResult:
    text: str
    token_ids: list[int]
    num_tokens: int
    num_rounds: int
    accept_lengths: list[int]
    target_forwards: int
    seconds: float
    finish_reason: str = "stop"
    lookup_rounds: int = 0
    logprobs: list | None = None
    decode_seconds: float = 0.0  # time of the decode loop alone (after prefill)

    @property
    def mean_accept_len(self) -> float:
        return self.num_tokens / max(self.num_rounds, 1)

    @property
    def tokens_per_sec(self) -> float:
        return self.num_tokens / max(self.seconds, 1e-9)


def eos_token_ids(tokenizer) -> set[int]:
    """eos ids of a tokenizer (generate.py:111-132, reduced to the id attributes)."""
    ids: set[int] = set()
    if tokenizer is None:
        return ids
    e = getattr(tokenizer, "eos_token_ids", None)
    if isinstance(e, int):
        ids.add(e)
    elif e:
        ids.update(int(x) for x in e)
    e1 = getattr(tokenizer, "eos_token_id", None)
    if isinstance(e1, int):
        ids.add(e1)
    return ids


def _flat_ids(r) -> list[int] | None:
    """A flat id list out of what a chat template returns: ids, a batch of one, or an
    encoding with input_ids / ids."""
    if hasattr(r, "input_ids"):
        r = r.input_ids
    elif isinstance(r, dict) and "input_ids" in r:
        r = r["input_ids"]
    elif hasattr(r, "ids"):
        r = r.ids
    if hasattr(r, "tolist"):
        r = r.tolist()
    if isinstance(r, (list, tuple)):
        if r and isinstance(r[0], (list, tuple)):
            r = r[0]
        return [int(x) for x in r]
    return None


def encode_messages(tokenizer, messages: list[dict], add_generation_prompt: bool = True,
                    **template_kwargs) -> list[int]:
    """Ids of a chat transcript through the tokenizer's chat template (generate.py:71-96);
    template keyword arguments a tokenizer rejects are dropped and the call retried; without a
    template, the message contents joined by newlines."""
    if getattr(tokenizer, "chat_template", None):
        try:
            r = tokenizer.apply_chat_template(messages, add_generation_prompt=add_generation_prompt,
                                              **template_kwargs)
        except (TypeError, ValueError):
            r = tokenizer.apply_chat_template(messages, add_generation_prompt=add_generation_prompt)
        ids = _flat_ids(r)
        if ids is not None:
            return ids
    return list(tokenizer.encode("\n".join(str(m.get("content", "")) for m in messages)))


def encode_prompt(tokenizer, prompt: str, use_chat: bool = True) -> list[int]:
    """Ids of one user prompt, through the chat template when the tokenizer has one and
    use_chat is set (generate.py:99-108)."""
    if use_chat and getattr(tokenizer, "chat_template", None):
        return encode_messages(tokenizer, [{"role": "user", "content": prompt}])
    return list(tokenizer.encode(prompt))


def capture_graph(fn) -> torch.cuda.CUDAGraph:
    """Record fn()'s launches into a CUDA graph on a side stream. capture_begin/capture_end
    directly: the torch.cuda.graph context also empties the caching allocator on entry, which
    frees every cached block (seconds after a large session is released) and would land inside
    the first decode round. Thread-local capture mode: a serving process captures on its device
    thread while other threads (request intake, the NCCL watchdog) keep making CUDA calls of
    their own, which the global mode would count against the capture."""
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        g.capture_begin(capture_error_mode="thread_local")
        try:
            fn()
        finally:
            g.capture_end()
    torch.cuda.current_stream().wait_stream(s)
    return g


def _decode(tokenizer, ids):
    if tokenizer is None or not hasattr(tokenizer, "decode"):
        return ""
    return tokenizer.decode(ids)


def _finish_reason(out_ids, max_new_tokens, last_tok, eos_ids, stopped: bool = False) -> str:
    """'stop' when eos or a stop string (or the streaming callback) ended the decode, else
    'length' at the token cap (generate.py:365-370)."""
    if stopped or last_tok in eos_ids:
        return "stop"
    return "length" if len(out_ids) >= max_new_tokens else "stop"


# ----------------------------------------------------------------------------------------
def prefill_rows(target, ids: list[int], tstate, tap=(), drafter=None, cstate=None,
                 dbuf_key=None):
    """Chunked prefill of one row with the tap feeding the drafter context per chunk
    (_prefill_tapped, generate.py:632-656). `tstate`/`cstate` are one-row views whose
    lengths advance on the device. Returns the last chunk's logits row (bf16, device).
    Chunks of more than target.wide_min_tokens tokens (up to PREFILL_CHUNK) run through the
    large-M GEMM (Target.prefill_chunk, BlockDrafter.update_context_wide); the rest through
    the verify forward."""
    T = target.chunk_len(1)
    n = len(ids)
    ids_dev = torch.as_tensor(ids, dtype=torch.int32).to(target.device)
    last = None
    pos = 0
    while pos < n:
        if n - pos > target.wide_min_tokens:
            t = min(PREFILL_CHUNK, n - pos)
            buf = target.prefill_buffers(t, len(tap))
            buf.ids.copy_(ids_dev[pos:pos + t])
            target.prefill_chunk(buf, tstate, tap, logits="last" if pos + t == n else None)
            if drafter is not None:
                drafter.update_context_wide(buf.fused16, t, cstate)
                cstate.seq_len.add_(t)
            tstate.seq_len.add_(t)
            pos += t
            if pos == n:
                last = buf.logits[0].clone()
            continue
        t = min(T, n - pos)
        buf = target.buffers(1, t, len(tap))
        buf.ids.copy_(ids_dev[pos:pos + t])
        target.forward(buf, tstate, tap, with_logits=(pos + t == n))
        if drafter is not None:
            dbuf = drafter.buffers(1, drafter.block_size, t)
            drafter.update_context_dev(buf.fused16, 1, t, cstate, dbuf)
            cstate.seq_len.add_(t)
        tstate.seq_len.add_(t)
        pos += t
        if pos == n:
            last = buf.logits[t - 1].clone()
    return last


class SpecSession:
    """Static state and buffers of a B-row speculative decode with `cap` drafts per round.

    The verify width T = cap + 1 is baked into a round's buffers and captured graph. set_cap()
    switches to another cap (up to max_cap) over the same KV state, keeping one set of round
    buffers and one graph per cap used, so a cap controller can move the cap between rounds."""

    _ROUND = ("T", "vbuf", "dbuf", "draft", "argmax", "plan", "plan_host", "q", "graph",
              "_graph_versions")

    def __init__(self, target, drafter, B: int, cap: int, max_tokens: int, *,
                 override: dict | None = None, sampling: Sampling | None = None,
                 seeds=None, penalties: tuple[float, float] = (0.0, 0.0), states=None,
                 max_cap: int | None = None, logprobs: int | None = None):
        if getattr(drafter, "target", None) is not target:
            drafter.bind(target)   # a drafter from load_drafter / load_dflash comes unbound
        self.target, self.drafter = target, drafter
        self.B, self.cap = B, cap
        self.max_cap = max(cap, int(max_cap or cap))
        self.sampling = sampling if (sampling is not None and sampling.active) else None
        if self.sampling is not None and getattr(target, "world", 1) > 1:
            raise NotImplementedError("sampled decoding of a tensor-parallel target is not built")
        # OpenAI presence / frequency penalties on the target rows (_Penalizer,
        # generate.py:179-228): completion-token counts per row live on the device
        self.penalties = (float(penalties[0] or 0.0), float(penalties[1] or 0.0))
        self.counts = None
        if any(self.penalties):
            self.counts = torch.zeros(B, target.cfg.vocab_size, dtype=torch.int32,
                                      device=target.device)
        # per-token logprobs of the committed tokens (rows of a drafter round or of a lookup
        # round, up to 64 wide), read from a raw copy of the logits when penalties are on
        self.lp = None
        if logprobs is not None:
            if getattr(target, "world", 1) > 1:
                raise NotImplementedError("logprobs of a tensor-parallel target are not built")
            self.lp = LogprobRows(target.device, max(B * (self.max_cap + 1), 64), logprobs,
                                  target.cfg.vocab_size, raw=self.counts is not None)
        self.k = drafter.block_size
        self.tap = list(drafter.config.target_layer_ids)
        dev = target.device
        # pages for the whole request budget, plus one drafted block past the end
        cap_tokens = max_tokens + self.k + self.max_cap + 1 + 64
        self._owns_states = states is None
        if states is None:
            self.tstate = CacheState(target.new_pool(cap_tokens, B), B, cap_tokens, dev)
            self.cstate = CacheState(drafter.new_pool(cap_tokens, B), B, cap_tokens, dev)
            for b in range(B):
                self.tstate.ensure(b, cap_tokens)
                self.cstate.ensure(b, cap_tokens)
        else:
            # caller-owned rows (prefix reuse, the batch engine): the caller provides pages
            self.tstate, self.cstate = states
        self.pending = torch.zeros(B, dtype=torch.int32, device=dev)
        self.pending_host = torch.zeros(B, dtype=torch.int32, pin_memory=True)
        self.splits_t = target.attn_splits(B, self.tstate.max_pages)
        self.splits_c = target.attn_splits(B, self.cstate.max_pages)
        self.rng = ops.rng_state(list(seeds) if seeds is not None else [0] * B, dev)
        self._rounds: dict[int, dict] = {}
        for f, v in self._make_round(cap).items():
            setattr(self, f, v)
        self.override = None
        if override is not None:
            if self.sampling is not None:
                raise ValueError("the draft override is a greedy benchmark harness")
            o = override
            self.override = {
                "ref": o["ref"].to(dev, torch.int32).contiguous(),        # [B, ref_len]
                "agree": o["agree"].to(dev, torch.uint8).contiguous(),    # [B, rounds, cap]
                "round": torch.zeros(B, dtype=torch.int32, device=dev),
                "prompt_len": torch.as_tensor(o["prompt_len"], dtype=torch.int32).to(dev),
            }
        self.done = torch.cuda.Event()
        self._conf = None  # confidence buffers (device, pinned host), made by conf_step

    def _make_round(self, cap: int) -> dict:
        t, d, B, dev = self.target, self.drafter, self.B, self.target.device
        T = cap + 1
        return {"T": T, "vbuf": t.buffers(B, T, len(self.tap)),
                "dbuf": d.buffers(B, self.k, B * T),
                "draft": torch.zeros(B, cap, dtype=torch.int32, device=dev),
                "argmax": torch.zeros(B * T, dtype=torch.int32, device=dev),
                "plan": torch.zeros(B, T + 2, dtype=torch.int32, device=dev),
                "plan_host": torch.zeros(B, T + 2, dtype=torch.int32, pin_memory=True),
                "q": (torch.zeros(B * cap, t.cfg.vocab_size, dtype=torch.float32, device=dev)
                      if self.sampling is not None else None),
                "graph": None, "_graph_versions": None}

    def set_cap(self, cap: int) -> None:
        """Draft and verify `cap` tokens from the next round on (1 <= cap <= max_cap)."""
        cap = int(cap)
        if cap == self.cap:
            return
        if not 1 <= cap <= self.max_cap:
            raise ValueError(f"cap {cap} outside [1, {self.max_cap}]")
        if self.override is not None:
            raise ValueError("the draft override fixes the cap")
        self._rounds[self.cap] = {f: getattr(self, f) for f in self._ROUND}
        r = self._rounds.pop(cap, None) or self._make_round(cap)
        for f, v in r.items():
            setattr(self, f, v)
        self.cap = cap

    def release(self):
        self.graph = None
        self._rounds.clear()
        if self._owns_states:
            self.tstate.release()
            self.cstate.release()

    def launch_draft(self) -> None:
        """Draft cap tokens per row into self.draft and the verify ids of this cap's round."""
        d, t = self.drafter, self.target
        B, cap = self.B, self.cap
        d.draft_dev(self.pending, B, cap, self.cstate, self.dbuf, self.draft, self.vbuf.ids,
                    self.splits_c, sampling=self.sampling, rng=self.rng, q_probs=self.q)
        if self.override is not None:
            o = self.override
            ops.draft_override(B, cap, t.cfg.vocab_size, o["ref"], o["agree"], o["round"],
                               self.tstate.seq_len, o["prompt_len"], self.vbuf.ids)

    def launch_verify(self, r: dict | None = None) -> None:
        """Verify, accept and commit the block held in round r's verify ids (default: this
        cap's round); the draft distributions and context buffers are this cap's."""
        r = self._current() if r is None else r
        d, t, sc = self.drafter, self.target, self.target.scratch
        B, T = self.B, r["T"]
        vbuf, plan, sm = r["vbuf"], r["plan"], self.sampling
        t.forward(vbuf, self.tstate, self.tap, splits=self.splits_t)
        if self.lp is not None and self.counts is not None:
            self.lp.snapshot(vbuf.logits, B * T)
        if self.counts is not None:
            ops.apply_penalties(vbuf.logits, B, T, self.counts, vbuf.ids, *self.penalties)
        if sm is None:
            t.greedy_accept(vbuf.logits, B, T, vbuf.ids, r["argmax"], None, False, self.pending,
                            plan)
        else:
            ops.accept_sample(vbuf.logits, B, T, vbuf.ids, self.q, sm.temperature, sm.top_p,
                              sm.top_k, self.rng, None, False, self.pending, plan, sc)
        if self.counts is not None:
            ops.penalty_counts_add(self.counts, plan, B)
        if self.lp is not None:
            self.lp.launch(vbuf.logits, B * T, plan[:, 2:], T + 2, T)
        d.update_context_dev(vbuf.fused16, B, T, self.cstate, self.dbuf)
        ops.commit_lengths(plan, B, self.tstate.seq_len, self.cstate.seq_len)
        r["plan_host"].copy_(plan, non_blocking=True)
        t.scratch.read_status_async()

    def launch_round(self) -> None:
        self.launch_draft()
        self.launch_verify()

    def _current(self) -> dict:
        return {f: getattr(self, f) for f in self._ROUND}

    def _round(self, cap: int) -> dict:
        """Round buffers for `cap` drafts without switching to them (conf_step's shorter
        verify); made on first use and kept with the other caps' rounds."""
        if cap == self.cap:
            return self._current()
        r = self._rounds.get(cap)
        if r is None:
            r = self._rounds[cap] = self._make_round(cap)
        return r

    def conf_step(self, threshold: float) -> tuple[list[int], int]:
        """A drafter round with confidence truncation (generate.py:855-887): draft cap tokens
        and their survival probabilities, keep the longest prefix whose running product stays
        >= threshold (at least one token), then verify, accept and commit that block. Runs
        eagerly with one host sync between the phases, like the reference's two-phase path.
        The round's input token comes from pending_host. Returns (plan row, drafted count)."""
        if self.B != 1:
            raise NotImplementedError("confidence truncation is batch 1 (as the reference)")
        if self.drafter.confidence_head is None:
            raise ValueError("the drafter has no confidence head")
        if self._conf is None:
            dev = self.target.device
            self._conf = (torch.zeros(self.max_cap, dtype=torch.float32, device=dev),
                          torch.zeros(self.max_cap, dtype=torch.float32, pin_memory=True))
        conf_dev, conf_host = self._conf
        cap = self.cap
        self.pending.copy_(self.pending_host, non_blocking=True)
        self.launch_draft()
        self.drafter.confidence_dev(self.dbuf, self.pending, self.draft, cap, conf_dev)
        conf_host[:cap].copy_(conf_dev[:cap], non_blocking=True)
        self.target.scratch.read_status_async()
        self.done.record()
        self.done.synchronize()
        self.target.scratch.raise_on_status()
        surv, keep = 1.0, 0
        for i, c in enumerate(conf_host[:cap].tolist()):
            surv *= c
            if surv < threshold:
                break
            keep = i + 1
        keep = max(keep, 1)   # always propose at least one token
        r = self._round(keep)
        if keep != cap:
            r["vbuf"].ids[:keep + 1].copy_(self.vbuf.ids[:keep + 1])
        self.launch_verify(r)
        self.done.record()
        self.done.synchronize()
        self.target.scratch.raise_on_status()
        return r["plan_host"][0].tolist(), keep

    def _versions(self):
        return (self.tstate.pool.version, self.cstate.pool.version,
                self.target.scratch.version, self.tstate.max_pages, self.cstate.max_pages)

    def capture(self) -> None:
        if not self.target.capturable:
            return
        self.graph = capture_graph(self.launch_round)
        self._graph_versions = self._versions()

    def lookup_round(self, pending: int, draft: list[int]) -> list[int]:
        """A hybrid round that verifies an n-gram lookup draft instead of drafting
        (generate.py:807-837): verify [pending] + draft with the tap, accept (greedy, or the
        one-hot proposal when sampling), write the drafter context from the verified rows,
        then commit both lengths. Runs eagerly: its width follows the match length."""
        from .lookup import BlockVerifier  # lookup imports this module
        if self.B != 1:
            raise NotImplementedError("hybrid lookup rounds are batch 1 (as the reference)")
        if getattr(self, "_verifier", None) is None:
            self._verifier = BlockVerifier(self.target, self.tstate, self.tap, self.sampling,
                                           self.rng, self.counts, self.penalties, self.pending)
            self._verifier.lp = self.lp
        T = len(draft) + 1
        buf, plan, plan_host = self._verifier.launch(pending, draft, commit=False)
        self.drafter.update_context_dev(buf.fused16, 1, T, self.cstate,
                                        self.drafter.buffers(1, self.k, T))
        ops.commit_lengths(plan, 1, self.tstate.seq_len, self.cstate.seq_len)
        return self._verifier.finish(plan, plan_host)

    def step(self, use_graph: bool = True, feed_pending: bool = False):
        """Run one round; returns the plan rows [B, T+2] as python lists. With feed_pending
        the round's input token comes from pending_host (pinned) by one H2D copy, as in a
        host-driven loop where the host owns the committed sequence."""
        if feed_pending:
            self.pending.copy_(self.pending_host, non_blocking=True)
        if self.graph is not None and self._graph_versions != self._versions():
            self.graph = None  # a pool, block table or workspace moved: capture again
        if use_graph and self.graph is not None and self.target.capturable:
            self.graph.replay()
        else:
            self.launch_round()
        self.done.record()
        self.done.synchronize()
        self.target.scratch.raise_on_status()
        return self.plan_host.tolist()


def _pick_first(target, last_row: torch.Tensor, sampling: Sampling | None, rng: torch.Tensor) -> int:
    """First committed token from the prefill's last logits (_pick, generate.py:144-146):
    argmax, or a draw with Philox {offset 0, row 0, stream 2}."""
    if sampling is None:
        return target.argmax_row(last_row)
    tok = torch.zeros(1, dtype=torch.int32, device=target.device)
    ops.sample_rows(last_row.view(1, -1), 1, 1, sampling.temperature, sampling.top_p,
                    sampling.top_k, rng[:1], tok, stream_id=2)
    return int(tok.item())


def _caller_states(drafter, cache, ctx_caches, reuse_len: int, tokens: int):
    """The CacheStates of caller-provided caches, widened and paged for `tokens` positions and
    trimmed to the reused prefix (the reference trims its caches to reuse_len the same way)."""
    if ctx_caches is None:
        ctx_caches = drafter.make_ctx_cache(tokens)
        if reuse_len:
            raise ValueError("reuse_len needs the drafter context caches of the reused prefix")
    tstate, cstate = cache.state, ctx_caches.state
    for st in (tstate, cstate):
        st.grow(tokens)
        st.ensure(0, tokens)
        st.set_len(0, reuse_len)
    return tstate, cstate, ctx_caches


def _spec_loop(target, tokenizer, drafter, ids, cap, max_new_tokens, sampling, seed, use_graph,
               draft_override, verbose, penalties=(0.0, 0.0), lookup_max_draft=0, cache=None,
               ctx_caches=None, reuse_len: int = 0, cap_controller=None,
               logprobs: int | None = None, confidence_threshold: float = 0.0, stop=None,
               on_text=None) -> GenResult:
    """The decode loop of speculative_generate / dflash_generate. `cap` is the ceiling; with a
    cap_controller each drafter round uses min(controller.cap, cap) and feeds the outcome back
    (generate.py:846-847,924-925); lookup rounds neither use nor update it. Text streams to
    on_text and stop strings end the decode at a round boundary (TextStream)."""
    eos_ids = eos_token_ids(tokenizer)
    st = TextStream(tokenizer, eos_ids, on_text, stop)
    budget = len(ids) + max_new_tokens + cap + 1
    sampling = sampling if (sampling is not None and sampling.active) else None
    states = None
    if cache is not None:
        tokens = budget + drafter.block_size + cap + 1 + 64
        tstate, cstate, ctx_caches = _caller_states(drafter, cache, ctx_caches, int(reuse_len),
                                                    tokens)
        states = (tstate, cstate)
    else:
        reuse_len = 0
    ctrl = cap_controller
    # confidence truncation needs the drafter's confidence head; without one the threshold is
    # ignored, as in the reference (generate.py:808)
    use_conf = confidence_threshold > 0.0 and getattr(drafter, "confidence_head", None) is not None
    first_cap = cap if ctrl is None else max(1, min(int(ctrl.cap), cap))
    sess = SpecSession(target, drafter, 1, first_cap, budget, override=draft_override,
                       sampling=sampling, seeds=[0 if seed is None else int(seed)],
                       penalties=penalties, states=states, max_cap=cap, logprobs=logprobs)
    try:
        t0 = time.time()
        # prefill only the part of the prompt past the reused prefix (generate.py:640-650)
        last = prefill_rows(target, ids[reuse_len:], sess.tstate, sess.tap, drafter, sess.cstate)
        pending = _pick_first(target, last, sampling, sess.rng)
        sess.pending.fill_(pending)
        if sess.counts is not None:
            sess.counts[0, pending] += 1          # pen.add([pending]) (generate.py:784)
        lp_list = None
        if sess.lp is not None:
            # the first token's entry comes from the prefill's last row (generate.py:786-787)
            sess.lp.launch(last.view(1, -1), 1, sess.pending, 1, 1, use_snapshot=False)
            torch.cuda.current_stream().synchronize()
            lp_list = sess.lp.entries([pending])
        index = None
        if lookup_max_draft:
            from .lookup import NGramIndex  # lookup imports this module
            # hybrid mode: a stricter 4-gram minimum than pure lookup (generate.py:789-798)
            index = NGramIndex(min_n=4, max_n=5, max_draft=lookup_max_draft)
            index.extend(ids + [pending])
        torch.cuda.synchronize()
        t1 = time.time()
        out = [pending]
        st.update(out)
        accept = []
        rounds = lookup_rounds = 0
        while len(out) < max_new_tokens and pending not in eos_ids and not st.stopped:
            lk = index.propose() if index is not None else []
            if lk:
                lookup_rounds += 1
                plan = sess.lookup_round(pending, lk)
            else:
                if ctrl is not None:
                    sess.set_cap(max(1, min(int(ctrl.cap), cap)))
                sess.pending_host[0] = pending
                if use_conf:
                    plan, drafted = sess.conf_step(confidence_threshold)
                else:
                    plan = sess.step(use_graph, feed_pending=True)[0]
                    drafted = sess.cap
                    if use_graph and sess.graph is None:
                        sess.capture()
                if ctrl is not None:
                    ctrl.update(plan[0], drafted)
            n = plan[0]
            committed = plan[2:3 + n]
            accept.append(len(committed))
            appended = []
            for tok in committed:
                out.append(tok)
                appended.append(tok)
                if tok in eos_ids:
                    break
            if lp_list is not None:
                lp_list.extend(sess.lp.entries(appended))
            if index is not None:
                index.extend(appended)
            pending = out[-1]
            st.update(out)
            rounds += 1
            if verbose:
                src = "lookup" if lk else "drafter"
                print(f"  round {rounds:3d}: {src} drafted {len(lk) if lk else drafted}, accepted {n}, "
                      f"committed {len(committed)}")
        st.flush()
        t2 = time.time()
        text = st.final_text(tokenizer, out, _decode)
        return GenResult(text=text, token_ids=out, num_tokens=len(out), num_rounds=len(accept),
                         accept_lengths=accept, target_forwards=len(accept) + 1,
                         seconds=t2 - t0, decode_seconds=t2 - t1, lookup_rounds=lookup_rounds,
                         finish_reason=_finish_reason(out, max_new_tokens, pending, eos_ids,
                                                      st.stopped),
                         logprobs=lp_list)
    finally:
        sess.release()
        if cache is not None:
            # the caller's caches now hold prompt + every committed token but the pending one
            n = sess.tstate.sync_from_device()[0]
            cache.set_offset(n)
            sess.cstate.sync_from_device()


def speculative_generate(target, tokenizer, drafter, prompt: str = "", *,
                         prompt_ids: list[int] | None = None, cache=None, ctx_caches=None,
                         reuse_len: int = 0, max_new_tokens: int = 128,
                         confidence_threshold: float = 0.0, max_draft_tokens: int | None = 2,
                         cap_controller=None, lookup_drafts: bool = True,
                         lookup_max_draft: int = 6, temperature: float = 0.0, top_p: float = 1.0,
                         top_k: int = 0, presence_penalty: float = 0.0,
                         frequency_penalty: float = 0.0, logprobs: int | None = None,
                         seed: int | None = None, apply_chat_template: bool = True,
                         stop: list[str] | None = None, on_text=None, verbose: bool = False,
                         use_graph: bool = True, draft_override: dict | None = None) -> GenResult:
    """Speculative decoding with the DSpark drafter, batch 1 (generate.py:691-978).
    temperature 0: the output is the target's greedy decoding. temperature > 0: drafts are drawn
    from the drafter's truncated distributions and accepted by rejection sampling, so the output
    is a sample of top-p/top-k(softmax(target / T)) (lossless); `seed` seeds the Philox stream.
    confidence_threshold > 0 with a drafter that has a confidence head truncates each drafted
    block where the running product of its survival probabilities falls below the threshold
    (the output is unchanged; rounds get shorter). logprobs (an int, 0 = the committed token
    only) returns per-token entries of the raw target distribution in GenResult.logprobs."""
    k = drafter.config.block_size
    cap = k if max_draft_tokens is None else max(1, min(int(max_draft_tokens), k))
    if prompt_ids is None:
        prompt_ids = encode_prompt(tokenizer, prompt, apply_chat_template)
    return _spec_loop(target, tokenizer, drafter, list(prompt_ids), cap, max_new_tokens,
                      Sampling(temperature, top_p, top_k), seed, use_graph, draft_override,
                      verbose, (presence_penalty, frequency_penalty),
                      max(1, int(lookup_max_draft)) if lookup_drafts else 0, cache, ctx_caches,
                      reuse_len, cap_controller, logprobs, float(confidence_threshold), stop,
                      on_text)


def dflash_generate(target_model, tokenizer, drafter, prompt: str = "", *,
                    prompt_ids: list[int] | None = None, max_new_tokens: int = 128,
                    max_draft_tokens: int | None = None, cap_controller=None,
                    temperature: float = 0.0, top_p: float = 1.0, top_k: int = 0,
                    apply_chat_template: bool = True, seed: int | None = None,
                    stop: list[str] | None = None, on_text=None, use_graph: bool = True,
                    verbose: bool = False) -> GenResult:
    """Speculative decoding with the DFlash block-diffusion drafter (generate.py:468-601). The
    backbone drafts the full block; `max_draft_tokens` bounds how many drafted tokens are
    verified (None = block - 1, DFlash's native operating point)."""
    kdraft = drafter.config.block_size - 1
    cap = kdraft if max_draft_tokens is None else max(1, min(int(max_draft_tokens), kdraft))
    if prompt_ids is None:
        prompt_ids = encode_prompt(tokenizer, prompt, apply_chat_template)
    return _spec_loop(target_model, tokenizer, drafter, list(prompt_ids), cap, max_new_tokens,
                      Sampling(temperature, top_p, top_k), seed, use_graph, None, verbose,
                      cap_controller=cap_controller, stop=stop, on_text=on_text)


class GreedySession:
    """Plain decode of B rows, one token per step (generate.py:373-465): argmax, or with
    temperature > 0 a draw from top-p/top-k(softmax(logits / T)) whose Philox offset the
    draw kernel advances on the device (so the step stays one CUDA graph)."""

    def __init__(self, target, B: int, max_tokens: int, sampling: Sampling | None = None,
                 seeds=None, penalties: tuple[float, float] = (0.0, 0.0),
                 logprobs: int | None = None):
        self.target, self.B = target, B
        self.penalties = (float(penalties[0] or 0.0), float(penalties[1] or 0.0))
        self.counts = None
        if any(self.penalties):
            self.counts = torch.zeros(B, target.cfg.vocab_size, dtype=torch.int32,
                                      device=target.device)
        self.sampling = sampling if (sampling is not None and sampling.active) else None
        if self.sampling is not None and getattr(target, "world", 1) > 1:
            raise NotImplementedError("sampled decoding of a tensor-parallel target is not built")
        self.lp = None
        if logprobs is not None:
            if getattr(target, "world", 1) > 1:
                raise NotImplementedError("logprobs of a tensor-parallel target are not built")
            self.lp = LogprobRows(target.device, B, logprobs, target.cfg.vocab_size,
                                  raw=self.counts is not None)
        self.rng = ops.rng_state(list(seeds) if seeds is not None else [0] * B, target.device)
        dev = target.device
        cap_tokens = max_tokens + 64
        self.tstate = CacheState(target.new_pool(cap_tokens, B), B, cap_tokens, dev)
        for b in range(B):
            self.tstate.ensure(b, cap_tokens)
        self.buf = target.buffers(B, 1, 0)
        self.argmax = torch.zeros(B, dtype=torch.int32, device=dev)
        self.plan = torch.zeros(B, 3, dtype=torch.int32, device=dev)
        self.plan_host = torch.zeros(B, 3, dtype=torch.int32, pin_memory=True)
        self.splits = target.attn_splits(B, self.tstate.max_pages)
        self.graph = None
        self.done = torch.cuda.Event()

    def release(self):
        self.graph = None
        self.tstate.release()

    def launch_step(self):
        t = self.target
        t.forward(self.buf, self.tstate, (), splits=self.splits)
        # T = 1: n = 0, bonus = argmax (or a draw); the next input id is written in place
        sm = self.sampling
        if self.lp is not None and self.counts is not None:
            self.lp.snapshot(self.buf.logits, self.B)
        if self.counts is not None:
            ops.apply_penalties(self.buf.logits, self.B, 1, self.counts, None, *self.penalties)
        if sm is None:
            t.greedy_accept(self.buf.logits, self.B, 1, self.buf.ids, self.argmax,
                            self.tstate.seq_len, True, self.buf.ids, self.plan)
        else:
            ops.accept_sample(self.buf.logits, self.B, 1, self.buf.ids, None, sm.temperature,
                              sm.top_p, sm.top_k, self.rng, self.tstate.seq_len, True,
                              self.buf.ids, self.plan, t.scratch)
        if self.counts is not None:
            ops.penalty_counts_add(self.counts, self.plan, self.B)
        if self.lp is not None:
            self.lp.launch(self.buf.logits, self.B, self.plan[:, 2:], 3, 1)
        self.plan_host.copy_(self.plan, non_blocking=True)
        t.scratch.read_status_async()

    def capture(self):
        if not self.target.capturable:
            return
        self.graph = capture_graph(self.launch_step)

    def step(self, use_graph=True):
        if use_graph and self.graph is not None and self.target.capturable:
            self.graph.replay()
        else:
            self.launch_step()
        self.done.record()
        self.done.synchronize()
        self.target.scratch.raise_on_status()
        return self.plan_host.tolist()


def greedy_generate(target, tokenizer, prompt: str = "", *, prompt_ids: list[int] | None = None,
                    cache=None, reuse_len: int = 0, max_new_tokens: int = 128,
                    temperature: float = 0.0, top_p: float = 1.0, top_k: int = 0,
                    presence_penalty: float = 0.0, frequency_penalty: float = 0.0,
                    logprobs: int | None = None, seed: int | None = None,
                    apply_chat_template: bool = True, stop=None, on_text=None,
                    use_graph: bool = True) -> GenResult:
    """Plain decoding of the target (the baseline the speedup is measured against): greedy, or
    sampled with temperature / top-p / top-k from a Philox stream seeded by `seed`."""
    eos_ids = eos_token_ids(tokenizer)
    st = TextStream(tokenizer, eos_ids, on_text, stop)
    if prompt_ids is None:
        prompt_ids = encode_prompt(tokenizer, prompt, apply_chat_template)
    ids = list(prompt_ids)
    sampling = Sampling(temperature, top_p, top_k)
    sess = GreedySession(target, 1, len(ids) + max_new_tokens + 1, sampling,
                         [0 if seed is None else int(seed)],
                         (presence_penalty, frequency_penalty), logprobs)
    try:
        t0 = time.time()
        last = prefill_rows(target, ids, sess.tstate, ())
        nxt = _pick_first(target, last, sess.sampling, sess.rng)
        if sess.counts is not None:
            sess.counts[0, nxt] += 1             # pen.add([nxt]) (generate.py:427)
        sess.buf.ids.fill_(nxt)
        lp_list = None
        if sess.lp is not None:
            # every entry, the first included, is the raw row the token was picked from
            # (generate.py:417-429)
            sess.lp.launch(last.view(1, -1), 1, sess.buf.ids, 1, 1, use_snapshot=False)
        torch.cuda.synchronize()
        if sess.lp is not None:
            lp_list = sess.lp.entries([nxt])
        t1 = time.time()
        out = [nxt]
        st.update(out)
        while len(out) < max_new_tokens and nxt not in eos_ids and not st.stopped:
            plan = sess.step(use_graph)[0]
            if use_graph and sess.graph is None:
                sess.capture()
            nxt = plan[2]
            out.append(nxt)
            if lp_list is not None:
                lp_list.extend(sess.lp.entries([nxt]))
            st.update(out)
        st.flush()
        t2 = time.time()
        text = st.final_text(tokenizer, out, _decode)
        return GenResult(text=text, token_ids=out, num_tokens=len(out), num_rounds=len(out),
                         accept_lengths=[1] * len(out), target_forwards=len(out),
                         seconds=t2 - t0, decode_seconds=t2 - t1,
                         finish_reason=_finish_reason(out, max_new_tokens, nxt, eos_ids,
                                                      st.stopped),
                         logprobs=lp_list)
    finally:
        sess.release()


__all__ = ["GenResult", "SpecSession", "GreedySession", "speculative_generate",
           "dflash_generate", "greedy_generate", "prefill_rows", "eos_token_ids", "RowView",
           "StopStreaming", "encode_messages", "encode_prompt"]
