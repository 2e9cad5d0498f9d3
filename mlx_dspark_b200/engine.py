"""The serving layer between requests and the decode loops: Engine and BatchEngine.

Drop-in for the scheduling half of src/mlx_dspark/server.py (Engine 75-365, BatchEngine
381-608, maybe_batch_engine 611-622); the HTTP handler, CLI and request parsing are out of scope.

Engine runs every request on one worker thread (one CUDA stream, one set of captured graphs),
reuses a stored conversation prefix through PrefixCache (acquire before, store after; reset on
any error), dispatches by mode (dspark / dflash / lookup / baseline) and keeps the cumulative
stats that /metrics and the `x_mlx_dspark` block report.

BatchEngine puts a scheduler loop on that same thread. Requests queue up, the loop gathers
them for a short window (20 ms), groups them by sampling parameters, and:
  - penalties or logprobs: serial (the batched round applies neither);
  - a lone request, or a dspark group with temperature > 0: serial;
  - a greedy dspark group: one continuous SpecSlots session - a finished row is delivered at
    once and its slot admits the next queued or newly arriving greedy request; an arrival that
    cannot join (sampled, penalised, too long) stops admissions and runs after the session;
  - a greedy baseline group: the static batched baseline.
Stop strings and streaming callbacks are not built: requests that use them are refused with
NotImplementedError instead of being run without them.
"""
from __future__ import annotations

import atexit
import queue as _queue
import threading
import time
from concurrent.futures import ThreadPoolExecutor

from .batch_engine import SpecSlots, batch_generate_baseline, batchable
from .generate import GenResult, dflash_generate, greedy_generate, speculative_generate
from .lookup import lookup_generate
from .prefix_cache import PrefixCache, target_cache_reusable

MODES = ("dspark", "dflash", "lookup", "baseline")


def _refuse_unbuilt(stop, on_text) -> None:
    if stop or on_text is not None:
        raise NotImplementedError("stop strings and streaming callbacks are not built")


class Engine:
    """Loaded target/drafter -> GenResult, one request at a time (server.py:75-365)."""

    def __init__(self, target, tokenizer, drafter, *, mode: str, model_id: str = "",
                 target_repo: str = "", drafter_repo: str | None = None,
                 max_draft_tokens: int | None = None, prefix_cache: bool = True,
                 prefix_cache_slots: int = 2, cache_tokens: int = 4096, cap_controller=None,
                 lookup_drafts: bool = True, default_max_tokens: int = 2048,
                 max_tokens_cap: int = 32768, executor: ThreadPoolExecutor | None = None):
        if mode not in MODES:
            raise ValueError(f"mode must be one of {MODES}, not {mode!r}")
        if mode in ("dspark", "dflash") and drafter is None:
            raise ValueError(f"mode {mode!r} needs a drafter")
        self.target, self.tokenizer, self.drafter = target, tokenizer, drafter
        self.mode = mode
        self.model_id = model_id or str(target_repo).rstrip("/").split("/")[-1]
        self.target_repo, self.drafter_repo = target_repo, drafter_repo
        self.max_draft_tokens = max_draft_tokens
        self.cap_controller = cap_controller      # persists across requests (--max-draft auto)
        self.lookup_drafts = lookup_drafts
        self.cache_tokens = int(cache_tokens)     # initial size of a cache (they grow on demand)
        self.prefix_cache_slots = max(1, int(prefix_cache_slots))
        self.default_max_tokens = default_max_tokens
        self.max_tokens_cap = max_tokens_cap
        self._executor = executor or ThreadPoolExecutor(max_workers=1,
                                                        thread_name_prefix="dspark-gen")
        self.prefix = self._build_prefix_cache(prefix_cache)
        self.created = int(time.time())
        self.stats = {"requests": 0, "prompt_tokens": 0, "completion_tokens": 0,
                      "generation_seconds": 0.0, "sum_accept_len": 0.0}

    def _build_prefix_cache(self, enabled: bool):
        """Prefix reuse where a cache can roll back exactly: dspark, lookup and baseline
        (server.py:143-160); DFlash's drafter cache cannot, so it runs without."""
        if not enabled or self.mode == "dflash":
            return None
        probe = self.target.make_cache(64)
        try:
            if not target_cache_reusable(probe):
                return None
        finally:
            probe.release()
        n = self.cache_tokens
        make_ctx = (lambda: self.drafter.make_ctx_cache(n)) if self.mode == "dspark" else None
        return PrefixCache(lambda: self.target.make_cache(n), make_ctx,
                           slots=self.prefix_cache_slots)

    # ---------------------------------------------------------------- generation
    def generate(self, prompt_ids, *, max_tokens: int, temperature: float, top_p: float = 1.0,
                 top_k: int = 0, presence_penalty: float = 0.0, frequency_penalty: float = 0.0,
                 logprobs: int | None = None, stop=None, seed: int | None = None,
                 on_text=None) -> GenResult:
        return self._executor.submit(
            self._generate_impl, list(prompt_ids), max_tokens, temperature, top_p, top_k, stop,
            seed, on_text, presence_penalty, frequency_penalty, logprobs).result()

    def _generate_impl(self, prompt_ids, max_tokens, temperature, top_p, top_k, stop, seed,
                       on_text, presence_penalty=0.0, frequency_penalty=0.0,
                       logprobs=None) -> GenResult:
        _refuse_unbuilt(stop, on_text)
        cache = ctx = None
        reuse = 0
        if self.prefix is not None:
            cache, ctx, reuse = self.prefix.acquire(prompt_ids)
        try:
            if self.mode == "dspark":
                res = speculative_generate(
                    self.target, self.tokenizer, self.drafter, prompt_ids=prompt_ids,
                    cache=cache, ctx_caches=ctx, reuse_len=reuse, max_new_tokens=max_tokens,
                    max_draft_tokens=self.max_draft_tokens, cap_controller=self.cap_controller,
                    lookup_drafts=self.lookup_drafts, temperature=temperature, top_p=top_p,
                    top_k=top_k, presence_penalty=presence_penalty,
                    frequency_penalty=frequency_penalty, logprobs=logprobs, seed=seed)
            elif self.mode == "dflash":
                res = dflash_generate(
                    self.target, self.tokenizer, self.drafter, prompt_ids=prompt_ids,
                    max_new_tokens=max_tokens, max_draft_tokens=self.max_draft_tokens,
                    cap_controller=self.cap_controller, temperature=temperature, top_p=top_p,
                    top_k=top_k, seed=seed)
            elif self.mode == "lookup":
                res = lookup_generate(
                    self.target, self.tokenizer, prompt_ids=prompt_ids, cache=cache,
                    reuse_len=reuse, max_new_tokens=max_tokens,
                    max_draft_tokens=self.max_draft_tokens or 6, temperature=temperature,
                    top_p=top_p, top_k=top_k, seed=seed)
            else:
                res = greedy_generate(
                    self.target, self.tokenizer, prompt_ids=prompt_ids, cache=cache,
                    reuse_len=reuse, max_new_tokens=max_tokens, temperature=temperature,
                    top_p=top_p, top_k=top_k, presence_penalty=presence_penalty,
                    frequency_penalty=frequency_penalty, logprobs=logprobs, seed=seed)
        except BaseException:
            # never keep a cache whose contents no longer match its recorded tokens
            if self.prefix is not None:
                self.prefix.reset()
                for c in (cache, ctx):
                    if c is not None:
                        c.release()
            raise
        if self.prefix is not None and cache is not None:
            self.prefix.store(cache, ctx, prompt_ids, res.token_ids)
        self._count(len(prompt_ids), res, res.seconds)
        return res

    def _count(self, prompt_tokens: int, res: GenResult, seconds: float | None) -> None:
        s = self.stats
        s["requests"] += 1
        s["prompt_tokens"] += prompt_tokens
        s["completion_tokens"] += res.num_tokens
        if seconds is not None:
            s["generation_seconds"] += seconds
        s["sum_accept_len"] += res.mean_accept_len * res.num_tokens

    # ---------------------------------------------------------------- reporting
    def spec_info(self, res: GenResult) -> dict:
        """The non-standard `x_mlx_dspark` block of a response (server.py:331-343)."""
        info = {"mode": self.mode, "accept_len": round(res.mean_accept_len, 3),
                "tokens_per_sec": round(res.tokens_per_sec, 1),
                "target_forwards": res.target_forwards}
        if self.cap_controller is not None:
            info["cap"] = self.cap_controller.cap
        if res.lookup_rounds:
            info["lookup_rounds"] = res.lookup_rounds
        return info

    def metrics(self) -> dict:
        s = self.stats
        ct = s["completion_tokens"]
        return {"model": self.model_id, "mode": self.mode, "requests": s["requests"],
                "prompt_tokens": s["prompt_tokens"], "completion_tokens": ct,
                "mean_accept_len": round(s["sum_accept_len"] / ct, 3) if ct else 0.0,
                "mean_tokens_per_sec": (round(ct / s["generation_seconds"], 1)
                                        if s["generation_seconds"] else 0.0),
                "prefix_cache": self.prefix.info() if self.prefix is not None else {"enabled": False},
                "auto_cap": self.cap_controller.info() if self.cap_controller is not None else None}

    def close(self) -> None:
        if self.prefix is not None:
            self._executor.submit(self.prefix.reset).result()


# -------------------------------------------------------------------------------------------
_STOP = object()   # wakes the scheduler so it can return


class _Job:
    __slots__ = ("prompt_ids", "params", "on_text", "result", "error", "done")

    def __init__(self, prompt_ids, params, on_text):
        self.prompt_ids = list(prompt_ids)
        self.params = params
        self.on_text = on_text
        self.result = None
        self.error = None
        self.done = threading.Event()


class BatchEngine:
    """Continuous batching in front of an Engine (server.py:381-608); see the module docstring
    for the routing. Callers block in generate() while the scheduler runs their job."""

    def __init__(self, engine: Engine, *, max_batch: int = 4, window_s: float = 0.02,
                 slot_tokens: int | None = None):
        self.engine = engine
        self.max_batch = max(2, int(max_batch))
        self.window_s = float(window_s)
        # positions per slot of a session (its page pools are sized up front)
        self.slot_tokens = int(slot_tokens or engine.cache_tokens)
        self._q: _queue.Queue = _queue.Queue()
        self.batch_stats = {"batched_requests": 0, "batches": 0, "max_batch_seen": 0,
                            "serial_requests": 0}
        self._closed = False
        engine._executor.submit(self._scheduler)
        atexit.register(self.close)

    def close(self) -> None:
        if not self._closed:
            self._closed = True
            self._q.put(_STOP)

    def __getattr__(self, name):   # model_id, mode, spec_info, created, ... of the engine
        return getattr(self.engine, name)

    def generate(self, prompt_ids, *, max_tokens: int, temperature: float, top_p: float = 1.0,
                 top_k: int = 0, presence_penalty: float = 0.0, frequency_penalty: float = 0.0,
                 logprobs: int | None = None, stop=None, seed: int | None = None,
                 on_text=None) -> GenResult:
        job = _Job(prompt_ids, dict(max_tokens=max_tokens, temperature=temperature, top_p=top_p,
                                    top_k=top_k, presence_penalty=presence_penalty,
                                    frequency_penalty=frequency_penalty, logprobs=logprobs,
                                    stop=list(stop or []), seed=seed), on_text)
        self._q.put(job)
        job.done.wait()
        if job.error is not None:
            raise job.error
        return job.result

    def metrics(self) -> dict:
        m = self.engine.metrics()
        m["batching"] = {"max_batch": self.max_batch, **self.batch_stats}
        return m

    # ---------------------------------------------------------------- scheduler
    def _scheduler(self) -> None:
        while True:
            batch = []
            try:
                job = self._q.get()
                if job is _STOP:
                    return
                batch = [job]
                end = time.time() + self.window_s
                while len(batch) < self.max_batch:
                    left = end - time.time()
                    if left <= 0:
                        break
                    try:
                        nxt = self._q.get(timeout=left)
                    except _queue.Empty:
                        break
                    if nxt is _STOP:
                        self._q.put(nxt)          # finish this batch, return on the next get
                        break
                    batch.append(nxt)
                self._run(batch)
            except Exception as e:  # noqa: BLE001 - a dead scheduler would strand every caller
                for j in batch:
                    if not j.done.is_set():
                        j.error = RuntimeError(f"batch scheduler error: {e}")
                        j.done.set()

    def _run(self, batch: list[_Job]) -> None:
        groups: dict = {}
        for j in batch:
            p = j.params
            if p["presence_penalty"] or p["frequency_penalty"] or p["logprobs"] is not None:
                self._run_serial(j)
                continue
            groups.setdefault((p["temperature"], p["top_p"], p["top_k"]), []).append(j)
        mode = self.engine.mode
        for key, jobs in groups.items():
            sampled = key[0] > 0
            if len(jobs) == 1 or sampled or mode not in ("dspark", "baseline"):
                # lone requests and sampled groups (no batched sampling round here) run serially
                for j in jobs:
                    self._run_serial(j)
            elif mode == "dspark":
                self._run_session(jobs)
            else:
                self._run_batched(jobs)

    def _batchable_greedy(self, job: _Job) -> bool:
        p = job.params
        need = len(job.prompt_ids) + int(p["max_tokens"]) + 2 * self.engine.drafter.block_size + 2
        return (not p["presence_penalty"] and not p["frequency_penalty"]
                and p["logprobs"] is None and not p["temperature"] and not p["stop"]
                and job.on_text is None and need <= self.slot_tokens)

    def _admit(self, slots: SpecSlots, job: _Job) -> bool:
        try:
            slots.admit(job.prompt_ids, max_new_tokens=job.params["max_tokens"], meta=job)
            return True
        except BaseException as e:  # noqa: BLE001 - one bad request must not end the session
            job.error = e
            job.done.set()
            return False

    def _run_session(self, jobs: list[_Job]) -> None:
        eng = self.engine
        waiting, deferred = [], []
        for j in jobs:
            (waiting if self._batchable_greedy(j) else deferred).append(j)
        admitted = peak = 0
        t0 = time.time()
        slots = SpecSlots(eng.target, eng.tokenizer, eng.drafter, capacity=self.max_batch,
                          max_draft_tokens=eng.max_draft_tokens or 2,
                          cap_controller=eng.cap_controller, max_tokens=self.slot_tokens)
        try:
            while slots.n_active or waiting:
                while waiting and slots.has_free_slot:
                    admitted += self._admit(slots, waiting.pop(0))
                if not deferred:
                    # pull requests that arrived meanwhile into the free capacity
                    while len(waiting) < self.max_batch:
                        try:
                            nj = self._q.get_nowait()
                        except _queue.Empty:
                            break
                        if nj is _STOP:
                            self._q.put(nj)
                            break
                        if self._batchable_greedy(nj):
                            waiting.append(nj)
                        else:
                            deferred.append(nj)   # stop admitting; it runs after the session
                            break
                    while waiting and slots.has_free_slot:
                        admitted += self._admit(slots, waiting.pop(0))
                peak = max(peak, slots.n_active)
                for job, res in slots.step():
                    job.result = res
                    job.done.set()
                    eng._count(len(job.prompt_ids), res, None)
        except BaseException as e:  # noqa: BLE001
            for j in waiting + [slots.meta[b] for b in range(slots.n_active)]:
                if j is not None and not j.done.is_set():
                    j.error = e
                    j.done.set()
        finally:
            slots.release()
        eng.stats["generation_seconds"] += time.time() - t0
        self.batch_stats["batched_requests"] += admitted
        self.batch_stats["batches"] += 1
        self.batch_stats["max_batch_seen"] = max(self.batch_stats["max_batch_seen"], peak)
        for j in deferred:
            self._run_serial(j)

    def _run_serial(self, job: _Job) -> None:
        try:
            p = job.params
            job.result = self.engine._generate_impl(
                job.prompt_ids, p["max_tokens"], p["temperature"], p["top_p"], p["top_k"],
                p["stop"], p["seed"], job.on_text, p["presence_penalty"],
                p["frequency_penalty"], p["logprobs"])
            self.batch_stats["serial_requests"] += 1
        except BaseException as e:  # noqa: BLE001
            job.error = e
        finally:
            job.done.set()

    def _run_batched(self, jobs: list[_Job]) -> None:
        """Greedy baseline rows through the static batched kernel; one wall time per batch."""
        try:
            for j in jobs:
                _refuse_unbuilt(j.params["stop"], j.on_text)
            res = batch_generate_baseline(self.engine.target, self.engine.tokenizer,
                                          [j.prompt_ids for j in jobs],
                                          max_new_tokens=[j.params["max_tokens"] for j in jobs])
        except BaseException as e:  # noqa: BLE001
            for j in jobs:
                j.error = e
                j.done.set()
            return
        for j, r in zip(jobs, res):
            j.result = r
            j.done.set()
            self.engine._count(len(j.prompt_ids), r, None)
        self.engine.stats["generation_seconds"] += res[0].seconds
        self.batch_stats["batched_requests"] += len(jobs)
        self.batch_stats["batches"] += 1
        self.batch_stats["max_batch_seen"] = max(self.batch_stats["max_batch_seen"], len(jobs))


def maybe_batch_engine(engine: Engine, max_batch: int):
    """A BatchEngine around `engine` when batching applies (max_batch > 1, a batchable target,
    mode dspark or baseline); otherwise the engine itself (server.py:611-622)."""
    if max_batch <= 1 or engine.mode not in ("dspark", "baseline") or not batchable(engine.target):
        return engine
    return BatchEngine(engine, max_batch=max_batch)


__all__ = ["Engine", "BatchEngine", "maybe_batch_engine", "MODES"]
