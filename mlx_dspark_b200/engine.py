"""Serving on the device: Engine (one request at a time), BatchEngine (continuous batching on
one GPU) and ReplicaPool (request-parallel serving over several GPUs).

The reference's serving layer (src/mlx_dspark/server.py:75-622) schedules one MLX device from
an HTTP server; the HTTP handler, CLI and request parsing stay out of scope here. What is kept
is the interface: Engine(target, tokenizer, drafter, mode=...).generate(...) -> GenResult with
the same prefix-reuse rules (acquire before, store after, reset on any error), the same
per-mode decode loops, the cumulative stats behind /metrics, and the `x_mlx_dspark` block;
BatchEngine and maybe_batch_engine wrap an Engine the same way.

How work reaches the GPU is this build's own:
  * Engine owns one device thread (a single-worker executor): every launch, captured graph and
    cache of a GPU is touched from that thread only.
  * BatchEngine turns that thread into a loop over a slot table that lives as long as the
    engine (its page pools and captured round graphs are made once). A request is classified
    once, when submitted: a greedy request that fits a slot joins the admission queue, any
    other request (sampled, penalised, logprobs, too long) the solo queue. Each pass of the
    loop admits queued requests into free slots (a prefill that maps stored prefix pages),
    runs one speculative round over the active rows and hands finished rows back at once; solo
    requests run alone when the table is empty. A solo request that has waited longer than
    solo_wait_s pauses admissions so the table drains and it gets the GPU.
  * ReplicaPool runs one worker process per GPU, each with its own model replica and
    BatchEngine, and no collective between them. The host sends each request to the replica
    with the least outstanding work (prompt plus max new tokens of its unfinished requests).
Stop strings and on_text streaming callbacks work in the slot table (each row keeps its own
text stream) and on the solo path. A ReplicaPool takes stop strings but not callbacks, which
cannot be sent to its worker processes.
"""
from __future__ import annotations

import atexit
import itertools
import threading
import time
from collections import deque
from concurrent.futures import Future, ThreadPoolExecutor

from .batch_engine import SpecSlots, batch_generate_baseline, batchable
from .generate import GenResult, dflash_generate, greedy_generate, speculative_generate
from .lookup import lookup_generate
from .prefix_cache import PrefixCache, target_cache_reusable

MODES = ("dspark", "dflash", "lookup", "baseline")


def _params(max_tokens, temperature, top_p=1.0, top_k=0, presence_penalty=0.0,
            frequency_penalty=0.0, logprobs=None, stop=None, seed=None) -> dict:
    return dict(max_tokens=int(max_tokens), temperature=float(temperature), top_p=float(top_p),
                top_k=int(top_k or 0), presence_penalty=float(presence_penalty or 0.0),
                frequency_penalty=float(frequency_penalty or 0.0), logprobs=logprobs,
                stop=list(stop or []), seed=seed)


class Engine:
    """Loaded target/drafter -> GenResult, one request at a time on the engine's device thread
    (the reference's Engine, server.py:75-365)."""

    def __init__(self, target, tokenizer, drafter, *, mode: str, model_id: str = "",
                 target_repo: str = "", drafter_repo: str | None = None,
                 max_draft_tokens: int | None = None, confidence_threshold: float = 0.0,
                 prefix_cache: bool = True,
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
        self.confidence_threshold = float(confidence_threshold or 0.0)
        self.cap_controller = cap_controller      # kept across requests (auto cap)
        self.lookup_drafts = lookup_drafts
        self.cache_tokens = int(cache_tokens)     # first size of a cache; caches grow on demand
        self.prefix_cache_slots = max(1, int(prefix_cache_slots))
        self.default_max_tokens = default_max_tokens
        self.max_tokens_cap = max_tokens_cap
        # the CUDA current device is per thread: the device thread runs on the target's
        self._executor = executor or ThreadPoolExecutor(
            max_workers=1, thread_name_prefix="dspark-device",
            initializer=_bind_device, initargs=(_cuda_index(getattr(target, "device", None)),))
        self.prefix = self._make_prefix_cache(prefix_cache)
        self.created = int(time.time())
        self.stats = {"requests": 0, "prompt_tokens": 0, "completion_tokens": 0,
                      "generation_seconds": 0.0, "sum_accept_len": 0.0}
        self._decode = {"dspark": self._run_dspark, "dflash": self._run_dflash,
                        "lookup": self._run_lookup, "baseline": self._run_baseline}[mode]

    def _make_prefix_cache(self, enabled: bool):
        """Conversation prefix reuse for the modes whose caches roll back exactly (dspark,
        lookup, baseline); the DFlash drafter's context cache cannot (server.py:143-160)."""
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
        p = _params(max_tokens, temperature, top_p, top_k, presence_penalty, frequency_penalty,
                    logprobs, stop, seed)
        return self._executor.submit(self.run_request, list(prompt_ids), p, on_text).result()

    def run_request(self, prompt_ids: list[int], p: dict, on_text=None) -> GenResult:
        """One request on the calling thread (the engine's device thread)."""
        cache = ctx = None
        reuse = 0
        if self.prefix is not None:
            cache, ctx, reuse = self.prefix.acquire(prompt_ids)
        try:
            res = self._decode(prompt_ids, p, cache, ctx, reuse, on_text)
        except BaseException:
            # a cache whose contents no longer match its token record is never kept
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

    def _run_dspark(self, ids, p, cache, ctx, reuse, on_text=None) -> GenResult:
        return speculative_generate(
            self.target, self.tokenizer, self.drafter, prompt_ids=ids, cache=cache,
            ctx_caches=ctx, reuse_len=reuse, max_new_tokens=p["max_tokens"],
            max_draft_tokens=self.max_draft_tokens, cap_controller=self.cap_controller,
            confidence_threshold=self.confidence_threshold,
            lookup_drafts=self.lookup_drafts, temperature=p["temperature"], top_p=p["top_p"],
            top_k=p["top_k"], presence_penalty=p["presence_penalty"],
            frequency_penalty=p["frequency_penalty"], logprobs=p["logprobs"], seed=p["seed"],
            stop=p["stop"], on_text=on_text)

    def _run_dflash(self, ids, p, cache, ctx, reuse, on_text=None) -> GenResult:
        return dflash_generate(
            self.target, self.tokenizer, self.drafter, prompt_ids=ids,
            max_new_tokens=p["max_tokens"], max_draft_tokens=self.max_draft_tokens,
            cap_controller=self.cap_controller, temperature=p["temperature"], top_p=p["top_p"],
            top_k=p["top_k"], seed=p["seed"], stop=p["stop"], on_text=on_text)

    def _run_lookup(self, ids, p, cache, ctx, reuse, on_text=None) -> GenResult:
        return lookup_generate(
            self.target, self.tokenizer, prompt_ids=ids, cache=cache, reuse_len=reuse,
            max_new_tokens=p["max_tokens"], max_draft_tokens=self.max_draft_tokens or 6,
            temperature=p["temperature"], top_p=p["top_p"], top_k=p["top_k"], seed=p["seed"],
            stop=p["stop"], on_text=on_text)

    def _run_baseline(self, ids, p, cache, ctx, reuse, on_text=None) -> GenResult:
        return greedy_generate(
            self.target, self.tokenizer, prompt_ids=ids, cache=cache, reuse_len=reuse,
            max_new_tokens=p["max_tokens"], temperature=p["temperature"], top_p=p["top_p"],
            top_k=p["top_k"], presence_penalty=p["presence_penalty"],
            frequency_penalty=p["frequency_penalty"], logprobs=p["logprobs"], seed=p["seed"],
            stop=p["stop"], on_text=on_text)

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
        """The `x_mlx_dspark` block of a response (server.py:331-343)."""
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
class _Request:
    __slots__ = ("prompt_ids", "params", "on_text", "future", "t_submit")

    def __init__(self, prompt_ids, params: dict, on_text=None):
        self.prompt_ids = list(prompt_ids)
        self.params = params
        self.on_text = on_text
        self.future: Future = Future()
        self.t_submit = time.time()


class BatchEngine:
    """Continuous batching in front of an Engine on its device thread (see the module
    docstring). generate() blocks its caller until the request's result is ready."""

    def __init__(self, engine: Engine, *, max_batch: int = 4, slot_tokens: int | None = None,
                 solo_wait_s: float = 0.25):
        self.engine = engine
        self.max_batch = max(2, int(max_batch))
        # positions per slot (the slot table's page pools are sized up front)
        self.slot_tokens = int(slot_tokens or engine.cache_tokens)
        self.solo_wait_s = float(solo_wait_s)
        self._cv = threading.Condition()
        self._slot_q: deque[_Request] = deque()
        self._solo_q: deque[_Request] = deque()
        self._closed = False
        self._slots: SpecSlots | None = None
        self.batch_stats = {"slot_requests": 0, "solo_requests": 0, "rounds": 0,
                            "max_active": 0, "static_batches": 0}
        self._loop = engine._executor.submit(self._device_loop)
        atexit.register(self.close)

    def __getattr__(self, name):   # model_id, mode, spec_info, created, ... of the engine
        if name == "engine":
            raise AttributeError(name)
        return getattr(self.engine, name)

    # ---------------------------------------------------------------- submission
    def fits_slot(self, prompt_ids, p: dict, on_text=None) -> bool:
        """A request runs in the slot table when it decodes greedily with no per-request
        state the batched round lacks (penalties, logprobs; those run alone) and its prompt
        plus output fits one slot. Stop strings and streaming callbacks are per-row host state
        of the table (server.py:488-500)."""
        if self.engine.mode not in ("dspark", "baseline"):
            return False
        block = self.engine.drafter.block_size if self.engine.drafter is not None else 0
        need = len(prompt_ids) + p["max_tokens"] + 2 * block + 2
        return (p["temperature"] == 0.0 and not p["presence_penalty"]
                and not p["frequency_penalty"] and p["logprobs"] is None
                and need <= self.slot_tokens)

    def submit(self, prompt_ids, *, max_tokens: int, temperature: float, top_p: float = 1.0,
               top_k: int = 0, presence_penalty: float = 0.0, frequency_penalty: float = 0.0,
               logprobs: int | None = None, stop=None, seed: int | None = None,
               on_text=None) -> Future:
        p = _params(max_tokens, temperature, top_p, top_k, presence_penalty, frequency_penalty,
                    logprobs, stop, seed)
        req = _Request(prompt_ids, p, on_text)
        with self._cv:
            if self._closed:
                raise RuntimeError("BatchEngine is closed")
            (self._slot_q if self.fits_slot(req.prompt_ids, p, on_text) else self._solo_q).append(req)
            self._cv.notify()
        return req.future

    def generate(self, prompt_ids, **kw) -> GenResult:
        return self.submit(prompt_ids, **kw).result()

    def close(self) -> None:
        with self._cv:
            if self._closed:
                return
            self._closed = True
            self._cv.notify()
        try:
            self._loop.result(timeout=600)
        except Exception:  # noqa: BLE001 - closing must not raise from a failed loop
            pass

    def metrics(self) -> dict:
        m = self.engine.metrics()
        m["batching"] = {"max_batch": self.max_batch, **self.batch_stats}
        return m

    # ---------------------------------------------------------------- device thread
    def _active(self) -> int:
        return self._slots.n_active if self._slots is not None else 0

    def _device_loop(self) -> None:
        while True:
            admit: list[_Request] = []
            solo = None
            with self._cv:
                while not (self._slot_q or self._solo_q or self._active() or self._closed):
                    self._cv.wait()
                if self._closed and not (self._slot_q or self._solo_q or self._active()):
                    break
                active = self._active()
                solo_due = bool(self._solo_q) and (
                    not active or time.time() - self._solo_q[0].t_submit > self.solo_wait_s)
                if not solo_due:
                    free = self.max_batch - active
                    while self._slot_q and len(admit) < free:
                        admit.append(self._slot_q.popleft())
                if self._solo_q and not active and not admit:
                    solo = self._solo_q.popleft()
            try:
                if self.engine.mode == "baseline" and admit:
                    self._static_batch(admit)
                    continue
                for r in admit:
                    self._admit(r)
                if self._active():
                    self._round()
                elif solo is not None:
                    self._solo(solo)
            except BaseException as e:  # noqa: BLE001 - the loop must keep serving
                self._fail_active(e)
        if self._slots is not None:
            self._slots.release()
            self._slots = None

    def _table(self) -> SpecSlots:
        if self._slots is None:
            eng = self.engine
            self._slots = SpecSlots(eng.target, eng.tokenizer, eng.drafter,
                                    capacity=self.max_batch,
                                    max_draft_tokens=eng.max_draft_tokens or 2,
                                    cap_controller=eng.cap_controller,
                                    max_tokens=self.slot_tokens)
        return self._slots

    def _admit(self, r: _Request) -> None:
        try:
            self._table().admit(r.prompt_ids, max_new_tokens=r.params["max_tokens"],
                                on_text=r.on_text, stop=r.params["stop"] or None, meta=r)
            self.batch_stats["slot_requests"] += 1
        except BaseException as e:  # noqa: BLE001 - one bad request must not stop the table
            r.future.set_exception(e)

    def _round(self) -> None:
        t0 = time.time()
        table = self._table()
        self.batch_stats["max_active"] = max(self.batch_stats["max_active"], table.n_active)
        for r, res in table.step():
            self.engine._count(len(r.prompt_ids), res, None)
            r.future.set_result(res)
        self.batch_stats["rounds"] += 1
        self.engine.stats["generation_seconds"] += time.time() - t0

    def _fail_active(self, e: BaseException) -> None:
        """A failed round ends every row of the table; the table is rebuilt on next use."""
        if self._slots is not None:
            for b in range(self._slots.n_active):
                r = self._slots.meta[b]
                if r is not None and not r.future.done():
                    r.future.set_exception(e)
            try:
                self._slots.release()
            finally:
                self._slots = None

    def _solo(self, r: _Request) -> None:
        try:
            r.future.set_result(self.engine.run_request(r.prompt_ids, r.params, r.on_text))
            self.batch_stats["solo_requests"] += 1
        except BaseException as e:  # noqa: BLE001
            r.future.set_exception(e)

    def _static_batch(self, reqs: list[_Request]) -> None:
        """Baseline mode: greedy rows decoded together by the batched plain-decode graph."""
        try:
            res = batch_generate_baseline(self.engine.target, self.engine.tokenizer,
                                          [r.prompt_ids for r in reqs],
                                          max_new_tokens=[r.params["max_tokens"] for r in reqs])
        except BaseException as e:  # noqa: BLE001
            for r in reqs:
                r.future.set_exception(e)
            return
        for r, x in zip(reqs, res):
            self.engine._count(len(r.prompt_ids), x, None)
            r.future.set_result(x)
        self.engine.stats["generation_seconds"] += res[0].seconds
        self.batch_stats["slot_requests"] += len(reqs)
        self.batch_stats["static_batches"] += 1
        self.batch_stats["max_active"] = max(self.batch_stats["max_active"], len(reqs))


def maybe_batch_engine(engine: Engine, max_batch: int):
    """A BatchEngine around `engine` when batching applies (max_batch > 1, mode dspark or
    baseline, a target that batches), else the engine itself (server.py:611-622)."""
    if max_batch <= 1 or engine.mode not in ("dspark", "baseline") or not batchable(engine.target):
        return engine
    return BatchEngine(engine, max_batch=max_batch)


# -------------------------------------------------------------------------------------------
def _cuda_index(device) -> int | None:
    """The CUDA device index of `device` (the constructing thread's current device for a bare
    "cuda"), or None for a host device."""
    import torch
    if device is None:
        return None
    dev = torch.device(device)
    if dev.type != "cuda":
        return None
    return dev.index if dev.index is not None else torch.cuda.current_device()


def _bind_device(index: int | None) -> None:
    """Make CUDA device `index` the calling thread's current device."""
    if index is not None:
        import torch
        torch.cuda.set_device(index)


def _replica_main(index: int, device, factory, inbox, outbox) -> None:
    """Worker process of a ReplicaPool: build the serving object on `device`, then answer
    (id, prompt_ids, params) messages from `inbox` on `outbox` until it receives None."""
    try:
        if device is not None:
            import torch
            torch.cuda.set_device(device)
        server = factory(device)
    except BaseException as e:  # noqa: BLE001 - report and exit
        outbox.put(("failed", index, f"{type(e).__name__}: {e}"))
        return
    outbox.put(("ready", index, None))
    lock = threading.Lock()

    def reply(rid, fut):
        try:
            msg = ("done", rid, fut.result())
        except BaseException as e:  # noqa: BLE001
            msg = ("error", rid, f"{type(e).__name__}: {e}")
        with lock:
            outbox.put(msg)

    while True:
        msg = inbox.get()
        if msg is None:
            break
        rid, prompt_ids, params = msg
        fut = server.submit(prompt_ids, **params)
        fut.add_done_callback(lambda f, rid=rid: reply(rid, f))
    try:
        server.close()
    finally:
        outbox.put(("closed", index, getattr(server, "metrics", lambda: {})()))


class ReplicaPool:
    """Request-parallel serving over several GPUs (no collective): one worker process per
    device, each running factory(device) -> an object with submit(prompt_ids, **params) ->
    Future and close() (a BatchEngine, as serving_replica builds). submit() sends a request to
    the replica whose unfinished requests hold the fewest prompt + max-new tokens, ties to the
    lowest index, and returns a Future of its GenResult."""

    def __init__(self, factory, devices, *, start_timeout_s: float = 1800.0):
        import torch.multiprocessing as mp
        ctx = mp.get_context("spawn")
        self.devices = list(devices)
        self._inbox = [ctx.Queue() for _ in self.devices]
        self._outbox = ctx.Queue()
        self._procs = [ctx.Process(target=_replica_main, args=(i, d, factory, self._inbox[i],
                                                               self._outbox), daemon=True)
                       for i, d in enumerate(self.devices)]
        for p in self._procs:
            p.start()
        self.load = [0] * len(self.devices)        # outstanding tokens per replica
        self.assigned = [0] * len(self.devices)    # requests sent to each replica
        self.replica_metrics: dict[int, dict] = {}
        self._pending: dict[int, tuple[Future, int, int]] = {}
        self._ids = itertools.count()
        self._lock = threading.Lock()
        ready = 0
        deadline = time.time() + start_timeout_s
        while ready < len(self.devices):
            left = deadline - time.time()
            kind, idx, info = self._outbox.get(timeout=max(1.0, left))
            if kind == "failed":
                self._stop_all()
                raise RuntimeError(f"replica {idx} failed to start: {info}")
            ready += kind == "ready"
        self._collector = threading.Thread(target=self._collect, daemon=True)
        self._collector.start()

    def submit(self, prompt_ids, **params) -> Future:
        if params.get("on_text") is not None:
            raise ValueError("on_text callbacks cannot be sent to replica processes; stream "
                             "from an in-process Engine or BatchEngine")
        cost = len(prompt_ids) + int(params.get("max_tokens", 0))
        fut: Future = Future()
        with self._lock:
            i = min(range(len(self.devices)), key=lambda k: (self.load[k], k))
            rid = next(self._ids)
            self.load[i] += cost
            self.assigned[i] += 1
            self._pending[rid] = (fut, i, cost)
        self._inbox[i].put((rid, list(prompt_ids), dict(params)))
        return fut

    def generate(self, prompt_ids, **params) -> GenResult:
        return self.submit(prompt_ids, **params).result()

    def _collect(self) -> None:
        closed = 0
        while closed < len(self.devices):
            kind, key, payload = self._outbox.get()
            if kind == "closed":
                self.replica_metrics[key] = payload
                closed += 1
                continue
            with self._lock:
                fut, i, cost = self._pending.pop(key)
                self.load[i] -= cost
            if kind == "done":
                fut.set_result(payload)
            else:
                fut.set_exception(RuntimeError(payload))

    def _stop_all(self) -> None:
        for q in self._inbox:
            q.put(None)
        for p in self._procs:
            p.join(timeout=120)
            if p.is_alive():
                p.terminate()

    def close(self) -> None:
        self._stop_all()
        self._collector.join(timeout=60)


def serving_replica(device, *, target: str = "qwen3-8b", seed: int = 1, kv_bits: int | None = 8,
                    block_size: int = 8, max_batch: int = 4, slot_tokens: int = 4608,
                    max_draft_tokens: int = 8):
    """A ReplicaPool factory: a synthetic target of a preset architecture (seeded weights, the
    same on every replica) with a DSpark drafter, served by a BatchEngine on `device`."""
    import functools  # noqa: F401 - the factory is usually passed as functools.partial
    from .config import TARGETS, dspark_for
    from .load import drafter_for, load_target
    tgt, tok = load_target(target, kv_bits=kv_bits, seed=seed, device=device)
    drafter, _ = drafter_for(tgt, dspark_for(TARGETS[target], block_size=block_size), seed=seed,
                             device=device)
    eng = Engine(tgt, tok, drafter, mode="dspark", max_draft_tokens=max_draft_tokens,
                 lookup_drafts=False, cache_tokens=slot_tokens)
    return BatchEngine(eng, max_batch=max_batch, slot_tokens=slot_tokens)


__all__ = ["Engine", "BatchEngine", "ReplicaPool", "maybe_batch_engine", "serving_replica",
           "MODES"]
