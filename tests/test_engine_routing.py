"""The serving layer's host logic on the CPU: how BatchEngine classifies requests (slot table or
solo), that its device loop admits into free slots, steps the table, runs solo requests when the
table is empty and pauses admissions for a solo request that waited too long, that a failed round
fails only the table's rows, and that ReplicaPool sends each request to the least-loaded replica
(worker processes started with spawn, stub servers, no GPU)."""
import threading
import time
from concurrent.futures import Future
from types import SimpleNamespace

import pytest

from mlx_dspark_b200 import engine as eng_mod
from mlx_dspark_b200.generate import GenResult


def _res(ids, n=1):
    return GenResult(text="", token_ids=list(ids), num_tokens=len(ids), num_rounds=n,
                     accept_lengths=[1] * n, target_forwards=n, seconds=0.0)


class _StubEngine:
    """Stands in for Engine: runs solo requests instantly and records them."""

    def __init__(self, mode="dspark"):
        from concurrent.futures import ThreadPoolExecutor
        self.mode = mode
        self._executor = ThreadPoolExecutor(max_workers=1)
        self.cache_tokens = 4096
        self.drafter = SimpleNamespace(block_size=8)
        self.max_draft_tokens = 2
        self.cap_controller = None
        self.stats = {"requests": 0, "prompt_tokens": 0, "completion_tokens": 0,
                      "generation_seconds": 0.0, "sum_accept_len": 0.0}
        self.solo = []
        self.on_text = []

    def run_request(self, prompt_ids, p, on_text=None):
        self.solo.append(prompt_ids[0])
        self.on_text.append(on_text)
        return _res(prompt_ids)

    def _count(self, *a):
        self.stats["requests"] += 1

    def metrics(self):
        return dict(self.stats)


class _FakeTable:
    """A slot table whose rows finish after `rounds` steps each."""

    def __init__(self, capacity, rounds=2, fail_on=None):
        self.capacity, self.rounds, self.fail_on = capacity, rounds, fail_on
        self.rows = []            # [request, steps left]
        self.admitted = []
        self.steps = 0
        self.released = False

    @property
    def n_active(self):
        return len(self.rows)

    @property
    def meta(self):
        return [r for r, _ in self.rows]

    def admit(self, ids, *, max_new_tokens, meta, on_text=None, stop=None):
        assert len(self.rows) < self.capacity
        self.admitted.append(ids[0])
        self.text_args = (on_text, stop)
        self.rows.append([meta, self.rounds])

    def step(self):
        self.steps += 1
        if self.fail_on is not None and self.steps == self.fail_on:
            raise RuntimeError("device error")
        done, keep = [], []
        for r in self.rows:
            r[1] -= 1
            (done if r[1] == 0 else keep).append(r)
        self.rows = keep
        return [(r, _res(r.prompt_ids)) for r, _ in done]

    def release(self):
        self.released = True


@pytest.fixture()
def batch_engine(monkeypatch):
    tables = []

    def fake_table(self):
        if self._slots is None:
            self._slots = _FakeTable(self.max_batch, fail_on=getattr(self, "_fail_on", None))
            tables.append(self._slots)
        return self._slots

    monkeypatch.setattr(eng_mod.BatchEngine, "_table", fake_table)
    e = _StubEngine()
    be = eng_mod.BatchEngine(e, max_batch=2, solo_wait_s=0.05)
    yield e, be, tables
    be.close()
    e._executor.shutdown(wait=True)


def test_classification():
    e = _StubEngine()
    be = eng_mod.BatchEngine.__new__(eng_mod.BatchEngine)
    be.engine, be.slot_tokens = e, 4096
    ok = eng_mod._params(16, 0.0)
    assert be.fits_slot([1] * 10, ok)
    assert not be.fits_slot([1] * 10, eng_mod._params(16, 0.7))                  # sampled
    assert not be.fits_slot([1] * 10, eng_mod._params(16, 0.0, presence_penalty=0.5))
    assert not be.fits_slot([1] * 10, eng_mod._params(16, 0.0, logprobs=2))
    assert not be.fits_slot([1] * 5000, ok)                                       # too long
    assert be.fits_slot([1] * 10, eng_mod._params(16, 0.0, stop=["\n"]))         # per-row text
    assert be.fits_slot([1] * 10, ok, on_text=print)
    e.mode = "lookup"
    assert not be.fits_slot([1] * 10, ok)


def test_loop_batches_greedy_and_runs_solo_requests(batch_engine):
    e, be, tables = batch_engine
    futs = [be.submit([i], max_tokens=4, temperature=0.0) for i in range(5)]
    futs.append(be.submit([9], max_tokens=4, temperature=0.8))
    futs.append(be.submit([10], max_tokens=4, temperature=0.0, presence_penalty=0.3))
    res = [f.result(timeout=10) for f in futs]
    assert [r.token_ids[0] for r in res] == [0, 1, 2, 3, 4, 9, 10]
    assert sorted(tables[0].admitted) == [0, 1, 2, 3, 4] and sorted(e.solo) == [9, 10]
    st = be.metrics()["batching"]
    assert st["slot_requests"] == 5 and st["solo_requests"] == 2 and st["max_active"] == 2
    # stop strings and streaming callbacks go to the table with the row
    r = be.generate([11], max_tokens=4, temperature=0.0, stop=["x"], on_text=print)
    assert r.token_ids == [11] and tables[0].admitted[-1] == 11
    assert tables[0].text_args == (print, ["x"])
    # and to the engine with a solo request
    r = be.generate([12], max_tokens=4, temperature=0.5, stop=["y"], on_text=print)
    assert e.solo[-1] == 12 and e.on_text[-1] is print


def test_failed_round_fails_only_its_rows(batch_engine):
    e, be, tables = batch_engine
    be._fail_on = 1
    a = be.submit([1], max_tokens=4, temperature=0.0)
    with pytest.raises(RuntimeError):
        a.result(timeout=10)
    assert tables[0].released
    be._fail_on = None
    b = be.submit([2], max_tokens=4, temperature=0.0)
    assert b.result(timeout=10).token_ids == [2]      # a fresh table serves the next request


def _stub_server(device, delay=0.0):
    class S:
        def submit(self, prompt_ids, **params):
            f = Future()

            def done():
                time.sleep(delay * len(prompt_ids))
                f.set_result(_res(prompt_ids + [params["max_tokens"]]))
            threading.Thread(target=done).start()
            return f

        def close(self):
            pass

        def metrics(self):
            return {"device": device}
    return S()


def test_replica_pool_least_loaded_dispatch():
    import functools
    pool = eng_mod.ReplicaPool(functools.partial(_stub_server, delay=0.002), [None, None],
                               start_timeout_s=120)
    try:
        # one long request, then short ones: the short ones go to the other replica first
        fl = pool.submit([1] * 200, max_tokens=100)
        fs = [pool.submit([2] * 10, max_tokens=10) for _ in range(4)]
        assert pool.assigned == [1, 4]
        out = [f.result(timeout=60) for f in [fl] + fs]
        assert out[0].token_ids[-1] == 100 and all(o.token_ids[-1] == 10 for o in out[1:])
        assert pool.load == [0, 0]
    finally:
        pool.close()
    assert set(pool.replica_metrics) == {0, 1}


def test_replica_pool_refuses_callbacks():
    """Callbacks cannot be sent to worker processes; stop strings can."""
    pool = eng_mod.ReplicaPool.__new__(eng_mod.ReplicaPool)
    with pytest.raises(ValueError, match="on_text"):
        pool.submit([1], max_tokens=4, temperature=0.0, on_text=print)


def test_row_tracker_text_stream():
    """The slot table's per-row state: a stop string ends the row, its text is cut, the
    callback gets exactly that text, and a row without one decodes every id (fake tokenizer,
    no GPU)."""
    from mlx_dspark_b200.batch_engine import _RowTracker

    class Tok:
        eos_token_id = 99

        def decode(self, ids):
            return "".join(chr(97 + i) for i in ids)

    got = []
    t = _RowTracker(Tok(), 0, 50, on_text=got.append, stop=["de"])
    t.commit([1, 2], accept_len=3)
    assert not t.finished
    t.commit([3, 4, 5], accept_len=4)
    assert t.finished
    t.commit([6])                              # ignored once finished
    r = t.result(0.0)
    assert r.text == "abc" and "".join(got) == "abc" and r.finish_reason == "stop"
    assert r.token_ids == [0, 1, 2, 3, 4, 5] and r.accept_lengths == [3, 4]
    plain = _RowTracker(Tok(), 0, 4)
    plain.commit([1, 99, 7])
    r = plain.result(0.0)
    assert r.text == "ab" and r.token_ids == [0, 1, 99] and r.finish_reason == "stop"
