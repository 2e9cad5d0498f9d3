"""BatchEngine routing on the CPU with a stub engine (src/mlx_dspark/server.py:438-487): which
requests share a continuous session, which go serial, and that every caller gets its result."""
import threading
from concurrent.futures import ThreadPoolExecutor
from types import SimpleNamespace

import pytest

from mlx_dspark_b200 import engine as eng_mod
from mlx_dspark_b200.generate import GenResult


class _StubEngine:
    def __init__(self, mode="dspark"):
        self.mode = mode
        self._executor = ThreadPoolExecutor(max_workers=1)
        self.cache_tokens = 4096
        self.drafter = SimpleNamespace(block_size=8)
        self.max_draft_tokens = 2
        self.cap_controller = None
        self.stats = {"requests": 0, "prompt_tokens": 0, "completion_tokens": 0,
                      "generation_seconds": 0.0, "sum_accept_len": 0.0}
        self.serial = []

    def _generate_impl(self, prompt_ids, max_tokens, temperature, *rest):
        stop, on_text = rest[2], rest[4]
        eng_mod._refuse_unbuilt(stop, on_text)
        self.serial.append(tuple(prompt_ids))
        return GenResult(text="", token_ids=list(prompt_ids), num_tokens=len(prompt_ids),
                         num_rounds=1, accept_lengths=[1], target_forwards=1, seconds=0.0)

    def metrics(self):
        return {}


def _job(ids, **kw):
    p = dict(max_tokens=8, temperature=0.0, top_p=1.0, top_k=0, presence_penalty=0.0,
             frequency_penalty=0.0, logprobs=None, stop=[], seed=None)
    p.update(kw)
    return eng_mod._Job(ids, p, None)


@pytest.fixture()
def batch_engine(monkeypatch):
    e = _StubEngine()
    be = eng_mod.BatchEngine(e, max_batch=4, window_s=0.2)
    sessions, batched = [], []

    def fake_session(self, jobs):
        sessions.append([j.prompt_ids[0] for j in jobs])
        for j in jobs:
            j.result = "batched"
            j.done.set()

    def fake_batched(self, jobs):
        batched.append([j.prompt_ids[0] for j in jobs])
        for j in jobs:
            j.result = "static"
            j.done.set()

    monkeypatch.setattr(eng_mod.BatchEngine, "_run_session", fake_session)
    monkeypatch.setattr(eng_mod.BatchEngine, "_run_batched", fake_batched)
    yield e, be, sessions, batched
    be.close()
    e._executor.shutdown(wait=True)


def test_routing_by_sampling_and_penalties(batch_engine):
    e, be, sessions, batched = batch_engine
    jobs = [_job([1]), _job([2]), _job([3], temperature=0.7), _job([4], temperature=0.7),
            _job([5], presence_penalty=0.5), _job([6], logprobs=2), _job([7], top_k=5)]
    be._run(jobs)
    assert sessions == [[1, 2]]                        # the greedy group shares a session
    assert sorted(s[0] for s in e.serial) == [3, 4, 5, 6, 7]   # sampled, penalised, logprobs, alone
    assert all(j.done.is_set() for j in jobs) and be.batch_stats["serial_requests"] == 5
    e.mode = "baseline"
    sessions.clear()
    be._run([_job([8]), _job([9])])
    assert batched == [[8, 9]] and not sessions


def test_queue_delivers_every_caller_and_refusals(batch_engine):
    e, be, sessions, _ = batch_engine
    out = {}

    def call(i, **kw):
        try:
            out[i] = be.generate([i], max_tokens=4, temperature=kw.get("t", 0.0),
                                 stop=kw.get("stop"))
        except NotImplementedError as err:
            out[i] = err

    ts = [threading.Thread(target=call, args=(i,)) for i in range(3)]
    ts.append(threading.Thread(target=call, args=(9,), kwargs={"t": 0.5, "stop": ["x"]}))
    for t in ts:
        t.start()
    for t in ts:
        t.join(10)
    assert out[0] == out[1] == out[2] == "batched" and sessions and sum(map(len, sessions)) == 3
    assert isinstance(out[9], NotImplementedError)
    assert be._batchable_greedy(_job([1] * 5000)) is False      # longer than a slot
    assert be._batchable_greedy(_job([1], stop=["\n"])) is False
