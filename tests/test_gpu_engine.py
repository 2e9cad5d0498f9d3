"""Engine and BatchEngine on the GPU (the reference's serving layer, src/mlx_dspark/server.py:
75-622): prefix reuse across requests, a concurrent mix (greedy rows in the persistent slot
table, sampled and penalised requests solo) whose greedy outputs are the target's greedy
decoding, stats, and the refusal of stop strings."""
import threading

import pytest
import torch

from mlx_dspark_b200.config import TINY, dspark_for
from mlx_dspark_b200.engine import BatchEngine, Engine, maybe_batch_engine
from mlx_dspark_b200.load import drafter_for, load_target
from mlx_dspark_b200.weights import generate_dspark, generate_target
from oracle.qwen3 import Qwen3Ref

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pair(cuda):
    tw = generate_target(TINY, 6, "cpu")
    dcfg = dspark_for(TINY)
    target, _ = load_target(TINY, weights=tw, device=cuda)
    drafter, _ = drafter_for(target, dcfg, weights=generate_dspark(dcfg, 6, "cpu"), device=cuda)
    return target, drafter, Qwen3Ref(tw)


def _prompt(n, seed):
    return torch.randint(0, TINY.vocab_size, (n,), generator=torch.Generator().manual_seed(seed)).tolist()


def _greedy_ok(ref_t, prompt, tokens):
    """Teacher-forced oracle check with the end-to-end tests' near-tie margin (two bf16 ulps of
    the top logit, at least 1e-3); returns how many tokens needed the margin."""
    cache = ref_t.make_cache()
    seq = list(prompt) + list(tokens[:-1])
    rows = torch.cat([ref_t.run(seq[p:p + 64], cache, ())[0] for p in range(0, len(seq), 64)], 0)
    rows = rows[len(prompt) - 1:]
    excused = 0
    for i, t in enumerate(tokens):
        r = rows[i]
        top = int(r.argmax())
        if t != top:
            ulp = 2.0 ** (int(torch.tensor(abs(float(r[top])) + 1e-30).log2().floor()) - 7)
            assert float(r[top] - r[t]) <= max(1e-3, 2 * ulp), (i, t, top)
            excused += 1
    return excused


def test_engine_prefix_reuse_and_metrics(pair):
    target, drafter, ref = pair
    engine = Engine(target, None, drafter, mode="dspark", max_draft_tokens=4,
                    lookup_drafts=False, cache_tokens=512)
    try:
        p1 = _prompt(80, 1)
        r1 = engine.generate(p1, max_tokens=24, temperature=0.0)
        assert _greedy_ok(ref, p1, r1.token_ids[:24]) <= 2
        # the follow-up turn extends the first conversation: its prefix is reused
        p2 = p1 + r1.token_ids[:-1] + _prompt(20, 2)
        r2 = engine.generate(p2, max_tokens=24, temperature=0.0)
        assert _greedy_ok(ref, p2, r2.token_ids[:24]) <= 2
        m = engine.metrics()
        assert m["requests"] == 2 and m["prefix_cache"]["hits"] == 1
        assert m["prefix_cache"]["reused_tokens"] >= len(p1)
        assert m["completion_tokens"] == r1.num_tokens + r2.num_tokens
        info = engine.spec_info(r2)
        assert info["mode"] == "dspark" and info["target_forwards"] == r2.target_forwards
        with pytest.raises(NotImplementedError):
            engine.generate(p1, max_tokens=4, temperature=0.0, stop=["x"])
    finally:
        engine.close()


def test_batch_engine_concurrent_mix(pair):
    target, drafter, ref = pair
    engine = Engine(target, None, drafter, mode="dspark", max_draft_tokens=2,
                    lookup_drafts=False, cache_tokens=512)
    be = maybe_batch_engine(engine, 4)
    assert isinstance(be, BatchEngine)
    prompts = [_prompt(60 + 5 * i, 10 + i) for i in range(4)]
    out, errs = {}, {}

    def call(i, **kw):
        try:
            out[i] = be.generate(prompts[i % 4], max_tokens=20, **kw)
        except Exception as e:  # noqa: BLE001
            errs[i] = e

    threads = [threading.Thread(target=call, args=(i,), kwargs={"temperature": 0.0})
               for i in range(4)]
    threads.append(threading.Thread(target=call, args=(4,),
                                    kwargs={"temperature": 0.8, "top_k": 20, "seed": 1}))
    threads.append(threading.Thread(target=call, args=(5,),
                                    kwargs={"temperature": 0.0, "presence_penalty": 0.5}))
    try:
        for t in threads:
            t.start()
        for t in threads:
            t.join(300)
        assert not errs, errs
        for i in range(4):
            assert out[i].num_tokens >= 20
            assert _greedy_ok(ref, prompts[i], out[i].token_ids[:20]) <= 2
        assert out[4].num_tokens >= 20 and out[5].num_tokens >= 20
        st = be.metrics()["batching"]
        assert st["slot_requests"] == 4 and st["solo_requests"] == 2
        assert st["max_active"] >= 1 and be.metrics()["requests"] == 6
        # a second wave reuses the same slot table (no new pools or graphs)
        table = be._slots
        more = [be.submit(prompts[i], max_tokens=12, temperature=0.0) for i in range(4)]
        for i, f in enumerate(more):
            r = f.result(timeout=300)
            assert _greedy_ok(ref, prompts[i], r.token_ids[:12]) <= 2
        assert be._slots is table
    finally:
        be.close()
        engine.close()
