"""Continuous batching on the device (tiny config; BASELINE C4 in miniature).

Every row of a batch must decode its own prompt greedily: checked teacher-forced against the
CPU oracle (bf16 KV, or 8-bit KV pages against the oracle's KV8 cache), with near-ties excused
as in test_gpu_e2e. The queue runner must reuse the shared prompt prefix's pages (prefix
hits, fewer prefilled tokens) and survive staggered retirement (row compaction)."""
import pytest
import torch

from mlx_dspark_b200.batch_engine import (SpecSlots, batch_generate_baseline, batch_spec_generate,
                                          serve_requests)
from mlx_dspark_b200.config import TINY, dspark_for
from mlx_dspark_b200.load import drafter_for, load_target
from mlx_dspark_b200.weights import generate_dspark, generate_target
from oracle.qwen3 import Qwen3Ref

from test_gpu_e2e import _gap_tol

pytestmark = pytest.mark.gpu


def _tf_check(ref_t, prompt, tokens, kv8=False):
    cache = ref_t.make_cache(kv8)
    seq = list(prompt) + list(tokens[:-1])
    rows, pos = [], 0
    while pos < len(seq):
        lg, _ = ref_t.run(seq[pos:pos + 64], cache, ())
        rows.append(lg)
        pos += 64
    rows = torch.cat(rows, 0)[len(prompt) - 1:]
    excused = 0
    for i, t in enumerate(tokens):
        r = rows[i]
        top = int(r.argmax())
        if t != top:
            assert float(r[top] - r[t]) <= _gap_tol(float(r[top])), (i, t, top)
            excused += 1
    return excused


@pytest.fixture(scope="module")
def tiny(cuda):
    tw = generate_target(TINY, 0, "cpu")
    dcfg = dspark_for(TINY)
    dw = generate_dspark(dcfg, 0, "cpu")
    out = {"tw": tw, "ref": Qwen3Ref(tw)}
    for kv in (None, 8):
        t, _ = load_target(TINY, weights=tw, kv_bits=kv, device=cuda)
        d, _ = drafter_for(t, dcfg, weights=dw, device=cuda)
        out[kv] = (t, d)
    g = torch.Generator().manual_seed(5)
    shared = torch.randint(0, TINY.vocab_size, (130,), generator=g).tolist()
    out["prompts"] = [shared + torch.randint(0, TINY.vocab_size, (n,), generator=g).tolist()
                      for n in (3, 70, 21, 140, 9)]
    return out


@pytest.mark.parametrize("kv", [None, 8])
def test_batch_spec_rows_are_each_greedy(tiny, kv):
    target, drafter = tiny[kv]
    prompts = tiny["prompts"][:3]
    res = batch_spec_generate(target, None, drafter, prompts, max_new_tokens=[40, 24, 32],
                              max_draft_tokens=8)
    for p, r, n in zip(prompts, res, [40, 24, 32]):
        assert r.num_tokens >= n and sum(r.accept_lengths) + 1 == r.num_tokens
        assert _tf_check(tiny["ref"], p, r.token_ids[:n], kv8=kv == 8) <= 3


def test_batch_baseline_rows_are_each_greedy(tiny):
    target, _ = tiny[None]
    prompts = tiny["prompts"][:3]
    res = batch_generate_baseline(target, None, prompts, max_new_tokens=[20, 12, 16])
    for p, r, n in zip(prompts, res, [20, 12, 16]):
        assert r.num_tokens == n
        assert _tf_check(tiny["ref"], p, r.token_ids, kv8=False) <= 2


def test_queue_reuses_prefix_pages_and_compacts(tiny):
    target, drafter = tiny[8]
    prompts = tiny["prompts"]
    reqs = [(p, n) for p, n in zip(prompts, [30, 12, 44, 18, 26])]
    res, stats = serve_requests(target, None, drafter, reqs, capacity=2, max_draft_tokens=8)
    assert stats["prefix_hits"] >= 4                     # the 128-token shared prefix (2 pages)
    assert stats["prefix_reused_tokens"] >= 4 * 128
    assert stats["prefill_tokens"] <= sum(len(p) for p in prompts) - 4 * 128
    for (p, n), r in zip(reqs, res):
        assert r.num_tokens >= n
        assert _tf_check(tiny["ref"], p, r.token_ids[:n], kv8=True) <= 3
    # the same requests without prefix reuse give the same tokens (up to near-ties)
    res2, stats2 = serve_requests(target, None, drafter, reqs, capacity=2, max_draft_tokens=8,
                                  prefix_reuse=False)
    assert stats2["prefix_hits"] == 0
    for (p, n), a, b in zip(reqs, res, res2):
        agree = sum(x == y for x, y in zip(a.token_ids[:n], b.token_ids[:n]))
        assert agree >= n - 4, (a.token_ids[:n], b.token_ids[:n])
