"""Per-token logprobs (GenResult.logprobs, generate.py:149-176) on the GPU.

The dspark_logprobs kernel against the CPU restatement on random, tie-heavy, signed-zero and
small-vocabulary rows; then the decode loops: every entry's row is the raw target row the
token was committed from (greedy: the token is its row's top entry; with penalties: the
entries match the oracle's log-softmax at each position, which they would not if the
penalised logits had been read), through drafter rounds, lookup rounds and plain decoding."""
import math

import numpy as np
import pytest
import torch

from mlx_dspark_b200 import ops
from mlx_dspark_b200.config import TINY, dspark_for
from mlx_dspark_b200.generate import greedy_generate, speculative_generate
from mlx_dspark_b200.load import drafter_for, load_target
from mlx_dspark_b200.weights import generate_dspark, generate_target
from oracle.logprobs import log_softmax_f32, logprobs_for_block
from oracle.qwen3 import Qwen3Ref

pytestmark = pytest.mark.gpu

ATOL = 2e-5  # fp32 log-softmax: sum order and exp/log rounding


def _kernel(rows_bf16: torch.Tensor, ids: list[int], top_k: int, cuda, ld: int | None = None):
    R, V = rows_bf16.shape
    ld = V if ld is None else ld
    buf = torch.zeros(R, ld, dtype=torch.bfloat16)
    buf[:, :V] = rows_bf16
    buf = buf.to(cuda)
    ids_d = torch.tensor(ids, dtype=torch.int32, device=cuda)
    logp = torch.zeros(R, dtype=torch.float32, device=cuda)
    k = max(top_k, 1)
    ti = torch.full((R, k), -7, dtype=torch.int32, device=cuda)
    tv = torch.zeros(R, k, dtype=torch.float32, device=cuda)
    ops.logprobs(buf, R, ids_d, R, R, top_k, logp, ti if top_k else None, tv if top_k else None,
                 V=V)
    torch.cuda.synchronize()
    return logp.cpu(), ti.cpu(), tv.cpu()


def _compare(rows_bf16, ids, top_k, cuda, ld=None):
    logp, ti, tv = _kernel(rows_bf16, ids, top_k, cuda, ld)
    want = logprobs_for_block(rows_bf16.float().numpy(), ids, top_k)
    for r, e in enumerate(want):
        assert abs(float(logp[r]) - e["logprob"]) <= ATOL, (r, float(logp[r]), e["logprob"])
        if top_k:
            k = len(e["top"])
            assert ti[r, :k].tolist() == [t for t, _ in e["top"]], r
            assert np.allclose(tv[r, :k].numpy(), [v for _, v in e["top"]], rtol=0, atol=ATOL)
            assert (ti[r, k:] == -7).all()          # nothing past min(top_k, V)


@pytest.mark.parametrize("top_k", [0, 1, 5, 20, 1024])
def test_kernel_random_rows(cuda, top_k):
    g = torch.Generator().manual_seed(top_k)
    V = 151936
    rows = (torch.randn(9, V, generator=g) * 3).to(torch.bfloat16)
    ids = torch.randint(0, V, (9,), generator=g).tolist()
    _compare(rows, ids, top_k, cuda)


@pytest.mark.parametrize("top_k", [3, 20, 700])
def test_kernel_tie_heavy_rows(cuda, top_k):
    g = torch.Generator().manual_seed(1)
    V = 32768
    levels = torch.tensor([-1.0, 0.0, 0.5, 1.0])
    rows = levels[torch.randint(0, 4, (4, V), generator=g)].to(torch.bfloat16)
    rows[1, :] = 0.0                                  # one row of all-equal values
    ids = [0, 5, V - 1, 123]
    _compare(rows, ids, top_k, cuda)


def test_kernel_signed_zero_small_vocab_and_scalar_path(cuda):
    V = 50
    rows = torch.full((2, V), -2.0).to(torch.bfloat16)
    rows[0, 7] = -0.0
    rows[0, 3] = 0.0
    rows[1, 11] = 4.0
    # top_k past the vocabulary, and a row pitch (51) that rules out 16-byte loads
    _compare(rows, [7, 11], 64, cuda, ld=51)


def test_kernel_token_outside_vocab_is_nan(cuda):
    rows = torch.zeros(2, 1000).to(torch.bfloat16)
    logp, _, _ = _kernel(rows, [-1, 1000], 0, cuda)
    assert torch.isnan(logp).all()


@pytest.fixture(scope="module")
def tiny(cuda):
    tw = generate_target(TINY, 0, "cpu")
    target, _ = load_target(TINY, weights=tw, device=cuda)
    dcfg = dspark_for(TINY)
    drafter, _ = drafter_for(target, dcfg, weights=generate_dspark(dcfg, 0, "cpu"), device=cuda)
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, TINY.vocab_size, (128,), generator=g).tolist()
    return dict(target=target, drafter=drafter, ref=Qwen3Ref(tw), prompt=prompt)


def _oracle_logp(ref, prompt, tokens) -> np.ndarray:
    """Oracle log-softmax rows at the positions that committed tokens[0..]."""
    cache = ref.make_cache()
    seq = list(prompt) + list(tokens[:-1])
    rows = []
    for pos in range(0, len(seq), 64):
        lg, _ = ref.run(seq[pos:pos + 64], cache, ())
        rows.append(lg)
    rows = torch.cat(rows, 0)[len(prompt) - 1:]
    return log_softmax_f32(rows.to(torch.bfloat16).float().numpy())


def _greedy_consistent(res, top_k):
    assert res.logprobs is not None and len(res.logprobs) == res.num_tokens
    for e, t in zip(res.logprobs, res.token_ids):
        assert e["token_id"] == t
        assert math.isfinite(e["logprob"]) and e["logprob"] <= 0.0
        if top_k:
            assert len(e["top"]) == top_k
            # greedy: the committed token is its row's first maximum, the top entry
            assert e["top"][0][0] == t and e["top"][0][1] == e["logprob"], e
            vals = [v for _, v in e["top"]]
            assert vals == sorted(vals, reverse=True)


def test_speculative_logprobs_greedy(tiny):
    kw = dict(prompt_ids=tiny["prompt"], max_new_tokens=40, max_draft_tokens=None,
              lookup_drafts=False)
    plain = speculative_generate(tiny["target"], None, tiny["drafter"], **kw)
    res = speculative_generate(tiny["target"], None, tiny["drafter"], logprobs=4, **kw)
    assert res.token_ids == plain.token_ids and plain.logprobs is None
    _greedy_consistent(res, 4)
    chosen = speculative_generate(tiny["target"], None, tiny["drafter"], logprobs=0, **kw)
    assert all("top" not in e for e in chosen.logprobs)
    assert [e["logprob"] for e in chosen.logprobs] == [e["logprob"] for e in res.logprobs]


def test_lookup_rounds_logprobs(tiny):
    res = speculative_generate(tiny["target"], None, tiny["drafter"], prompt_ids=tiny["prompt"],
                               max_new_tokens=96, max_draft_tokens=None, lookup_drafts=True,
                               logprobs=2)
    assert res.lookup_rounds > 0
    _greedy_consistent(res, 2)


def test_greedy_generate_logprobs(tiny):
    res = greedy_generate(tiny["target"], None, prompt_ids=tiny["prompt"], max_new_tokens=24,
                          logprobs=3)
    _greedy_consistent(res, 3)


@pytest.mark.parametrize("lookup", [False, True])
def test_penalised_logprobs_are_raw_rows(tiny, lookup):
    """With penalties the entries are still the raw rows: they match the oracle's log-softmax
    at every position (a penalised row would be off by the 0.8 presence penalty on repeats)."""
    pen = dict(presence_penalty=0.8, frequency_penalty=0.3)
    res = speculative_generate(tiny["target"], None, tiny["drafter"], prompt_ids=tiny["prompt"],
                               max_new_tokens=48, max_draft_tokens=None, lookup_drafts=lookup,
                               logprobs=2, **pen)
    toks = res.token_ids[:48]
    want = _oracle_logp(tiny["ref"], tiny["prompt"], toks)
    got = np.array([e["logprob"] for e in res.logprobs[:48]])
    ref_chosen = want[np.arange(len(toks)), toks]
    assert np.abs(got - ref_chosen).max() < 0.1, np.abs(got - ref_chosen).max()
    tops = np.array([e["top"][0][1] for e in res.logprobs[:48]])
    assert np.abs(tops - want.max(-1)).max() < 0.1
    g = greedy_generate(tiny["target"], None, prompt_ids=tiny["prompt"], max_new_tokens=24,
                        logprobs=1, **pen)
    want_g = _oracle_logp(tiny["ref"], tiny["prompt"], g.token_ids)
    got_g = np.array([e["logprob"] for e in g.logprobs])
    assert np.abs(got_g - want_g[np.arange(len(g.token_ids)), g.token_ids]).max() < 0.1
