"""Confidence truncation of DSpark drafts (speculative_generate's confidence_threshold,
generate.py:855-887; ConfidenceHead model.py:211-217, confidence_logits :311-320) on the GPU.

The dspark_confidence kernel against the oracle's confidence head (bf16 logits and sigmoids,
one bf16 step of tolerance for fp32 sum order), from normalised rows and from the backbone's
pre-norm rows; then the decode loop, with drafts that all agree with the target: truncation
never changes the greedy output, a threshold no position reaches leaves rounds of one drafted
token, one every position passes leaves the rounds as without the head, and a round's drafted
count follows the survival rule on confidences that match the oracle drafter's."""
import dataclasses

import pytest
import torch

from mlx_dspark_b200 import ops
from mlx_dspark_b200.config import TINY, dspark_for
from mlx_dspark_b200.generate import (SpecSession, greedy_generate, prefill_rows,
                                      speculative_generate)
from mlx_dspark_b200.load import drafter_for, load_target
from mlx_dspark_b200.weights import generate_dspark, generate_target
from oracle.dspark import DSparkRef, truncate_by_confidence
from oracle.qwen3 import Qwen3Ref, rms_norm

pytestmark = pytest.mark.gpu


def _close_bf16(got: torch.Tensor, want: torch.Tensor) -> bool:
    return torch.allclose(got.float(), want.float(), rtol=2.0 ** -7, atol=2.0 ** -9)


@pytest.fixture(scope="module")
def conf(cuda):
    tw = generate_target(TINY, 0, "cpu")
    dcfg = dataclasses.replace(dspark_for(TINY), enable_confidence_head=True)
    dw = generate_dspark(dcfg, 0, "cpu")
    target, _ = load_target(TINY, weights=tw, device=cuda)
    drafter, _ = drafter_for(target, dcfg, weights=dw, device=cuda)
    plain_cfg = dspark_for(TINY)
    plain, _ = drafter_for(target, plain_cfg, weights=generate_dspark(plain_cfg, 0, "cpu"),
                           device=cuda)
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, TINY.vocab_size, (128,), generator=g).tolist()
    return dict(tw=tw, dw=dw, target=target, drafter=drafter, plain=plain, prompt=prompt,
                ref_t=Qwen3Ref(tw), ref_d=DSparkRef(dw, tw))


def test_confidence_kernel_normalised_rows(conf, cuda):
    d, ref = conf["drafter"], conf["ref_d"]
    g = torch.Generator().manual_seed(2)
    H = TINY.hidden_size
    h = torch.randn(8, H, generator=g).to(torch.bfloat16)
    prev = torch.randint(0, TINY.vocab_size, (8,), generator=g).tolist()
    got = d.confidence_logits(h.to(cuda), prev).cpu()
    want = ref.confidence_logits(h, prev)
    assert _close_bf16(got, want), (got, want)
    assert got.abs().max() > 0.5                   # the head is not trivially zero
    # one row: no previous-draft list
    one = d.confidence_logits(h[:1].to(cuda), prev[:1]).cpu()
    assert _close_bf16(one, want[:1])


def test_confidence_kernel_prenorm_rows(conf, cuda):
    d, ref, dw = conf["drafter"], conf["ref_d"], conf["dw"]
    g = torch.Generator().manual_seed(3)
    H = TINY.hidden_size
    h = (torch.randn(6, H, generator=g) * 4).to(torch.bfloat16)
    prev = torch.randint(0, TINY.vocab_size, (6,), generator=g).tolist()
    pend = torch.tensor(prev[:1], dtype=torch.int32, device=cuda)
    rest = torch.tensor(prev[1:], dtype=torch.int32, device=cuda)
    c = torch.zeros(6, dtype=torch.float32, device=cuda)
    lg = torch.zeros(6, dtype=torch.float32, device=cuda)
    ch = d.confidence_head
    ops.confidence(h.to(cuda), 6, ch.w, ch.b, c, norm_w=d.norm, eps=dw.cfg.rms_norm_eps,
                   w1=d.markov_head.w1, first_prev=pend, prev_rest=rest, logit=lg)
    torch.cuda.synchronize()
    hn = rms_norm(h, dw.norm, dw.cfg.rms_norm_eps)
    assert _close_bf16(lg.cpu(), ref.confidence_logits(hn, prev))
    assert _close_bf16(c.cpu(), ref.confidence(hn, prev))


def _agree_all(conf, n, cap):
    """Draft override whose drafts are the target's own greedy continuation (every draft is
    accepted unless the confidence head truncates it), with that continuation."""
    t, prompt = conf["target"], conf["prompt"]
    ref = greedy_generate(t, None, prompt_ids=prompt, max_new_tokens=n + cap + 2).token_ids
    ov = {"ref": torch.tensor([ref]), "agree": torch.ones(1, n, cap, dtype=torch.uint8),
          "prompt_len": [len(prompt)]}
    return ov, ref


def test_truncation_keeps_greedy_output(conf):
    N, cap = 48, 8
    ov, ref = _agree_all(conf, N, cap)
    kw = dict(prompt_ids=conf["prompt"], max_new_tokens=N, max_draft_tokens=cap,
              lookup_drafts=False, draft_override=ov)
    t, d = conf["target"], conf["drafter"]
    base = speculative_generate(t, None, d, **kw)
    assert base.token_ids[:N] == ref[:N] and set(base.accept_lengths) == {cap + 1}
    never = speculative_generate(t, None, d, confidence_threshold=1e-30, **kw)
    assert never.token_ids == base.token_ids and never.accept_lengths == base.accept_lengths
    always = speculative_generate(t, None, d, confidence_threshold=1.5, logprobs=1, **kw)
    assert always.token_ids[:N] == ref[:N] and set(always.accept_lengths) == {2}
    assert len(always.logprobs) == always.num_tokens
    mid = speculative_generate(t, None, d, confidence_threshold=0.5, **kw)
    assert mid.token_ids[:N] == ref[:N]
    assert all(2 <= a <= cap + 1 for a in mid.accept_lengths)
    # survival products of ~0.7-0.9 per position fall below 0.5 before the eighth draft
    assert max(mid.accept_lengths) < cap + 1
    # a drafter without the head ignores the threshold (generate.py:808)
    p = conf["plain"]
    assert (speculative_generate(t, None, p, confidence_threshold=0.5, **kw).accept_lengths
            == speculative_generate(t, None, p, **kw).accept_lengths)


def test_conf_step_plan_and_oracle_confidences(conf, cuda):
    """One truncated round through SpecSession.conf_step: the drafted count follows the
    survival rule on the round's confidences, the plan accepts exactly that many (all drafts
    agree), and the confidences match the oracle drafter's for the same round."""
    t, d, prompt = conf["target"], conf["drafter"], conf["prompt"]
    cap = 8
    ov, ref = _agree_all(conf, 4, cap)
    sess = SpecSession(t, d, 1, cap, len(prompt) + 64, override=ov)
    try:
        last = prefill_rows(t, prompt, sess.tstate, sess.tap, d, sess.cstate)
        pending = t.argmax_row(last)
        assert pending == ref[0]
        sess.pending_host[0] = pending
        plan, drafted = sess.conf_step(0.5)
        vals = sess._conf[1][:cap].tolist()
    finally:
        sess.release()
    keep = len(truncate_by_confidence(list(range(cap)), vals, 0.5))
    assert drafted == keep and plan[0] == keep, (plan, drafted, vals)
    assert plan[2:3 + keep] == ref[1:2 + keep]
    # the oracle drafter's round: prefill, block backbone, Markov draft, confidences
    rt, rd, dcfg = conf["ref_t"], conf["ref_d"], conf["dw"].cfg
    cache, ctx = rt.make_cache(), rd.make_ctx_cache()
    _, fused = rt.run(prompt, cache, list(dcfg.target_layer_ids))
    rd.update_context(fused, 0, ctx)
    hidden = rd.backbone(rd.embed([pending] + [dcfg.mask_token_id] * (dcfg.block_size - 1)),
                         len(prompt), ctx)
    draft = rd.sample_block(rd.compute_logits(hidden[:cap]), pending)
    want = rd.confidence(hidden[:cap], [pending] + draft[:-1])
    assert torch.allclose(torch.tensor(vals), want.float(), rtol=0, atol=0.02), (vals, want)


def test_sampled_truncation_runs(conf):
    t, d = conf["target"], conf["drafter"]
    res = speculative_generate(t, None, d, prompt_ids=conf["prompt"], max_new_tokens=32,
                               max_draft_tokens=None, lookup_drafts=False, temperature=1.0,
                               top_p=0.95, top_k=50, seed=5, confidence_threshold=1.5)
    assert res.num_tokens >= 32 and max(res.accept_lengths) <= 2
    res = speculative_generate(t, None, d, prompt_ids=conf["prompt"], max_new_tokens=32,
                               max_draft_tokens=None, lookup_drafts=False, temperature=1.0,
                               top_p=0.95, top_k=50, seed=5, confidence_threshold=0.5)
    assert res.num_tokens >= 32
    assert all(0 <= x < TINY.vocab_size for x in res.token_ids)
