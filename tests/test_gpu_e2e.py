"""End-to-end GPU parity on the tiny config (BASELINE C1 shapes) against the CPU oracle.

Tolerances:
  * logits: |gpu - oracle| <= 2e-2 * max|oracle row| (bf16 rtol 2e-2 of the row scale);
  * greedy tokens, teacher-forced: every emitted token is the oracle's argmax at its
    position, unless the oracle's margin top1 - logit[token] is within GAP_TOL. The logits
    are bf16 (an MLX bf16 model's logits are), so two candidates one bf16 ulp apart can swap
    when one rounding lands differently; GAP_TOL = max(1e-3, 2 bf16 ulps of the top logit).
"""
import pytest
import torch

from mlx_dspark_b200.config import TINY, dspark_for
from mlx_dspark_b200.generate import greedy_generate, speculative_generate
from mlx_dspark_b200.load import drafter_for, load_target
from mlx_dspark_b200.weights import generate_dspark, generate_target
from oracle.dspark import DSparkRef
from oracle.qwen3 import Qwen3Ref, prefill

pytestmark = pytest.mark.gpu

SEED = 0


@pytest.fixture(scope="module")
def tiny(cuda):
    tw = generate_target(TINY, SEED, "cpu")
    dcfg = dspark_for(TINY)
    dw = generate_dspark(dcfg, SEED, "cpu")
    target, tok = load_target(TINY, weights=tw, device=cuda)
    drafter, _ = drafter_for(target, dcfg, weights=dw, device=cuda)
    ref_t = Qwen3Ref(tw)
    ref_d = DSparkRef(dw, tw)
    g = torch.Generator().manual_seed(SEED)
    prompt = torch.randint(0, TINY.vocab_size, (128,), generator=g).tolist()
    return dict(tw=tw, dw=dw, target=target, drafter=drafter, ref_t=ref_t, ref_d=ref_d,
                prompt=prompt, dcfg=dcfg)


def _gap_tol(top: float) -> float:
    ulp = 2.0 ** (int(torch.tensor(abs(top) + 1e-30).log2().floor()) - 7)
    return max(1e-3, 2 * ulp)


def teacher_forced_check(ref_t, prompt, tokens):
    """Run the oracle over prompt + tokens[:-1]; check each token against the oracle row."""
    cache = ref_t.make_cache()
    seq = list(prompt) + list(tokens[:-1])
    rows = []
    pos = 0
    while pos < len(seq):
        lg, _ = ref_t.run(seq[pos:pos + 64], cache, ())
        rows.append(lg)
        pos += 64
    rows = torch.cat(rows, 0)[len(prompt) - 1:]
    excused, worst = 0, 0.0
    for i, t in enumerate(tokens):
        r = rows[i]
        top = int(r.argmax())
        if t != top:
            gap = float(r[top] - r[t])
            assert gap <= _gap_tol(float(r[top])), (i, t, top, gap)
            excused += 1
            worst = max(worst, gap)
    return excused, worst


def test_target_forward_logits_and_taps(tiny):
    target, ref_t, prompt = tiny["target"], tiny["ref_t"], tiny["prompt"]
    tap = tiny["dcfg"].target_layer_ids
    cache = target.make_cache(512)
    logits, fused = target.run([prompt], cache, tap)
    rc = ref_t.make_cache()
    rl, rf = ref_t.run(prompt, rc, tap)
    gl = logits[0].float().cpu()
    scale = rl.abs().amax(dim=-1, keepdim=True)
    assert ((gl - rl).abs() <= 2e-2 * scale).all(), float(((gl - rl).abs() / scale).max())
    gf = fused[0].float().cpu()
    fs = rf.abs().amax(dim=-1, keepdim=True)
    assert ((gf - rf).abs() <= 2e-2 * fs).all()
    assert cache.offset == len(prompt)
    # a second call continues from the cache offset (KVCache semantics), then trim works
    l2, _ = target.run([[5, 6, 7]], cache, tap)
    rl2, _ = ref_t.run([5, 6, 7], rc, tap)
    assert ((l2[0].float().cpu() - rl2).abs() <= 2e-2 * rl2.abs().amax(-1, keepdim=True)).all()
    for c in cache:
        c.trim(2)
    for c in rc:
        c.trim(2)
    l3, _ = target.run([[9]], cache, tap)
    rl3, _ = ref_t.run([9], rc, tap)
    assert ((l3[0].float().cpu() - rl3).abs() <= 2e-2 * rl3.abs().amax(-1, keepdim=True)).all()


def test_greedy_decode_teacher_forced(tiny):
    res = greedy_generate(tiny["target"], None, prompt_ids=tiny["prompt"], max_new_tokens=64)
    assert res.num_tokens == 64
    excused, worst = teacher_forced_check(tiny["ref_t"], tiny["prompt"], res.token_ids)
    assert excused <= 3, (excused, worst)


def test_speculative_decode_is_target_greedy(tiny):
    res = speculative_generate(tiny["target"], None, tiny["drafter"], lookup_drafts=False, prompt_ids=tiny["prompt"],
                               max_new_tokens=96, max_draft_tokens=None)
    assert res.num_tokens >= 96
    assert sum(res.accept_lengths) + 1 == res.num_tokens
    assert all(1 <= a <= 9 for a in res.accept_lengths)
    excused, worst = teacher_forced_check(tiny["ref_t"], tiny["prompt"], res.token_ids)
    assert excused <= 3, (excused, worst)
    # the graph-replayed rounds and eager rounds agree exactly
    res2 = speculative_generate(tiny["target"], None, tiny["drafter"], lookup_drafts=False, prompt_ids=tiny["prompt"],
                                max_new_tokens=96, max_draft_tokens=None, use_graph=False)
    assert res2.token_ids == res.token_ids and res2.accept_lengths == res.accept_lengths


def test_drafter_matches_oracle(tiny):
    """The first draft block after prefill equals the oracle drafter's (same context)."""
    target, drafter, prompt = tiny["target"], tiny["drafter"], tiny["prompt"]
    from mlx_dspark_b200.generate import SpecSession, prefill_rows
    sess = SpecSession(target, drafter, 1, 8, len(prompt) + 64)
    last = prefill_rows(target, prompt, sess.tstate, sess.tap, drafter, sess.cstate)
    pending = int(last.float().argmax())
    sess.pending.fill_(pending)
    drafter.draft_dev(sess.pending, 1, 8, sess.cstate, sess.dbuf, sess.draft, sess.vbuf.ids,
                      sess.splits_c)
    torch.cuda.synchronize()
    gpu_draft = sess.draft[0].tolist()
    base_gpu = sess.dbuf.base[:8].float().cpu()
    sess.release()
    ref_t, ref_d = tiny["ref_t"], tiny["ref_d"]
    rc, ctx = ref_t.make_cache(), ref_d.make_ctx_cache()
    lg, fused = ref_t.run(prompt, rc, ref_d.cfg.target_layer_ids)
    ref_d.update_context(fused, 0, ctx)
    noise = ref_d.embed([pending] + [ref_d.cfg.mask_token_id] * 7)
    hidden = ref_d.backbone(noise, len(prompt), ctx)
    base = ref_d.compute_logits(hidden)
    sc = base.abs().amax(-1, keepdim=True)
    assert ((base_gpu - base).abs() <= 2e-2 * sc).all(), float(((base_gpu - base).abs() / sc).max())
    # greedy Markov chain over the GPU base logits reproduces the GPU draft exactly
    assert ref_d.sample_block(base_gpu, pending) == gpu_draft


def test_override_accept_lengths_exact(tiny):
    """Bernoulli(0.7) agree mask over the target's own greedy continuation: every round
    accepts exactly the leading run of agreements (+1 bonus)."""
    target, drafter, prompt = tiny["target"], tiny["drafter"], tiny["prompt"]
    N, cap = 80, 8
    ref = greedy_generate(target, None, prompt_ids=prompt, max_new_tokens=N + cap + 2).token_ids
    g = torch.Generator().manual_seed(123)
    rounds = N
    agree = (torch.rand(1, rounds, cap, generator=g) < 0.7).to(torch.uint8)
    ov = {"ref": torch.tensor([ref]), "agree": agree, "prompt_len": [len(prompt)]}
    res = speculative_generate(target, None, drafter, lookup_drafts=False, prompt_ids=prompt, max_new_tokens=N,
                               max_draft_tokens=cap, draft_override=ov)
    assert res.token_ids[:N] == ref[:N]
    for r, a in enumerate(res.accept_lengths):
        lead = 0
        while lead < cap and agree[0, r, lead]:
            lead += 1
        assert a == lead + 1, (r, a, lead)
