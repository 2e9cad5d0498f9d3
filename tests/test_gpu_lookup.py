"""GPU checks of the n-gram lookup drafts (pure lookup_generate and hybrid rounds inside
speculative_generate): greedy output equals the target's greedy decoding (teacher-forced
against the oracle, ties excused as in test_gpu_e2e), lookup drafts actually fire on the
repetitive random-init model, and a sampled lookup verify (one-hot proposal) is replayed
exactly by the CPU sampler on the GPU's logits."""
import pytest
import torch

from mlx_dspark_b200.config import TINY, dspark_for
from mlx_dspark_b200.generate import speculative_generate
from mlx_dspark_b200.kvcache import CacheState
from mlx_dspark_b200.load import drafter_for, load_target
from mlx_dspark_b200.lookup import BlockVerifier, lookup_generate
from mlx_dspark_b200.model import Sampling
from mlx_dspark_b200 import ops
from mlx_dspark_b200.generate import prefill_rows
from mlx_dspark_b200.weights import generate_dspark, generate_target
from oracle import sampling as S
from oracle.qwen3 import Qwen3Ref

from test_gpu_e2e import teacher_forced_check

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny(cuda):
    tw = generate_target(TINY, 0, "cpu")
    target, _ = load_target(TINY, weights=tw, device=cuda)
    dcfg = dspark_for(TINY)
    drafter, _ = drafter_for(target, dcfg, weights=generate_dspark(dcfg, 0, "cpu"), device=cuda)
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, TINY.vocab_size, (128,), generator=g).tolist()
    return dict(target=target, drafter=drafter, ref_t=Qwen3Ref(tw), prompt=prompt)


def test_lookup_generate_is_target_greedy(tiny):
    res = lookup_generate(tiny["target"], None, prompt_ids=tiny["prompt"], max_new_tokens=96)
    assert res.num_tokens >= 96
    assert sum(res.accept_lengths) + 1 == res.num_tokens
    assert max(res.accept_lengths) > 1          # the model repeats itself: lookups hit
    excused, worst = teacher_forced_check(tiny["ref_t"], tiny["prompt"], res.token_ids[:96])
    assert excused <= 3, (excused, worst)


def test_hybrid_lookup_rounds_are_target_greedy(tiny):
    res = speculative_generate(tiny["target"], None, tiny["drafter"], prompt_ids=tiny["prompt"],
                               max_new_tokens=96, max_draft_tokens=None, lookup_drafts=True)
    assert res.lookup_rounds > 0
    assert sum(res.accept_lengths) + 1 == res.num_tokens
    excused, worst = teacher_forced_check(tiny["ref_t"], tiny["prompt"], res.token_ids[:96])
    assert excused <= 3, (excused, worst)
    plain = speculative_generate(tiny["target"], None, tiny["drafter"], lookup_drafts=False, prompt_ids=tiny["prompt"],
                                 max_new_tokens=96, max_draft_tokens=None)
    n = min(len(res.token_ids), len(plain.token_ids), 96)
    assert res.token_ids[:n] == plain.token_ids[:n]


def test_sampled_lookup_verify_replays_exactly(tiny):
    t, prompt = tiny["target"], tiny["prompt"]
    st = CacheState(t.new_pool(512, 1), 1, 512, t.device)
    st.ensure(0, 512)
    sm, seed = Sampling(0.8, 0.9, 30), 5
    rng = ops.rng_state(seed, t.device)
    ver = BlockVerifier(t, st, (), sm, rng)
    prefill_rows(t, prompt, st, ())
    pending = prompt[-1]
    for r in range(4):
        draft = [prompt[(7 * r + i) % len(prompt)] for i in range(5)]
        buf, plan, plan_host = ver.launch(pending, draft, commit=True)
        logits = buf.logits.to(torch.bfloat16).cpu()
        row = ver.finish(plan, plan_host)
        n, repl, _, _ = S.accept_sample_exact(logits, [pending] + draft, None, sm.temperature, 0,
                                              sm.top_p, sm.top_k, seed, r, q_onehot=True)
        assert row[0] == n and row[2 + n] == repl, (r, row, n, repl)
        pending = repl
    st.release()
