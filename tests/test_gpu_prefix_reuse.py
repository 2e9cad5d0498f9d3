"""Prefix reuse on the device (tiny config): a second conversation turn acquires the first
turn's paged caches from PrefixCache, prefills only the new suffix and decodes the same tokens
as a cold run of the full prompt (greedy; positions where the cold and warm runs differ must be
near-ties, as test_gpu_e2e excuses)."""
import pytest
import torch

from mlx_dspark_b200.config import TINY, dspark_for
from mlx_dspark_b200.generate import speculative_generate
from mlx_dspark_b200.load import drafter_for, load_target
from mlx_dspark_b200.prefix_cache import PrefixCache, target_cache_reusable
from mlx_dspark_b200.weights import generate_dspark, generate_target
from oracle.qwen3 import Qwen3Ref

from test_gpu_e2e import teacher_forced_check

pytestmark = pytest.mark.gpu


def test_second_turn_reuses_the_first(cuda):
    tw = generate_target(TINY, 0, "cpu")
    target, _ = load_target(TINY, weights=tw, device=cuda)
    dcfg = dspark_for(TINY)
    drafter, _ = drafter_for(target, dcfg, weights=generate_dspark(dcfg, 0, "cpu"), device=cuda)
    g = torch.Generator().manual_seed(1)
    turn1 = torch.randint(0, TINY.vocab_size, (100,), generator=g).tolist()
    pc = PrefixCache(lambda: target.make_cache(256), lambda: drafter.make_ctx_cache(256),
                     min_reuse=16)
    cache, ctx, reuse = pc.acquire(turn1)
    assert reuse == 0 and target_cache_reusable(cache)
    r1 = speculative_generate(target, None, drafter, lookup_drafts=False, prompt_ids=turn1, cache=cache, ctx_caches=ctx,
                              reuse_len=reuse, max_new_tokens=40, max_draft_tokens=None)
    assert cache.offset == len(turn1) + len(r1.token_ids) - 1
    pc.store(cache, ctx, turn1, r1.token_ids)
    turn2 = turn1 + r1.token_ids + torch.randint(0, TINY.vocab_size, (30,), generator=g).tolist()
    cache2, ctx2, reuse2 = pc.acquire(turn2)
    assert cache2 is cache and reuse2 == len(turn1) + len(r1.token_ids) - 1
    warm = speculative_generate(target, None, drafter, lookup_drafts=False, prompt_ids=turn2, cache=cache2,
                                ctx_caches=ctx2, reuse_len=reuse2, max_new_tokens=40,
                                max_draft_tokens=None)
    cold = speculative_generate(target, None, drafter, lookup_drafts=False, prompt_ids=turn2, max_new_tokens=40,
                                max_draft_tokens=None)
    assert pc.hits == 1 and pc.reused_tokens == reuse2
    excused, worst = teacher_forced_check(Qwen3Ref(tw), turn2, warm.token_ids[:40])
    assert excused <= 3, (excused, worst)
    agree = sum(a == b for a, b in zip(warm.token_ids, cold.token_ids))
    assert agree >= 36, (warm.token_ids, cold.token_ids)
    pc.reset()
