"""CPU checks of the DFlash restatement (no GPU).

The reference has no DFlash test vectors, so these pin invariants the reference loop
guarantees: greedy dflash_generate (src/mlx_dspark/generate.py:468-601) emits exactly the
target's greedy decoding, and the drafter's context cache behaves like the reference's
KVCache (appending the context in two pieces gives the same block logits as in one).
"""
import torch

from mlx_dspark_b200.config import TINY, dflash_for
from mlx_dspark_b200.weights import generate_dflash, generate_target
from oracle.dflash import DFlashRef, dflash_generate_ref
from oracle.dspark import greedy_generate_ref
from oracle.qwen3 import Qwen3Ref


def _setup():
    tw = generate_target(TINY, 0, "cpu")
    fw = generate_dflash(dflash_for(TINY), 0, "cpu")
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, TINY.vocab_size, (40,), generator=g).tolist()
    return Qwen3Ref(tw), DFlashRef(fw, tw), prompt


def test_dflash_greedy_loop_is_target_greedy():
    t, f, prompt = _setup()
    out, acc = dflash_generate_ref(t, f, prompt, 24, max_draft_tokens=4)
    ref, _ = greedy_generate_ref(t, prompt, len(out))
    assert out == ref
    assert sum(acc) + 1 == len(out)


def test_dflash_context_append_is_piecewise():
    t, f, prompt = _setup()
    _, fused = t.run(prompt, t.make_cache(), list(f.cfg.target_layer_ids))
    a = f.draft_logits(7, fused, f.make_cache(), 15)
    c = f.make_cache()
    f.update_context(fused[:25], 0, c)
    b = f.draft_logits(7, fused[25:], c, 15)
    assert torch.equal(a, b)
