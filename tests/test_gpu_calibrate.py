"""Auto cap on the GPU: device-timed cost curves (cached on disk), and lossless decoding while
a controller moves the cap between rounds (src/mlx_dspark/calibrate.py,
src/mlx_dspark/generate.py:846-847,924-925, src/mlx_dspark/batch_engine.py:535-538)."""
import json

import pytest
import torch

import importlib

cal = importlib.import_module("mlx_dspark_b200.calibrate")
from mlx_dspark_b200.batch_engine import SpecSlots
from mlx_dspark_b200.config import TINY, dspark_for
from mlx_dspark_b200.generate import speculative_generate
from mlx_dspark_b200.load import drafter_for, load_target
from mlx_dspark_b200.weights import generate_dspark, generate_target
from oracle.qwen3 import Qwen3Ref

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pair(cuda):
    tw = generate_target(TINY, 5, "cpu")
    dcfg = dspark_for(TINY)
    target, _ = load_target(TINY, weights=tw, device=cuda)
    drafter, _ = drafter_for(target, dcfg, weights=generate_dspark(dcfg, 5, "cpu"), device=cuda)
    g = torch.Generator().manual_seed(5)
    prompt = torch.randint(0, TINY.vocab_size, (90,), generator=g).tolist()
    return target, drafter, prompt, Qwen3Ref(tw)


def _greedy_ok(ref_t, prompt, tokens):
    """Every token is the oracle's argmax at its position (teacher-forced), or within the
    end-to-end tests' margin of it: two bf16 ulps of the top logit, at least 1e-3. Different
    verify widths sum the GEMMs in another fp32 order, so near-ties may resolve either way."""
    cache = ref_t.make_cache()
    seq = list(prompt) + list(tokens[:-1])
    rows = []
    for pos in range(0, len(seq), 64):
        rows.append(ref_t.run(seq[pos:pos + 64], cache, ())[0])
    rows = torch.cat(rows, 0)[len(prompt) - 1:]
    excused = 0
    for i, t in enumerate(tokens):
        r = rows[i]
        top = int(r.argmax())
        if t != top:
            ulp = 2.0 ** (int(torch.tensor(abs(float(r[top])) + 1e-30).log2().floor()) - 7)
            assert float(r[top] - r[t]) <= max(1e-3, 2 * ulp), (i, t, top)
            excused += 1
    return excused


def test_calibrate_measures_and_caches(pair, tmp_path):
    target, drafter, _, _ = pair
    ctl = cal.calibrate(target, drafter, mode="dspark", target_repo="tiny", drafter_repo="tiny-d",
                        cache_dir=str(tmp_path), verbose=False, batch_widths=[2])
    k = drafter.block_size
    assert set(ctl.verify_ms) == set(range(2, k + 2)) and set(ctl.drafter_ms) == set(range(1, k + 1))
    assert all(v > 0 for v in ctl.verify_ms.values()) and all(v > 0 for v in ctl.drafter_ms.values())
    assert set(ctl.verify_grid) == {2} and all(v > 0 for v in ctl.verify_grid[2].values())
    # every verify width streams the same weights: the curve stays within 2x end to end
    assert max(ctl.verify_ms.values()) < 2.0 * min(ctl.verify_ms.values())
    assert ctl.cap == 2 and 1 <= max(range(1, k + 1), key=ctl.rate) <= k
    data = json.loads((tmp_path / cal.CACHE_FILE).read_text())
    assert len(data) == 1
    again = cal.calibrate(target, drafter, mode="dspark", target_repo="tiny",
                          drafter_repo="tiny-d", cache_dir=str(tmp_path), verbose=False,
                          batch_widths=[2])
    assert again.verify_ms == ctl.verify_ms and again.drafter_ms == ctl.drafter_ms
    assert json.loads((tmp_path / cal.CACHE_FILE).read_text()) == data   # loaded, not re-measured


class _CyclingCaps:
    """A controller whose cap walks 1, 2, ..., max and around, one step per update, recording
    the caps each round used: every round runs at another verify width."""

    def __init__(self, max_cap):
        self.max_cap, self.cap, self.used = max_cap, 1, []

    def update(self, accepted_n, cap_used):
        assert 0 <= accepted_n <= cap_used
        self.used.append(cap_used)
        self.cap = self.cap % self.max_cap + 1

    def cap_for(self, B):
        return self.cap


def test_spec_decode_lossless_under_changing_caps(pair):
    target, drafter, prompt, ref_t = pair
    ctl = _CyclingCaps(drafter.block_size)
    outs = []
    for use_graph in (True, False):
        ctl.used.clear()
        ctl.cap = 1
        res = speculative_generate(target, None, drafter, lookup_drafts=False, prompt_ids=prompt, max_new_tokens=64,
                                   max_draft_tokens=None, cap_controller=ctl, use_graph=use_graph)
        assert res.num_tokens >= 64 and _greedy_ok(ref_t, prompt, res.token_ids[:64]) <= 3
        assert len(set(ctl.used)) == min(drafter.block_size, len(ctl.used)) > 1
        outs.append(res.token_ids)
    # graph-replayed and eager rounds at the same cap sequence agree exactly
    assert outs[0] == outs[1]
    # the real controller drives the same loop
    live = cal.CapController({w: 1.0 for w in range(2, 10)}, 0.1, drafter.block_size,
                             init_cap=2, repick_every=2)
    res = speculative_generate(target, None, drafter, lookup_drafts=False, prompt_ids=prompt, max_new_tokens=64,
                               max_draft_tokens=None, cap_controller=live)
    assert _greedy_ok(ref_t, prompt, res.token_ids[:64]) <= 3
    assert live.rounds == res.num_rounds


def test_batched_slots_with_controller(pair):
    target, drafter, prompt, ref_t = pair
    prompts = [prompt, prompt[:70]]
    ctl = _CyclingCaps(drafter.block_size)
    mt = max(len(p) for p in prompts) + 32 + 2 * drafter.block_size + 64
    slots = SpecSlots(target, None, drafter, capacity=2, max_draft_tokens=2, cap_controller=ctl,
                      max_tokens=mt)
    try:
        for i, ids in enumerate(prompts):
            slots.admit(ids, max_new_tokens=32, meta=i)
        out = [None, None]
        while slots.n_active:
            for meta, r in slots.step():
                out[meta] = r
    finally:
        slots.release()
    for p, r in zip(prompts, out):
        assert r.num_tokens >= 32 and _greedy_ok(ref_t, p, r.token_ids[:32]) <= 2
    assert len(set(ctl.used)) > 1
