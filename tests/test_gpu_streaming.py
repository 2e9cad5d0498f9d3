"""Stop strings and streaming callbacks through the decode loops on the GPU (_Streamer,
generate.py:294-362, used by speculative_generate, greedy_generate and lookup_generate): a
stop string cuts the text and ends the decode at a round boundary with finish_reason "stop",
the callback receives exactly the result text, the committed tokens are those of the same
decode without streaming, and StopStreaming from the callback ends the decode normally."""
import pytest
import torch

from mlx_dspark_b200.config import TINY, dspark_for
from mlx_dspark_b200.generate import StopStreaming, greedy_generate, speculative_generate
from mlx_dspark_b200.load import drafter_for, load_target
from mlx_dspark_b200.lookup import lookup_generate
from mlx_dspark_b200.weights import generate_dspark, generate_target

pytestmark = pytest.mark.gpu


class IdTok:
    """Each id decodes to "<id>"; no eos ids."""

    def decode(self, ids):
        return "".join(f"<{int(i)}>" for i in ids)


@pytest.fixture(scope="module")
def tiny(cuda):
    tw = generate_target(TINY, 0, "cpu")
    target, _ = load_target(TINY, weights=tw, device=cuda)
    dcfg = dspark_for(TINY)
    drafter, _ = drafter_for(target, dcfg, weights=generate_dspark(dcfg, 0, "cpu"), device=cuda)
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, TINY.vocab_size, (128,), generator=g).tolist()
    return dict(target=target, drafter=drafter, prompt=prompt)


def _stop_after(tokens):
    """Index j of the first token unlike the first one, and the stop string of its text."""
    j = next((i for i, t in enumerate(tokens) if t != tokens[0]), None)
    if j is None:
        pytest.skip("the decode repeats one token")
    return j, f"<{tokens[j]}>"


@pytest.mark.parametrize("loop", ["speculative", "greedy", "lookup"])
def test_stop_string_and_callback(tiny, loop):
    t, d, prompt = tiny["target"], tiny["drafter"], tiny["prompt"]
    N = 40

    def run(**kw):
        if loop == "speculative":
            return speculative_generate(t, IdTok(), d, prompt_ids=prompt, max_new_tokens=N,
                                        max_draft_tokens=None, lookup_drafts=False, **kw)
        if loop == "greedy":
            return greedy_generate(t, IdTok(), prompt_ids=prompt, max_new_tokens=N, **kw)
        return lookup_generate(t, IdTok(), prompt_ids=prompt, max_new_tokens=N, **kw)

    plain = run()
    assert plain.text == IdTok().decode(plain.token_ids)
    j, stop = _stop_after(plain.token_ids)
    got = []
    res = run(stop=[stop], on_text=got.append)
    assert res.finish_reason == "stop"
    assert res.text == IdTok().decode(plain.token_ids[:j])
    assert "".join(got) == res.text
    n = len(res.token_ids)
    assert j < n < N and res.token_ids == plain.token_ids[:n]
    # a callback with no stop strings receives the whole text
    got = []
    full = run(on_text=got.append)
    assert "".join(got) == full.text == plain.text


def test_stop_streaming_ends_the_decode(tiny):
    calls = []

    def cb(s):
        calls.append(s)
        raise StopStreaming()

    res = speculative_generate(tiny["target"], IdTok(), tiny["drafter"], prompt_ids=tiny["prompt"],
                               max_new_tokens=40, max_draft_tokens=None, lookup_drafts=False,
                               on_text=cb)
    assert len(calls) == 1 and res.finish_reason == "stop" and res.num_tokens < 40
