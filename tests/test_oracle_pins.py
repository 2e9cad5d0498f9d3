"""Pins of the CPU oracle (no GPU): against the committed HF-transformers Qwen3 fixture and
against the known-answer unit tests of the reference (restated on the oracle)."""
import os

import pytest
import torch

from mlx_dspark_b200.config import TINY
from mlx_dspark_b200.weights import generate_target, quantize_w8g64
from oracle import qwen3 as oq
from oracle.sampling import batch_mask, ctx_block_mask, spec_sample_accept, truncate_probs

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "qwen3_tiny_hf.pt")


@pytest.fixture(scope="module")
def tiny_w():
    return generate_target(TINY, 0, "cpu")


def test_oracle_matches_hf_qwen3_fixture(tiny_w):
    """fp32 oracle forward == transformers Qwen3ForCausalLM on the same dequantized weights,
    including a chunked prefill through the KV cache (the fixture is one full forward)."""
    g = torch.load(GOLDEN)
    ids = g["ids"].tolist()
    m = oq.Qwen3Ref(tiny_w, rnd=False)
    cache = m.make_cache()
    tap_ids = tuple(sorted(g["taps"])) + (TINY.num_hidden_layers - 1,)
    rows, taps = [], {i: [] for i in tap_ids}
    H = TINY.hidden_size
    for s in range(0, len(ids), 20):  # 20 + 20 + 8: exercises cache offsets and masks
        lg, fused = m.run(ids[s:s + 20], cache, tap_ids)
        rows.append(lg)
        for j, i in enumerate(tap_ids):
            taps[i].append(fused[:, j * H:(j + 1) * H])
    logits = torch.cat(rows)
    last = torch.cat(taps[TINY.num_hidden_layers - 1])
    normed = oq.rms_norm(last, tiny_w.norm, TINY.rms_norm_eps, rnd=False)
    assert torch.allclose(normed[:, :64], g["final_hidden_norm"], atol=2e-5, rtol=1e-5)
    assert torch.allclose(logits[:, :256], g["logits_head"], atol=2e-5, rtol=1e-5)
    assert torch.allclose(logits[:, 1000:1016], g["logits_sel"], atol=2e-5, rtol=1e-5)
    assert torch.allclose(torch.logsumexp(logits, -1), g["lse"], atol=2e-5)
    assert torch.equal(torch.topk(logits, 8, -1).indices, g["top_idx"])
    assert len(g["taps"]) >= 2
    for i in g["taps"]:
        assert torch.allclose(torch.cat(taps[i])[:, :64], g["taps"][i], atol=2e-5, rtol=1e-5)


def test_bf16_rounding_model_stays_close_to_fp32(tiny_w):
    """The MLX-style bf16 rounding points perturb logits by well under the bf16 rtol."""
    ids = list(range(100, 132))
    l32 = oq.Qwen3Ref(tiny_w, rnd=False).run(ids, oq.Qwen3Ref(tiny_w).make_cache(), ())[0]
    lbf = oq.Qwen3Ref(tiny_w, rnd=True).run(ids, oq.Qwen3Ref(tiny_w).make_cache(), ())[0]
    scale = l32.abs().amax(-1, keepdim=True)
    assert ((lbf - l32).abs() <= 2e-2 * scale).all()


# --- reference known-answer tests, restated on the oracle ----------------------------------

def test_build_batch_mask_causal_and_padding():
    """tests/test_batch_engine.py:87-95 of the reference."""
    m = batch_mask([2, 0], T=2)
    assert m.shape == (2, 1, 2, 4)
    grid = m.to(torch.int32).tolist()
    assert grid[0][0][0] == [1, 1, 1, 0]
    assert grid[0][0][1] == [1, 1, 1, 1]
    assert grid[1][0][0] == [1, 0, 0, 0]
    assert grid[1][0][1] == [1, 1, 0, 0]


def test_build_batch_mask_single_token_decode():
    """tests/test_batch_engine.py:97-103 of the reference."""
    grid = batch_mask([5, 3, 0], T=1).to(torch.int32).tolist()
    assert grid[0][0][0] == [1, 1, 1, 1, 1, 1]
    assert grid[1][0][0] == [1, 1, 1, 1, 0, 0]
    assert grid[2][0][0] == [1, 0, 0, 0, 0, 0]


def test_ctx_block_mask_hides_context_padding():
    """tests/test_batch_engine.py:185-191 of the reference."""
    g = ctx_block_mask([2, 0], k=2).to(torch.int32).tolist()
    assert g[0][0][0] == [1, 1, 1, 1]
    assert g[1][0][0] == [0, 0, 1, 1]


def test_gqa_broadcast_equals_explicit_tiling():
    """tests/test_model.py:25-60 of the reference: native GQA == tiled K/V (atol 1e-5)."""
    torch.manual_seed(0)
    q = torch.randn(8, 3, 16)
    k = torch.randn(2, 8, 16)
    v = torch.randn(2, 8, 16)
    native = oq.sdpa(q, k, v, 16 ** -0.5, None, rnd=False)
    tiled = oq.sdpa(q, k.repeat_interleave(4, 0), v.repeat_interleave(4, 0), 16 ** -0.5, None, rnd=False)
    assert torch.allclose(native, tiled, atol=1e-5)


def test_topp_speculative_sampling_is_lossless():
    """tests/test_generate_helpers.py:145-170 of the reference: the committed token is an
    exact sample from top-p/top-k(softmax(target/T)) whatever the draft q (0.02 max-abs,
    20000 draws)."""
    import numpy as np

    gen = torch.Generator().manual_seed(0)
    V = 6
    target = torch.tensor([2.0, 1.0, 0.5, 0.0, -1.0, -2.0])
    q = torch.softmax(torch.tensor([-2.0, -1.0, 0.0, 0.5, 1.0, 2.0]), -1)
    v_logits = torch.stack([target, target])
    qrow = q.reshape(1, V)
    for (T, tp, tk) in [(1.0, 1.0, 0), (1.0, 0.8, 0), (0.7, 1.0, 3)]:
        exp = truncate_probs(torch.softmax(target / T, -1), tp, tk).numpy()
        counts = np.zeros(V)
        xs = torch.multinomial(q.expand(20000, V), 1, replacement=True, generator=gen)[:, 0]
        for x in xs.tolist():
            n, repl = spec_sample_accept(v_logits, [x], qrow, T, tp, tk, gen)
            counts[x if n == 1 else repl] += 1
        emp = counts / counts.sum()
        assert np.abs(emp - exp).max() < 0.02, (T, tp, tk, emp, exp)


def test_truncate_probs_rules():
    p = torch.tensor([[0.4, 0.3, 0.2, 0.1]])
    assert torch.equal(truncate_probs(p, 1.0, 0), p)                       # identity fast path
    assert torch.allclose(truncate_probs(p, 1.0, 2), torch.tensor([[4 / 7, 3 / 7, 0, 0]]))
    # nucleus 0.75: exclusive prefix masses 0, .4, .7, .9 -> keep the first three
    assert torch.allclose(truncate_probs(p, 0.75, 0), torch.tensor([[0.4, 0.3, 0.2, 0]]) / 0.9)
    # ties at the k-th value are kept
    t = torch.tensor([[0.3, 0.3, 0.3, 0.1]])
    assert (truncate_probs(t, 1.0, 2) > 0).sum() == 3


def test_batched_markov_rows_follow_their_own_chain():
    """tests/test_batch_engine.py:226-238 of the reference, on the oracle's sequential rule:
    a bias that strongly favours prev+1 makes each row walk its own chain."""
    V = 5

    def step_bias(prev):
        return (torch.arange(V) == (prev + 1) % V).float() * 100.0

    def sample_block(base, first):
        out, prev = [], first
        for i in range(base.shape[0]):
            prev = int((base[i] + step_bias(prev)).argmax())
            out.append(prev)
        return out

    assert [sample_block(torch.zeros(2, V), f) for f in (0, 2)] == [[1, 2], [3, 4]]


def test_quantizer_and_dequant_bound():
    w = torch.randn(64, 256) * 0.02
    qt = quantize_w8g64(w)
    err = (qt.dequant() - w).abs()
    step = qt.scales.float().repeat_interleave(64, 1)
    # rounding to the nearest level plus the bf16 rounding of scale/bias
    assert (err <= 0.5 * step + 2 ** -8 * w.abs() + 2 ** -8 * step * 255 + 1e-7).all()
    assert qt.q.dtype == torch.uint8 and qt.scales.shape == (64, 4)


def test_kv8_quantizer_levels():
    x = torch.randn(3, 7, 128)
    d = oq.quantize_kv(x)
    rng = (x.reshape(3, 7, 2, 64).amax(-1) - x.reshape(3, 7, 2, 64).amin(-1))
    assert ((d - x).abs().reshape(3, 7, 2, 64) <= rng[..., None] / 255 * 0.51 + 2e-2 * x.abs().reshape(3, 7, 2, 64).amax(-1, keepdim=True)).all()
