"""Known answers of the CPU logprobs restatement (oracle/logprobs.py, generate.py:149-176)."""
import numpy as np
import torch

from oracle.logprobs import log_softmax_f32, logprobs_for_block


def test_uniform_row():
    V = 1000
    e = logprobs_for_block(np.zeros((1, V), np.float32), [17], 3)[0]
    assert e["token_id"] == 17
    assert abs(e["logprob"] + np.log(V)) < 1e-5
    assert [t for t, _ in e["top"]] == [0, 1, 2]          # equal values: smaller index first
    assert all(abs(v + np.log(V)) < 1e-5 for _, v in e["top"])


def test_one_hot_row_and_chosen_only():
    x = np.zeros((2, 64), np.float32)
    x[0, 5] = 100.0
    x[1, 9] = 100.0
    es = logprobs_for_block(x, [5, 3], 0)
    assert "top" not in es[0]
    assert abs(es[0]["logprob"]) < 1e-6
    assert es[1]["logprob"] < -99.0


def test_ties_and_top_k_past_vocab():
    x = np.array([[1.0, 3.0, 3.0, 2.0, 3.0]], np.float32)
    e = logprobs_for_block(x, [0], 2)[0]
    assert [t for t, _ in e["top"]] == [1, 2]
    e = logprobs_for_block(x, [0], 9)[0]
    assert [t for t, _ in e["top"]] == [1, 2, 4, 3, 0]     # min(top_k, V) entries


def test_matches_float64_log_softmax():
    g = torch.Generator().manual_seed(0)
    x = (torch.randn(4, 151936, generator=g) * 3).to(torch.bfloat16).float()
    got = log_softmax_f32(x.numpy())
    want = torch.log_softmax(x.double(), -1).numpy()
    assert np.abs(got - want).max() < 2e-5


def test_confidence_truncation_rule():
    """generate.py:875-887: keep while the running survival product stays >= threshold,
    always at least one drafted token."""
    from oracle.dspark import truncate_by_confidence
    d = [11, 12, 13, 14]
    assert truncate_by_confidence(d, [0.9, 0.8, 0.5, 0.9], 0.5) == [11, 12]   # 0.9, 0.72, 0.36
    assert truncate_by_confidence(d, [0.9, 0.8, 0.5, 0.9], 0.3) == [11, 12, 13, 14]
    assert truncate_by_confidence(d, [0.4, 1.0, 1.0, 1.0], 0.5) == [11]       # none kept -> one
    assert truncate_by_confidence(d, [1.0, 1.0, 1.0, 1.0], 1.0) == d
