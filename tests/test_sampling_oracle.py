"""CPU checks of the sampling oracle (no GPU).

- Philox4x32-10 against the published known-answer vectors of the Random123 distribution.
- The bit-exact restatement of the device sampler (oracle.sampling.*_exact) against the
  direct restatement of truncate_probs (src/mlx_dspark/sampling.py:18-44): same kept set and
  probabilities within the 2^-40 weight resolution (tolerance 1e-6 absolute).
- Losslessness of the exact acceptance, mirroring the reference's
  test_topp_speculative_sampling_is_lossless (tests/test_generate_helpers.py:145-170): the
  committed token is distributed as truncate(softmax(target / T)) whatever the draft q.
"""
import numpy as np
import pytest
import torch

from oracle import sampling as S


def test_philox_known_answers():
    assert S.philox4x32_10((0, 0, 0, 0), (0, 0)) == (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)
    assert S.philox4x32_10((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2) == (
        0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)
    assert S.philox4x32_10((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344),
                           (0xA4093822, 0x299F31D0)) == (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)


CASES = [(1.0, 1.0, 0), (1.0, 0.95, 50), (0.7, 1.0, 3), (1.0, 0.9, 0), (1.3, 0.8, 1000),
         (0.6, 0.5, 20)]


@pytest.mark.parametrize("T,top_p,top_k", CASES)
def test_exact_truncation_matches_truncate_probs(T, top_p, top_k):
    g = torch.Generator().manual_seed(int(T * 100) + top_k)
    V = 32768
    row = (torch.randn(V, generator=g) * 2.5).to(torch.bfloat16)
    kept, _ = S.truncated_weights(S._row_bits(row), T, 0, top_p, top_k)
    p = torch.from_numpy(S.probs_of(kept).astype(np.float64))
    x = (row.float() / float(S.bf16_scalar(T))).to(torch.bfloat16).double()   # bf16(l / bf16(T))
    ref = S.truncate_probs(torch.softmax(x, -1)[None], top_p, top_k)[0]
    assert torch.equal(p > 0, ref > 0)
    assert float((p - ref).abs().max()) < 1e-6


def test_exact_truncation_keeps_ties():
    row = torch.zeros(1000, dtype=torch.bfloat16)
    row[:10] = 3.0
    kept, _ = S.truncated_weights(S._row_bits(row), 1.0, 0, 1.0, 5)   # the 5th largest ties 10 ways
    assert int((kept > 0).sum()) == 10
    kept, _ = S.truncated_weights(S._row_bits(row), 1.0, 0, 1.0, 11)  # 11th largest = 0: all kept
    assert int((kept > 0).sum()) == 1000


def test_exact_sampler_distribution():
    """Draws of sample_row_exact over many counters follow the truncated distribution."""
    V = 6
    row = torch.tensor([2.0, 1.0, 0.5, 0.0, -1.0, -2.0]).to(torch.bfloat16)
    kept, _ = S.truncated_weights(S._row_bits(row), 1.0, 0, 0.8, 0)
    exp = S.probs_of(kept)
    counts = np.zeros(V)
    for i in range(20000):
        tok, _ = S.sample_row_exact(row, 1.0, 0, 0.8, 0, 1234, i, 0, 2)
        counts[tok] += 1
    assert np.abs(counts / counts.sum() - exp).max() < 0.02


@pytest.mark.parametrize("T,top_p,top_k", [(1.0, 1.0, 0), (1.0, 0.8, 0), (0.7, 1.0, 3)])
def test_exact_accept_is_lossless(T, top_p, top_k):
    V = 6
    target = torch.tensor([2.0, 1.0, 0.5, 0.0, -1.0, -2.0]).to(torch.bfloat16)
    qlog = torch.tensor([-2.0, -1.0, 0.0, 0.5, 1.0, 2.0]).to(torch.bfloat16)
    v = torch.stack([target, target])
    kept_t, _ = S.truncated_weights(S._row_bits(target), T, 0, top_p, top_k)
    exp = S.probs_of(kept_t)
    counts = np.zeros(V)
    N = 20000
    for i in range(N):
        x, q = S.sample_row_exact(qlog, 1.0, 0, 1.0, 0, 7, i, 0, 1)
        n, repl, _, _ = S.accept_sample_exact(v, [0, x], q[None], T, 0, top_p, top_k, 7, i)
        counts[x if n == 1 else repl] += 1
    assert np.abs(counts / N - exp).max() < 0.02, (counts / N, exp)
