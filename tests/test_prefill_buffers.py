"""Prefill chunk buffers on the CPU: rows(T) views share storage with the full buffers, the
last-row logits buffer is one row unless every row's logits are kept, and the tap buffer
follows n_tap."""
import torch

from mlx_dspark_b200.config import TINY
from mlx_dspark_b200.target import PREFILL_CHUNK, PrefillBuffers


def test_rows_are_views_of_the_full_buffers():
    b = PrefillBuffers(TINY, 96, 3, "cpu")
    v = b.rows(40)
    assert v.T == 40 and b.T == b.cap == 96
    for f in ("ids", "h", "xn16", "qkv", "q", "attn16", "act16", "fused16"):
        full, part = getattr(b, f), getattr(v, f)
        assert part.shape[0] == 40 and part.data_ptr() == full.data_ptr()
        assert part.is_contiguous()
    assert v.logits.shape == (1, TINY.vocab_size) and v.logits.data_ptr() == b.logits.data_ptr()
    v.h.fill_(1.0)
    assert float(b.h[:40].sum()) == 40 * TINY.hidden_size and float(b.h[40:].abs().sum()) == 0
    assert v.fused16.shape[1] == 3 * TINY.hidden_size


def test_all_logits_and_no_taps():
    b = PrefillBuffers(TINY, 64, 0, "cpu", all_logits=True)
    assert b.fused16 is None and b.rows(10).fused16 is None
    assert b.logits.shape == (64, TINY.vocab_size) and b.rows(10).logits.shape[0] == 10
    assert PREFILL_CHUNK == 2048    # the reference's chunk (generate.py:613)
