"""The penalty oracle against the reference's own penalty tests (tests/test_penalties.py:14-57,
restated here on the same inputs with float32 rows, as the reference runs them)."""
import torch

from oracle.penalties import Penalizer


def test_inactive_is_noop():
    p = Penalizer(0.0, 0.0)
    assert not p.active
    logits = torch.randn(3, 8)
    assert p.apply(logits, [1, 2]) is logits


def test_base_penalty_presence_and_frequency():
    p = Penalizer(presence=1.0, frequency=0.5)
    p.add([5, 5, 2])
    row = p.block_penalty(8, [], torch.float32)[0].tolist()
    assert abs(row[5] - 2.0) < 1e-6 and abs(row[2] - 1.5) < 1e-6
    assert row[0] == 0.0 and row[3] == 0.0


def test_draft_prefix_new_token_gets_presence_then_frequency():
    p = Penalizer(presence=1.0, frequency=0.5)
    pen = p.block_penalty(8, [3, 3], torch.float32)
    assert pen.shape == (3, 8)
    assert [float(pen[i][3]) for i in range(3)] == [0.0, 1.5, 2.0]


def test_draft_prefix_token_already_in_base_only_frequency():
    p = Penalizer(presence=1.0, frequency=0.5)
    p.add([7])
    pen = p.block_penalty(8, [7], torch.float32)
    assert [float(pen[i][7]) for i in range(2)] == [1.5, 2.0]


def test_apply_subtracts_penalty():
    p = Penalizer(presence=2.0, frequency=0.0)
    p.add([1])
    out = p.apply(torch.zeros(2, 4), [3])
    assert out[0].tolist() == [0.0, -2.0, 0.0, 0.0]
    assert out[1].tolist() == [0.0, -2.0, 0.0, -2.0]


def test_bf16_rows_round_each_step():
    p = Penalizer(presence=0.3, frequency=0.7)
    p.add([4] * 300)                      # 300 is not a bf16 integer: bf16(300) = 300 (exact),
    p.add([5] * 257)                      # bf16(257) = 256
    pen = p.block_penalty(8, [5], torch.bfloat16)
    f, pr = torch.tensor(0.7).bfloat16().float(), torch.tensor(0.3).bfloat16().float()
    assert float(pen[0][5]) == float((pr + (f * 256.0).bfloat16().float()).bfloat16())
