"""Oracle presence / frequency penalties (CPU). TEST INFRASTRUCTURE ONLY.

Restates _Penalizer (src/mlx_dspark/generate.py:179-228) with the arithmetic of the penalty
dtype: in bf16, every MLX operation rounds to bf16 and a Python scalar operand is first cast to
bf16 (MLX's weak scalar typing); in float32 the same steps round to float32.
"""
from __future__ import annotations

import torch


class Penalizer:
    def __init__(self, presence: float = 0.0, frequency: float = 0.0):
        self.presence = float(presence or 0.0)
        self.frequency = float(frequency or 0.0)
        self.active = bool(self.presence or self.frequency)
        self.counts: dict[int, int] = {}

    def add(self, tokens) -> None:
        if not self.active:
            return
        for t in tokens:
            t = int(t)
            self.counts[t] = self.counts.get(t, 0) + 1

    def block_penalty(self, vocab: int, draft_prefix, dtype=torch.bfloat16) -> torch.Tensor:
        """[len(draft_prefix) + 1, vocab] penalty rows (generate.py:202-222)."""
        r = lambda x: torch.as_tensor(x, dtype=torch.float32).to(dtype)  # noqa: E731
        base = torch.zeros(vocab, dtype=dtype)
        if self.counts:
            ids = torch.tensor(list(self.counts.keys()))
            cs = r(list(self.counts.values()))
            f = (r(self.frequency).float() * cs.float()).to(dtype)
            base[ids] = (r(self.presence).float() + f.float()).to(dtype)
        rows = [base]
        extra = dict(self.counts)
        for d in draft_prefix:
            d = int(d)
            inc = self.frequency + (self.presence if extra.get(d, 0) == 0 else 0.0)
            nxt = rows[-1].clone()
            nxt[d] = (nxt[d].float() + r(inc).float()).to(dtype)
            rows.append(nxt)
            extra[d] = extra.get(d, 0) + 1
        return torch.stack(rows)

    def apply(self, v_logits_rows: torch.Tensor, draft_prefix) -> torch.Tensor:
        if not self.active:
            return v_logits_rows
        pen = self.block_penalty(v_logits_rows.shape[-1], draft_prefix, v_logits_rows.dtype)
        return (v_logits_rows.float() - pen.float()).to(v_logits_rows.dtype)
