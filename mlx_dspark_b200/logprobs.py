"""Per-token logprobs of the committed tokens (GenResult.logprobs; generate.py:149-176).

Each entry is {"token_id", "logprob"} plus, when top entries are requested, "top": the
(id, logprob) pairs of the row's largest entries in descending order. The values are the
target's raw log-softmax at the committed verify positions (before penalties or temperature),
computed on the device by dspark_logprobs and read back with the round's plan.
"""
from __future__ import annotations

import torch

from . import ops


class LogprobRows:
    """Device outputs and pinned host mirrors for up to `rows_max` rows of one decode.

    With `raw` the caller snapshots each round's logits before penalties change them in place
    (snapshot()); the logprobs are then read from the snapshot."""

    def __init__(self, device, rows_max: int, top_k: int, vocab_size: int, raw: bool = False):
        top_k = int(top_k)
        if top_k < 0:
            raise ValueError(f"logprobs must be >= 0, got {top_k}")
        if top_k > 1024:
            raise ValueError(f"logprobs top entries are limited to 1024 on this build, got {top_k}")
        self.rows_max, self.top_k, self.V = rows_max, top_k, vocab_size
        self.k_out = min(top_k, vocab_size)
        self.logp = torch.zeros(rows_max, dtype=torch.float32, device=device)
        self.logp_host = torch.zeros(rows_max, dtype=torch.float32, pin_memory=True)
        self.top_ids = self.top_vals = self.top_ids_host = self.top_vals_host = None
        if top_k > 0:
            self.top_ids = torch.zeros(rows_max, top_k, dtype=torch.int32, device=device)
            self.top_vals = torch.zeros(rows_max, top_k, dtype=torch.float32, device=device)
            self.top_ids_host = torch.zeros(rows_max, top_k, dtype=torch.int32, pin_memory=True)
            self.top_vals_host = torch.zeros(rows_max, top_k, dtype=torch.float32, pin_memory=True)
        self.raw = (torch.zeros(rows_max, vocab_size, dtype=torch.bfloat16, device=device)
                    if raw else None)

    def snapshot(self, logits: torch.Tensor, rows: int) -> None:
        """Keep the raw logits of `rows` rows (before penalties are applied in place)."""
        self.raw[:rows].copy_(logits[:rows, :self.V])

    def launch(self, logits: torch.Tensor, rows: int, ids: torch.Tensor, ids_ld: int,
               T: int, use_snapshot: bool = True) -> None:
        """Compute `rows` rows (from the snapshot when there is one and use_snapshot) and queue
        their copies to the host on the current stream."""
        if rows > self.rows_max:
            raise ValueError(f"{rows} logprob rows > {self.rows_max}")
        src = self.raw if (use_snapshot and self.raw is not None) else logits
        ops.logprobs(src, rows, ids, ids_ld, T, self.top_k, self.logp, self.top_ids,
                     self.top_vals, V=self.V)
        self.logp_host[:rows].copy_(self.logp[:rows], non_blocking=True)
        if self.top_k > 0:
            self.top_ids_host[:rows].copy_(self.top_ids[:rows], non_blocking=True)
            self.top_vals_host[:rows].copy_(self.top_vals[:rows], non_blocking=True)

    def entries(self, tokens: list[int], first_row: int = 0) -> list[dict]:
        """Entries of rows first_row.. for the committed `tokens` (after the copies finished)."""
        n = len(tokens)
        lp = self.logp_host[first_row:first_row + n].tolist()
        out = []
        if self.top_k > 0:
            ids = self.top_ids_host[first_row:first_row + n, :self.k_out].tolist()
            vals = self.top_vals_host[first_row:first_row + n, :self.k_out].tolist()
        for i, tok in enumerate(tokens):
            e = {"token_id": int(tok), "logprob": float(lp[i])}
            if self.top_k > 0:
                e["top"] = [(int(t), float(v)) for t, v in zip(ids[i], vals[i])]
            out.append(e)
        return out
