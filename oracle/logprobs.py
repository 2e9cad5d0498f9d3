"""CPU restatement of the per-token logprobs (test infrastructure: only tests/ import this).

_logprobs_for_block (src/mlx_dspark/generate.py:149-176): the raw float32 log-softmax of each
verify row, the committed token's entry, and with top_k > 0 the row's min(top_k, V) largest
entries in descending order. MLX's argsort does not promise an order among equal values; this
restatement (and the CUDA kernel) orders them by smaller index, as a stable sort does.
"""
from __future__ import annotations

import numpy as np


def log_softmax_f32(rows) -> np.ndarray:
    """x - max(x) - log(sum(exp(x - max(x)))) in float32 (generate.py:155-157)."""
    x = np.asarray(rows, dtype=np.float32)
    m = x.max(axis=-1, keepdims=True)
    s = np.exp(x - m).sum(axis=-1, keepdims=True, dtype=np.float32)
    return (x - m) - np.log(s)


def logprobs_for_block(rows, token_ids, top_k: int) -> list[dict]:
    """Entries {token_id, logprob[, top]} of the P rows and their committed tokens
    (generate.py:149-176)."""
    logp = log_softmax_f32(rows)
    P = len(token_ids)
    out = []
    idx = vals = None
    if top_k > 0:
        kth = min(top_k, logp.shape[-1])
        idx = np.argsort(-logp[:P], axis=-1, kind="stable")[:, :kth]
        vals = np.take_along_axis(logp[:P], idx, axis=-1)
    for i in range(P):
        e = {"token_id": int(token_ids[i]), "logprob": float(logp[i, int(token_ids[i])])}
        if idx is not None:
            e["top"] = [(int(t), float(v)) for t, v in zip(idx[i], vals[i])]
        out.append(e)
    return out
