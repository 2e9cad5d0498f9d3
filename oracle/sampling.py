"""Oracle top-k / top-p truncation and speculative-sampling acceptance (CPU).
TEST INFRASTRUCTURE ONLY.

truncate_probs follows src/mlx_dspark/sampling.py:18-44 (top-k keeps p >= kth largest,
ties kept; nucleus keeps p >= cutoff where cutoff is the smallest sorted value whose
exclusive prefix mass is < top_p; renormalise by max(sum, 1e-12)).
spec_sample_accept follows src/mlx_dspark/generate.py:659-688 (accept u < min(1, p/max(q,
1e-9)); first reject resamples from norm(max(p - q, 0)); all accepted -> bonus from p[L]).
The reference draws from mx.random; here a torch.Generator stands in (parity is
distributional, not bit-exact).
"""
from __future__ import annotations

import torch


def truncate_probs(probs: torch.Tensor, top_p: float = 1.0, top_k: int = 0) -> torch.Tensor:
    top_p = 1.0 if top_p is None else float(top_p)
    top_k = 0 if not top_k else int(top_k)
    if top_p >= 1.0 and top_k <= 0:
        return probs
    p = probs
    v = p.shape[-1]
    if 0 < top_k < v:
        kth = torch.sort(p, dim=-1).values[..., v - top_k][..., None]
        p = torch.where(p >= kth, p, torch.zeros_like(p))
    if top_p < 1.0:
        sd = torch.sort(p, dim=-1, descending=True).values
        csum = torch.cumsum(sd, dim=-1)
        in_nucleus = (csum - sd) < top_p
        cutoff = torch.where(in_nucleus, sd, torch.full_like(sd, float("inf"))).amin(-1, keepdim=True)
        p = torch.where(p >= cutoff, p, torch.zeros_like(p))
    return p / torch.clamp(p.sum(-1, keepdim=True), min=1e-12)


def target_probs(v_logits: torch.Tensor, temperature: float, top_p=1.0, top_k=0):
    return truncate_probs(torch.softmax(v_logits.float() / temperature, dim=-1), top_p, top_k)


def spec_sample_accept(v_logits, draft, q_probs, temperature, top_p=1.0, top_k=0,
                       gen: torch.Generator | None = None):
    """Returns (n_accepted, replacement_token)."""
    L = len(draft)
    p = target_probs(v_logits, temperature, top_p, top_k)
    idx = torch.as_tensor(draft, dtype=torch.long)
    rows = torch.arange(L)
    pd = p[rows, idx]
    qd = q_probs[rows, idx]
    u = torch.rand(L, generator=gen)
    acc = u < torch.clamp(pd / torch.clamp(qd, min=1e-9), max=1.0)
    n = int(torch.cumprod(acc.to(torch.int64), 0).sum())
    if n < L:
        resid = torch.clamp(p[n] - q_probs[n], min=0.0)
        resid = resid / torch.clamp(resid.sum(), min=1e-9)
        repl = int(torch.multinomial(resid, 1, generator=gen))
    else:
        repl = int(torch.multinomial(p[L], 1, generator=gen))
    return n, repl


def batch_mask(offsets, T):
    """build_batch_mask (src/mlx_dspark/batch_engine.py:170-178): [B, 1, T, max+T] bool,
    row b query i attends column j iff j <= offsets[b] + i."""
    off = torch.as_tensor(offsets)[:, None, None, None]
    L = max(offsets) + T
    i = torch.arange(T)[None, None, :, None]
    j = torch.arange(L)[None, None, None, :]
    return j <= off + i


def ctx_block_mask(lens, k):
    """_ctx_block_mask (src/mlx_dspark/batch_engine.py:401-411): [B, 1, k, Lmax+k]."""
    B = len(lens)
    Lmax = max(lens)
    la = torch.as_tensor(lens)[:, None, None, None]
    j = torch.arange(Lmax + k)[None, None, None, :]
    m = (j >= Lmax) | (j < la)
    return m.expand(B, 1, k, Lmax + k)
