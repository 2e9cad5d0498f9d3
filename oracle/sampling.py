"""Oracle top-k / top-p truncation and speculative-sampling acceptance (CPU).
TEST INFRASTRUCTURE ONLY.

truncate_probs follows src/mlx_dspark/sampling.py:18-44 (top-k keeps p >= kth largest,
ties kept; nucleus keeps p >= cutoff where cutoff is the smallest sorted value whose
exclusive prefix mass is < top_p; renormalise by max(sum, 1e-12)).
spec_sample_accept follows src/mlx_dspark/generate.py:659-688 (accept u < min(1, p/max(q,
1e-9)); first reject resamples from norm(max(p - q, 0)); all accepted -> bonus from p[L]).
The reference draws from mx.random; here a torch.Generator stands in (parity is
distributional, not bit-exact).

The second half of this file (philox4x32_10 .. accept_sample_exact) restates the device
sampler's arithmetic step by step in numpy: the same truncation rules expressed on 16-bit keys
of the bf16 logits, 2^-40 fixed-point weights from the same exp2 polynomial (float32 multiply
and add rounded separately), and inverse-CDF draws from the same Philox4x32-10 words. Given the
same logits and {seed, offset} it returns the same tokens as the kernels, bit for bit, and its
truncated distribution matches truncate_probs above to within the 2^-40 weight resolution
(checked by tests/test_sampling_oracle.py).
"""
from __future__ import annotations

import numpy as np
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


# ------------------------------------------------------------------------------------------
# bit-exact restatement of the device sampler

_M0, _M1, _W0, _W1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85
_MASK32 = 0xFFFFFFFF


def philox4x32_10(ctr, key):
    """Philox4x32-10 (Salmon et al., SC 2011): ctr 4 x u32, key 2 x u32 -> 4 x u32."""
    c0, c1, c2, c3 = (int(v) & _MASK32 for v in ctr)
    k0, k1 = (int(v) & _MASK32 for v in key)
    for r in range(10):
        if r:
            k0 = (k0 + _W0) & _MASK32
            k1 = (k1 + _W1) & _MASK32
        p0 = _M0 * c0
        p1 = _M1 * c2
        c0, c1, c2, c3 = ((p1 >> 32) ^ c1 ^ k0) & _MASK32, p1 & _MASK32, \
            ((p0 >> 32) ^ c3 ^ k1) & _MASK32, p0 & _MASK32
    return c0, c1, c2, c3


def philox_words(seed, offset, row, stream):
    """The device's counter layout: {offset_lo, offset_hi, row, stream}, key {seed_lo, seed_hi}.
    Returns (u for the accept test, 64-bit draw word)."""
    x, _, z, w = philox4x32_10((offset & _MASK32, offset >> 32, row, stream),
                               (seed & _MASK32, seed >> 32))
    u = np.float32(x >> 8) * np.float32(1.0 / 16777216.0)
    return u, (z << 32) | w


def _bf16_bits_rne(x32: np.ndarray) -> np.ndarray:
    u = x32.astype(np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    r = np.where(nan, (u >> 16) | 0x40, r)
    return r.astype(np.uint16)


def bf16_scalar(v: float) -> np.float32:
    return (_bf16_bits_rne(np.array([v], dtype=np.float32)).astype(np.uint32) << 16).view(np.float32)[0]


def temperature_factor(temperature: float, temp_mode: int):
    """(factor, mode): mode 0 divides by bf16(T), 1 multiplies by bf16(1/T), 2 is identity."""
    tb = bf16_scalar(temperature if temp_mode == 0 else float(np.float32(1.0 / temperature)))
    return tb, (2 if tb == np.float32(1.0) else temp_mode)


def keys_of(bits: np.ndarray, tb, tmode) -> np.ndarray:
    """bf16 bit patterns -> order-preserving 16-bit keys of bf16(x / T) (or * 1/T)."""
    b = bits.astype(np.uint16)
    if tmode != 2:
        l32 = (b.astype(np.uint32) << 16).view(np.float32)
        x = (l32 / tb) if tmode == 0 else (l32 * tb)
        b = _bf16_bits_rne(x.astype(np.float32))
    b = np.where(b == 0x8000, 0, b).astype(np.uint32)
    return np.where(b & 0x8000, (~b) & 0xFFFF, b | 0x8000).astype(np.uint32)


def key_val(k: np.ndarray) -> np.ndarray:
    k = k.astype(np.uint32)
    b = np.where(k & 0x8000, k & 0x7FFF, (~k) & 0xFFFF).astype(np.uint32)
    return (b << 16).view(np.float32)


_C = [np.uint32(v).view(np.float32) for v in
      (0x3F800000, 0x3F317218, 0x3E75FDF0, 0x3D635847, 0x3C1D955B, 0x3AAEC3FF, 0x39218489,
       0x377FE5FE)]  # fp32(ln(2)^k / k!), k = 0..7
_LOG2E = np.uint32(0x3FB8AA3B).view(np.float32)


def wfix(keys: np.ndarray, m: np.float32) -> np.ndarray:
    """floor(2^40 * 2^((x - m) log2 e)) with the device's polynomial and rounding."""
    with np.errstate(invalid="ignore", over="ignore"):
        d = key_val(keys) - np.float32(m)
        t = (d * _LOG2E).astype(np.float32)
        ok = t >= np.float32(-45.0)
        t = np.where(ok, t, np.float32(0.0)).astype(np.float32)
        r = np.rint(t).astype(np.float32)
        f = (t - r).astype(np.float32)
        p = _C[7]
        for c in (_C[6], _C[5], _C[4], _C[3], _C[2], _C[1], _C[0]):
            p = ((p * f).astype(np.float32) + c).astype(np.float32)
        sc = np.ldexp(np.float32(1.0), (r.astype(np.int64) + 40)).astype(np.float32)
        w = (p * sc).astype(np.float32).astype(np.uint64)
    return np.where(ok, w, np.uint64(0)).astype(np.uint64)


def _draw(weights: np.ndarray, r64: int, V: int) -> int:
    S = int(weights.sum(dtype=np.uint64))
    if S == 0:
        return (r64 * V) >> 64
    target = (r64 * S) >> 64
    cum = np.cumsum(weights, dtype=np.uint64)
    return int(np.searchsorted(cum, np.uint64(target), side="right"))


def truncated_weights(bits: np.ndarray, temperature: float, temp_mode: int, top_p: float,
                      top_k: int):
    """Kept fixed-point weights of one row (zeros where cut) and the whole-row weight Z."""
    tb, tm = temperature_factor(temperature, temp_mode)
    keys = keys_of(bits, tb, tm)
    V = keys.shape[0]
    m = key_val(np.array([keys.max()], dtype=np.uint32))[0]
    w = wfix(keys, m)
    Z = int(w.sum(dtype=np.uint64))
    tk = 0
    if 0 < top_k < V:
        tk = int(np.sort(keys)[::-1][top_k - 1])
    thr_key = tk
    if top_p < 1.0:
        wk = np.where(keys >= tk, w, np.uint64(0))
        uk, inv = np.unique(keys, return_inverse=True)          # ascending distinct keys
        mass = np.zeros(uk.shape[0], dtype=np.uint64)
        np.add.at(mass, inv, wk)                                 # exact integer sums
        thr = float(top_p) * float(Z)
        above = 0
        tp = int(uk[-1])
        for j in range(uk.shape[0] - 1, -1, -1):               # descending keys
            if float(above) < thr:
                tp = int(uk[j])
            else:
                break
            above += int(mass[j])
        thr_key = max(tk, tp)
    kept = np.where(keys >= thr_key, w, np.uint64(0)).astype(np.uint64)
    return kept, Z


def probs_of(kept: np.ndarray) -> np.ndarray:
    S = int(kept.sum(dtype=np.uint64))
    if S == 0:
        return np.zeros(kept.shape[0], dtype=np.float32)
    inv = 1.0 / float(np.float64(np.uint64(S)))
    return (kept.astype(np.float64) * inv).astype(np.float32)


def _row_bits(row) -> np.ndarray:
    if isinstance(row, torch.Tensor):
        return row.detach().to(torch.bfloat16).cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
    return np.asarray(row, dtype=np.uint16)


def sample_row_exact(row, temperature, temp_mode, top_p, top_k, seed, offset, row_index, stream):
    """One draw of dspark_sample_rows: returns (token, q row as float32)."""
    bits = _row_bits(row)
    kept, _ = truncated_weights(bits, temperature, temp_mode, top_p, top_k)
    _, r64 = philox_words(seed, offset, row_index, stream)
    return _draw(kept, r64, bits.shape[0]), probs_of(kept)


def accept_sample_exact(v_logits, verify_ids, q_probs, temperature, temp_mode, top_p, top_k,
                        seed, offset, q_onehot=False):
    """dspark_accept_sample for one block: returns (n, replacement, flags, candidates)."""
    T = len(verify_ids)
    L = T - 1
    V = v_logits.shape[-1]
    flags, cands = [], []
    for i in range(T):
        bits = _row_bits(v_logits[i])
        kept, _ = truncated_weights(bits, temperature, temp_mode, top_p, top_k)
        p = probs_of(kept)
        u, r64 = philox_words(seed, offset, i, 0)
        if i < L:
            x = int(verify_ids[i + 1])
            if q_onehot:
                q = np.zeros(V, dtype=np.float32)
                if 0 <= x < V:
                    q[x] = 1.0
            else:
                q = np.asarray(q_probs[i], dtype=np.float32)
            pd = p[x] if 0 <= x < V else np.float32(0.0)
            qd = q[x] if 0 <= x < V else np.float32(0.0)
            ratio = np.float32(pd) / np.maximum(np.float32(qd), np.float32(1e-9))
            flags.append(bool(u < min(np.float32(1.0), np.float32(ratio))) and 0 <= x < V)
            d = (p - q).astype(np.float32)
            rw = np.where(d > 0, (d * np.float32(1099511627776.0)).astype(np.float32),
                          np.float32(0)).astype(np.uint64)
            cands.append(_draw(rw, r64, V))
        else:
            flags.append(False)
            cands.append(_draw(kept, r64, V))
    n = 0
    while n < L and flags[n]:
        n += 1
    return n, cands[n], flags, cands


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
