"""Oracle Qwen3 target forward with hidden-state tap and KV cache (CPU, fp32 math).

Follows src/mlx_dspark/target.py:58-75 (embed -> layers -> tap -> norm -> head, tied head
via embed_tokens.as_linear at :71-72) and the mlx-lm qwen3 layer it calls (restated from
the public Qwen3 architecture: pre-RMSNorm, per-head q/k RMSNorm before rotate-half RoPE
with theta 1e6, GQA SDPA with scale head_dim^-0.5 and the causal mask of
create_attention_mask, SwiGLU MLP, residual adds). KV cache semantics follow mlx-lm
KVCache / QuantizedKVCache(64, 8) as used at target.py:36-48: append on update, trim by
offset arithmetic. TEST INFRASTRUCTURE ONLY.
"""
from __future__ import annotations

import math

import torch

F32 = torch.float32


def bf(x: torch.Tensor, rnd: bool = True) -> torch.Tensor:
    """Round to bf16 and back (the storage rounding of a bf16 MLX array)."""
    return x.to(torch.bfloat16).to(F32) if rnd else x


def linear(x: torch.Tensor, wq, rnd: bool = True) -> torch.Tensor:
    """Affine W8 g64 QuantizedLinear: x[.., K] @ dequant(W)[N, K]^T, fp32 accumulation."""
    return bf(x.to(F32) @ wq.dequant().t(), rnd)


def rms_norm(x, w, eps, rnd=True):
    """mx.fast.rms_norm: x * rsqrt(mean(x^2) + eps) * w, fp32 math, one rounding."""
    x = x.to(F32)
    r = torch.rsqrt(x.pow(2).mean(dim=-1, keepdim=True) + eps)
    return bf(x * r * w.to(F32), rnd)


def inv_freq(head_dim: int, theta: float) -> torch.Tensor:
    """theta^(-2i/d), i < d/2 (non-traditional RoPE frequencies), fp32."""
    i = torch.arange(0, head_dim, 2, dtype=torch.float64)
    return (theta ** (-i / head_dim)).to(F32)


def rope(x, positions, freqs, rnd=True):
    """Rotate-half RoPE. x [..., T, hd] (heads leading), positions [T] (int)."""
    ang = positions.to(F32)[:, None] * freqs[None, :]  # fp32 angle, like the kernel
    cos, sin = torch.cos(ang), torch.sin(ang)
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return bf(torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1), rnd)


def sdpa(q, k, v, scale, mask=None, rnd=True):
    """mx.fast.scaled_dot_product_attention with GQA broadcast: q [Hq, T, d], k/v [Hkv, S, d];
    mask [T, S] bool (True = attend) or None. fp32 scores/softmax, output rounded."""
    Hq, Hkv = q.shape[0], k.shape[0]
    rep = Hq // Hkv
    k = k.repeat_interleave(rep, dim=0)
    v = v.repeat_interleave(rep, dim=0)
    s = (q.to(F32) @ k.to(F32).transpose(-1, -2)) * scale
    if mask is not None:
        s = s.masked_fill(~mask[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return bf(p @ v.to(F32), rnd)


def silu(x):
    return x / (1.0 + torch.exp(-x))


def _round_half_away(v: torch.Tensor) -> torch.Tensor:
    """Round to nearest with halves away from zero (C roundf / Metal round), exactly."""
    t = torch.trunc(v)
    return t + torch.where((v - t).abs() >= 0.5, torch.sign(v), torch.zeros_like(v))


def quantize_kv(x: torch.Tensor):
    """Affine 8-bit group-64 along head_dim with the rule of MLX's affine quantizer, which
    QuantizedKVCache(64, 8) applies (src/mlx_dspark/target.py:44-46 -> mx.quantize), in fp32:
    scale = max((max-min)/255, 1e-7), negated unless |min| > |max|; the larger-magnitude edge
    is made exact: q0 = round(edge/scale), scale = edge/q0, bias = edge (bias 0, scale kept,
    when q0 == 0); q = min(round((x-bias)/scale), 255), rounding halves away from zero; scale
    and bias stored as bf16. Returns the dequantized values bf16(scale_bf16 * q + bias_bf16)."""
    *lead, d = x.shape
    g = x.to(F32).reshape(*lead, d // 64, 64)
    mn, mx = g.amin(-1, keepdim=True), g.amax(-1, keepdim=True)
    sc = torch.clamp((mx - mn) / 255.0, min=1e-7)
    neg_edge = mn.abs() > mx.abs()
    sc = torch.where(neg_edge, sc, -sc)
    edge = torch.where(neg_edge, mn, mx)
    q0 = _round_half_away(edge / sc)
    at_zero = q0 == 0
    sc = torch.where(at_zero, sc, edge / torch.where(at_zero, torch.ones_like(q0), q0))
    bi = torch.where(at_zero, torch.zeros_like(edge), edge)
    q = _round_half_away((g - bi) / sc).clamp(0, 255)
    s = sc.to(torch.bfloat16).to(F32)
    b = bi.to(torch.bfloat16).to(F32)
    return bf(s * q + b).reshape(*lead, d)


class KVCacheRef:
    """mlx-lm KVCache duck type for one layer: keys/values [Hkv, S, d] (fp32 holding bf16)."""

    def __init__(self, kv8: bool = False):
        self.keys = None
        self.values = None
        self.offset = 0
        self.kv8 = kv8

    def update_and_fetch(self, k, v):
        if self.kv8:
            k, v = quantize_kv(k), quantize_kv(v)
        if self.keys is None:
            self.keys, self.values = k, v
        else:
            self.keys = torch.cat([self.keys[:, : self.offset], k], dim=1)
            self.values = torch.cat([self.values[:, : self.offset], v], dim=1)
        self.offset += k.shape[1]
        return self.keys[:, : self.offset], self.values[:, : self.offset]

    def trim(self, n: int) -> int:
        n = min(self.offset, n)
        self.offset -= n
        return n


class Qwen3Ref:
    """Oracle target. ``w`` is a mlx_dspark_b200.weights.TargetWeights on the CPU."""

    def __init__(self, w, rnd: bool = True):
        self.w = w
        self.cfg = w.cfg
        self.rnd = rnd
        self.freqs = inv_freq(self.cfg.head_dim, self.cfg.rope_theta)
        # dequantize once (fp32) — the oracle trades memory for speed on small configs
        self._deq = {}

    def _lin(self, x, qt):
        key = id(qt)
        if key not in self._deq:
            self._deq[key] = qt.dequant().t().contiguous()
        return bf(x.to(F32) @ self._deq[key], self.rnd)

    def make_cache(self, kv8: bool = False):
        return [KVCacheRef(kv8) for _ in range(self.cfg.num_hidden_layers)]

    def embed(self, ids: torch.Tensor) -> torch.Tensor:
        e = self.w.embed
        return bf(e.scales.to(F32).repeat_interleave(64, 1)[ids] * e.q[ids].to(F32)
                  + e.biases.to(F32).repeat_interleave(64, 1)[ids], self.rnd)

    def layer(self, i, h, cache):
        """One decoder layer over T new tokens at positions cache.offset..; h [T, H]."""
        c, L = self.cfg, self.w.layers[i]
        T = h.shape[0]
        x = rms_norm(h, L.input_ln, c.rms_norm_eps, self.rnd)
        q = self._lin(x, L.wq).reshape(T, c.num_attention_heads, c.head_dim).transpose(0, 1)
        k = self._lin(x, L.wk).reshape(T, c.num_key_value_heads, c.head_dim).transpose(0, 1)
        v = self._lin(x, L.wv).reshape(T, c.num_key_value_heads, c.head_dim).transpose(0, 1)
        q = rms_norm(q, L.q_norm, c.rms_norm_eps, self.rnd)
        k = rms_norm(k, L.k_norm, c.rms_norm_eps, self.rnd)
        off = cache.offset
        pos = torch.arange(off, off + T)
        q = rope(q, pos, self.freqs, self.rnd)
        k = rope(k, pos, self.freqs, self.rnd)
        K, V = cache.update_and_fetch(k, v)
        S = K.shape[1]
        # create_attention_mask: query t (absolute off+t) sees keys j <= off+t
        mask = torch.arange(S)[None, :] <= (off + torch.arange(T))[:, None]
        a = sdpa(q, K, V, c.head_dim ** -0.5, mask, self.rnd)
        a = a.transpose(0, 1).reshape(T, -1)
        h = bf(h + self._lin(a, L.wo), self.rnd)
        x = rms_norm(h, L.post_ln, c.rms_norm_eps, self.rnd)
        g = self._lin(x, L.gate)
        u = self._lin(x, L.up)
        act = bf(bf(silu(g), self.rnd) * u, self.rnd)
        return bf(h + self._lin(act, L.down), self.rnd)

    def run(self, ids, cache, tap=()):
        """ids [T] -> (logits [T, V], fused [T, n_tap*H]); target.py:58-75."""
        ids = torch.as_tensor(ids, dtype=torch.long).reshape(-1)
        h = self.embed(ids)
        cap = []
        tapset = set(tap)
        for i in range(self.cfg.num_hidden_layers):
            h = self.layer(i, h, cache[i])
            if i in tapset:
                cap.append(h)
        hn = rms_norm(h, self.w.norm, self.cfg.rms_norm_eps, self.rnd)
        logits = self._lin(hn, self.w.head)
        fused = torch.cat(cap, dim=-1) if cap else None
        return logits, fused

    def plain(self, ids, cache):
        return self.run(ids, cache, ())[0]


def prefill(model: Qwen3Ref, ids, cache, tap=(), chunk: int = 2048):
    """Chunked prefill (generate.py:619-656): returns the last chunk's logits and all fused."""
    logits, parts = None, []
    for i in range(0, len(ids), chunk):
        logits, fused = model.run(ids[i:i + chunk], cache, tap)
        if fused is not None:
            parts.append(fused)
    return logits, (torch.cat(parts, 0) if parts else None)


def top2_gap(row: torch.Tensor) -> float:
    v = torch.topk(row.to(F32), 2).values
    return float(v[0] - v[1])


__all__ = ["Qwen3Ref", "KVCacheRef", "bf", "linear", "rms_norm", "rope", "sdpa", "inv_freq",
           "quantize_kv", "prefill", "top2_gap", "silu", "math"]
