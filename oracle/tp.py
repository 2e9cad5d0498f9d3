"""Oracle of the tensor-parallel decomposition (CPU). TEST INFRASTRUCTURE ONLY.

TPRef runs one rank's share of the Qwen3 forward of Qwen3Ref (the restatement of
src/mlx_dspark/target.py:58-75 and the mlx-lm qwen3 layer) on sharded weights: the o_proj and
down_proj products stay fp32 partials, are summed across ranks by `all_reduce`, and the
residual rounds once, bf16(h + bf16(sum)) — the rounding point of the single-device layer.
The head yields this rank's vocabulary slice of the logits.
"""
from __future__ import annotations

import torch

from .qwen3 import F32, Qwen3Ref, bf, rms_norm, rope, sdpa, silu


class TPRef(Qwen3Ref):
    def __init__(self, shard_w, all_reduce, rnd: bool = True):
        super().__init__(shard_w, rnd)
        self.all_reduce = all_reduce

    def _partial(self, x, qt):
        key = id(qt)
        if key not in self._deq:
            self._deq[key] = qt.dequant().t().contiguous()
        p = x.to(F32) @ self._deq[key]
        self.all_reduce(p)
        return p

    def layer(self, i, h, cache):
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
        mask = torch.arange(K.shape[1])[None, :] <= (off + torch.arange(T))[:, None]
        a = sdpa(q, K, V, c.head_dim ** -0.5, mask, self.rnd).transpose(0, 1).reshape(T, -1)
        h = bf(h + bf(self._partial(a, L.wo), self.rnd), self.rnd)
        x = rms_norm(h, L.post_ln, c.rms_norm_eps, self.rnd)
        act = bf(bf(silu(self._lin(x, L.gate)), self.rnd) * self._lin(x, L.up), self.rnd)
        return bf(h + bf(self._partial(act, L.down), self.rnd), self.rnd)


def merge_argmax(vals, idx):
    """Vocabulary-parallel argmax: per row the largest shard maximum, ties to the smallest
    global index (mx.argmax's first-index rule over the whole row)."""
    out = []
    for r in range(len(vals[0])):
        best = max(range(len(vals)), key=lambda s: (vals[s][r], -idx[s][r]))
        out.append(int(idx[best][r]))
    return out
