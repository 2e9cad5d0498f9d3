"""Oracle DSpark drafter, greedy acceptance and decode loops (CPU). TEST INFRASTRUCTURE ONLY.

Drafter: src/mlx_dspark/model.py:48-320 (CtxCache append, DSparkAttention._kv /
update_ctx / attend, qwen 2-norm layer, VanillaMarkov, sample_block).
Greedy loops: speculative_generate's fused greedy path src/mlx_dspark/generate.py:806-961
(with lookup drafts off and no confidence head) and greedy_generate :373-465.
"""
from __future__ import annotations

import torch

from .qwen3 import F32, Qwen3Ref, bf, inv_freq, prefill, rms_norm, rope, sdpa, silu


class CtxCacheRef:
    """model.py:48-80 — per-layer context K/V, append-only (trim_to for prefix reuse)."""

    def __init__(self):
        self.k = None
        self.v = None

    def append(self, k, v):
        if self.k is None:
            self.k, self.v = k, v
        else:
            self.k = torch.cat([self.k, k], dim=1)
            self.v = torch.cat([self.v, v], dim=1)

    def trim_to(self, length):
        if self.k is not None and length < self.k.shape[1]:
            self.k, self.v = self.k[:, :length], self.v[:, :length]

    @property
    def length(self):
        return 0 if self.k is None else self.k.shape[1]


class DSparkRef:
    """Oracle drafter. ``w``: DSparkWeights (CPU); ``target_w``: TargetWeights for the shared
    embedding / head when the drafter config says so."""

    def __init__(self, w, target_w, rnd: bool = True):
        self.w, self.cfg, self.rnd = w, w.cfg, rnd
        self.embed_t = w.embed if w.embed is not None else target_w.embed
        self.head_t = w.lm_head if w.lm_head is not None else target_w.head
        self.freqs = inv_freq(self.cfg.head_dim, self.cfg.rope_theta)
        self._deq = {}

    def _lin(self, x, qt):
        if id(qt) not in self._deq:
            self._deq[id(qt)] = qt.dequant().t().contiguous()
        return bf(x.to(F32) @ self._deq[id(qt)], self.rnd)

    def make_ctx_cache(self):
        return [CtxCacheRef() for _ in self.w.layers]

    def embed(self, ids):
        e = self.embed_t
        ids = torch.as_tensor(ids, dtype=torch.long)
        return bf(e.scales.to(F32).repeat_interleave(64, 1)[ids] * e.q[ids].to(F32)
                  + e.biases.to(F32).repeat_interleave(64, 1)[ids], self.rnd)

    def _kv(self, L, x):
        """DSparkAttention._kv (model.py:113-124): K = k_norm(k_proj(x)), V = v_proj(x)."""
        c = self.cfg
        T = x.shape[0]
        k = self._lin(x, L.wk).reshape(T, c.num_key_value_heads, c.head_dim).transpose(0, 1)
        k = rms_norm(k, L.k_norm, c.rms_norm_eps, self.rnd)
        v = self._lin(x, L.wv).reshape(T, c.num_key_value_heads, c.head_dim).transpose(0, 1)
        return k, v

    def update_context(self, fused, ctx_offset, ctx_caches):
        """model.py:253-256 + update_ctx :126-128 (V is not roped)."""
        f = rms_norm(self._lin(fused, self.w.fc), self.w.hidden_norm, self.cfg.rms_norm_eps, self.rnd)
        pos = torch.arange(ctx_offset, ctx_offset + f.shape[0])
        for L, cache in zip(self.w.layers, ctx_caches):
            k, v = self._kv(L, f)
            cache.append(rope(k, pos, self.freqs, self.rnd), v)

    def attend(self, L, h, block_offset, cache):
        """model.py:130-156: Q from the block, K/V = [ctx; block], no mask."""
        c = self.cfg
        T = h.shape[0]
        q = self._lin(h, L.wq).reshape(T, c.num_attention_heads, c.head_dim).transpose(0, 1)
        pos = torch.arange(block_offset, block_offset + T)
        q = rope(rms_norm(q, L.q_norm, c.rms_norm_eps, self.rnd), pos, self.freqs, self.rnd)
        kb, vb = self._kv(L, h)
        kb = rope(kb, pos, self.freqs, self.rnd)
        K = kb if cache.k is None else torch.cat([cache.k, kb], dim=1)
        V = vb if cache.v is None else torch.cat([cache.v, vb], dim=1)
        a = sdpa(q, K, V, c.scaling, None, self.rnd)
        return self._lin(a.transpose(0, 1).reshape(T, -1), L.wo)

    def backbone(self, noise, block_offset, ctx_caches):
        """model.py:258-262 with the qwen 2-norm layer :185-194."""
        c = self.cfg
        h = noise
        for L, cache in zip(self.w.layers, ctx_caches):
            a = self.attend(L, rms_norm(h, L.input_ln, c.rms_norm_eps, self.rnd), block_offset, cache)
            h = bf(h + a, self.rnd)
            x = rms_norm(h, L.post_ln, c.rms_norm_eps, self.rnd)
            act = bf(bf(silu(self._lin(x, L.gate)), self.rnd) * self._lin(x, L.up), self.rnd)
            h = bf(h + self._lin(act, L.down), self.rnd)
        return rms_norm(h, self.w.norm, c.rms_norm_eps, self.rnd)

    def compute_logits(self, hidden):
        return self._lin(hidden, self.head_t)

    def step_bias(self, prev: int):
        """VanillaMarkov.step_bias (model.py:207-208): w2(w1[prev])."""
        w1, w2 = self.w.markov_w1, self.w.markov_w2
        e = bf(w1.scales[prev].to(F32).repeat_interleave(64) * w1.q[prev].to(F32)
               + w1.biases[prev].to(F32).repeat_interleave(64), self.rnd)
        return self._lin(e[None], w2)[0]

    def prev_embedding(self, prev: int):
        """VanillaMarkov.prev_embeddings (model.py:204-205): bf16(dequant w1[prev])."""
        w1 = self.w.markov_w1
        return bf(w1.scales[prev].to(F32).repeat_interleave(64) * w1.q[prev].to(F32)
                  + w1.biases[prev].to(F32).repeat_interleave(64), self.rnd)

    def confidence_logits(self, hidden, prev_tokens):
        """confidence_logits + ConfidenceHead (model.py:311-320, :211-217) over normalised block
        rows [cap, H]: bf16(w . [hidden_i, w1[prev_i]] + b), fp32 accumulation."""
        feats = hidden.to(F32)
        if self.cfg.confidence_head_with_markov and self.w.markov_w1 is not None:
            e = torch.stack([self.prev_embedding(int(p)) for p in prev_tokens])
            feats = torch.cat([feats, e.to(F32)], dim=-1)
        return bf(feats @ self.w.conf_w.to(F32) + self.w.conf_b.to(F32), self.rnd)

    def confidence(self, hidden, prev_tokens):
        """mx.sigmoid of the logits, rounded to bf16 (generate.py:878)."""
        return bf(torch.sigmoid(self.confidence_logits(hidden, prev_tokens)), self.rnd)

    def sample_block(self, base_logits, first_prev_token: int):
        """model.py:270-281 (argmax = first index of the maximum)."""
        if self.w.markov_w1 is None:
            return [int(i) for i in base_logits.argmax(-1)]
        toks, prev = [], int(first_prev_token)
        for i in range(base_logits.shape[0]):
            step = bf(base_logits[i] + self.step_bias(prev), self.rnd)
            prev = int(step.argmax())
            toks.append(prev)
        return toks


def accept_greedy(draft, tt):
    """generate.py:914-921: n = accepted prefix, committed = draft[:n] + [tt[n]]."""
    n = 0
    while n < len(draft) and draft[n] == tt[n]:
        n += 1
    return n, list(draft[:n]) + [tt[n]]


def greedy_generate_ref(target: Qwen3Ref, prompt_ids, max_new_tokens, kv8=False):
    """greedy_generate (generate.py:373-465), greedy, no eos: returns (ids, per-step logits)."""
    cache = target.make_cache(kv8)
    logits, _ = prefill(target, list(prompt_ids), cache, ())
    out, rows = [], []
    row = logits[-1]
    while True:
        nxt = int(row.argmax())
        out.append(nxt)
        rows.append(row)
        if len(out) >= max_new_tokens:
            break
        row = target.plain([nxt], cache)[-1]
    return out, rows


def truncate_by_confidence(draft, conf, threshold):
    """generate.py:875-887: keep drafted positions while the running product of survival
    probabilities stays >= threshold; always propose at least one token."""
    surv, keep = 1.0, 0
    for i, c in enumerate(conf):
        surv *= float(c)
        if surv < threshold:
            break
        keep = i + 1
    return list(draft[:keep]) or [draft[0]]


def speculative_generate_ref(target: Qwen3Ref, drafter: DSparkRef, prompt_ids, max_new_tokens,
                             max_draft_tokens=None, kv8=False, draft_override=None,
                             confidence_threshold=0.0):
    """speculative_generate greedy path (generate.py:806-961), lookup drafts off, with the
    confidence truncation of the two-phase path when confidence_threshold > 0 and the drafter
    has a confidence head. draft_override(round, draft, n_out) may replace the drafted tokens
    (benchmark configs). Returns (out_ids, accept_lengths)."""
    cfg = drafter.cfg
    tap = list(cfg.target_layer_ids)
    k = cfg.block_size
    cap = k if max_draft_tokens is None else max(1, min(max_draft_tokens, k))
    cache = target.make_cache(kv8)
    ctx = drafter.make_ctx_cache()
    logits, _ = None, None
    pos = 0
    ids = list(prompt_ids)
    for i in range(0, len(ids), 2048):
        piece = ids[i:i + 2048]
        logits, fused = target.run(piece, cache, tap)
        drafter.update_context(fused, pos, ctx)
        pos += len(piece)
    n_cached = len(ids)
    pending = int(logits[-1].argmax())
    out = [pending]
    accept = []
    rnd = 0
    while len(out) < max_new_tokens:
        noise = drafter.embed([pending] + [cfg.mask_token_id] * (k - 1))
        hidden = drafter.backbone(noise, n_cached, ctx)
        base = drafter.compute_logits(hidden[:cap])
        draft = drafter.sample_block(base, pending)
        if confidence_threshold > 0 and drafter.w.conf_w is not None:
            conf = drafter.confidence(hidden[:cap], [pending] + draft[:-1])
            draft = truncate_by_confidence(draft, conf.tolist(), confidence_threshold)
        if draft_override is not None:
            draft = draft_override(rnd, draft, len(out))
        v_logits, v_fused = target.run([pending] + draft, cache, tap)
        tt = [int(i) for i in v_logits.argmax(-1)]
        n, committed = accept_greedy(draft, tt)
        accept.append(len(committed))
        trim = len(draft) - n
        for c in cache:
            c.trim(trim)
        drafter.update_context(v_fused[: n + 1], n_cached, ctx)
        n_cached += n + 1
        out.extend(committed)
        pending = out[-1]
        rnd += 1
    return out, accept  # like the reference, the last round may pass max_new_tokens


__all__ = ["DSparkRef", "CtxCacheRef", "accept_greedy", "greedy_generate_ref",
           "speculative_generate_ref", "truncate_by_confidence", "Qwen3Ref"]
