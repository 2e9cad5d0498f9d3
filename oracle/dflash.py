"""Oracle DFlash drafter and dflash_generate loop (CPU). TEST INFRASTRUCTURE ONLY.

DFlashRef follows src/mlx_dspark/dflash_model.py:84-208 (full-attention layers): the block
[anchor, mask x 15] is embedded with the target's embedding; the new context rows
target_hidden go through fc -> hidden_norm and, per layer, k_norm(k_proj(.)) roped at the
cache offset and v_proj(.) are appended to the layer's cache (update_and_fetch); the block's
queries and keys are roped at offset + S; SDPA with no mask over [ctx; block]; final norm; the
target's head on rows logits_start.. . The decoder layer (input norm, attention, residual,
post norm, SwiGLU MLP, residual) is the qwen 2-norm layer DSparkRef already restates, so the
same code serves (dflash_model.py:137-147 vs model.py:185-194).

dflash_generate_ref follows src/mlx_dspark/generate.py:468-601: greedy (argmax drafts, exact
argmax-match verify) or sampled (q = truncate(softmax(head / T)), drafts drawn from q,
rejection-sampling acceptance) with the device sampler's exact arithmetic and Philox counters
(oracle.sampling.*_exact): first token {offset 0, row 0, stream 2}; round r drafts
{offset r, row i, stream 1}; round r acceptance {offset r, row i, stream 0}.
Parity of this restatement to the reference is unpinned beyond the shared layer math: the
reference has no DFlash test vectors.
"""
from __future__ import annotations

import torch

from . import sampling as S
from .dspark import CtxCacheRef, DSparkRef, accept_greedy
from .qwen3 import Qwen3Ref, inv_freq, prefill


class DFlashRef(DSparkRef):
    def __init__(self, w, target_w, rnd: bool = True):
        self.w, self.cfg, self.rnd = w, w.cfg, rnd
        if any(t != "full_attention" for t in self.cfg.layer_types):
            raise NotImplementedError("sliding-window layers")
        self.embed_t = target_w.embed
        self.head_t = target_w.head
        self.freqs = inv_freq(self.cfg.head_dim, self.cfg.rope_theta)
        self._deq = {}

    def make_cache(self):
        return [CtxCacheRef() for _ in self.w.layers]

    def __call__(self, block_ids, target_hidden, cache, logits_start: int = 0):
        """dflash_model.py:197-208 -> logits [L - logits_start, V] (fp32 of bf16 values)."""
        h = self.embed(block_ids)
        if target_hidden is not None and target_hidden.shape[0]:
            self.update_context(target_hidden, cache[0].length, cache)
        hidden = self.backbone(h, cache[0].length, cache)
        return self.compute_logits(hidden[logits_start:])

    def draft_logits(self, pending, target_hidden, cache, cap):
        """The rows the verify reads: head over block rows 1..cap (generate.py:537-539). The
        block K/V never enter the cache (attend concatenates them locally), so the cache keeps
        context K/V only, as DFlash's does."""
        k = self.cfg.block_size
        return self([pending] + [self.cfg.mask_token_id] * (k - 1), target_hidden, cache, 1)[:cap]


def dflash_generate_ref(target: Qwen3Ref, drafter: DFlashRef, prompt_ids, max_new_tokens,
                        max_draft_tokens=None, temperature: float = 0.0, top_p: float = 1.0,
                        top_k: int = 0, seed: int = 0):
    """Returns (out_ids, accept_lengths)."""
    cfg = drafter.cfg
    tap = list(cfg.target_layer_ids)
    bs = cfg.block_size
    kdraft = bs - 1
    cap = kdraft if max_draft_tokens is None else max(1, min(max_draft_tokens, kdraft))
    cache = target.make_cache(False)
    dcache = drafter.make_cache()
    logits, fused = prefill(target, list(prompt_ids), cache, tap)
    pending_ctx = fused
    sampled = temperature > 0.0
    if sampled:
        pending, _ = S.sample_row_exact(logits[-1], temperature, 0, top_p, top_k, seed, 0, 0, 2)
    else:
        pending = int(logits[-1].argmax())
    out = [pending]
    accept = []
    rnd = 0
    while len(out) < max_new_tokens:
        head = drafter.draft_logits(pending, pending_ctx, dcache, cap)
        if sampled:
            draft, qs = [], []
            for i in range(cap):
                t, q = S.sample_row_exact(head[i], temperature, 0, top_p, top_k, seed, rnd, i, 1)
                draft.append(t)
                qs.append(q)
            v_logits, v_fused = target.run([pending] + draft, cache, tap)
            n, repl, _, _ = S.accept_sample_exact(v_logits, [pending] + draft, qs, temperature, 0,
                                                  top_p, top_k, seed, rnd)
            committed = draft[:n] + [repl]
        else:
            draft = [int(i) for i in head.argmax(-1)]
            v_logits, v_fused = target.run([pending] + draft, cache, tap)
            tt = [int(i) for i in v_logits.argmax(-1)]
            n, committed = accept_greedy(draft, tt)
        accept.append(len(committed))
        for c in cache:
            c.trim(len(draft) - n)
        pending_ctx = v_fused[: n + 1]
        out.extend(committed)
        pending = out[-1]
        rnd += 1
    return out, accept


__all__ = ["DFlashRef", "dflash_generate_ref"]
