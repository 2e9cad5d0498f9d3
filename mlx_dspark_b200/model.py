"""GPU block drafters on the sm_100a kernels: DSpark (semi-autoregressive, Markov head) and
DFlash (block diffusion), both conditioned on target hidden states.

Both follow the same device path (BlockDrafter):
  context : fused target hidden [rows, n_tap*H] -> fc -> hidden_norm -> per layer
            k_norm/RoPE K and V written into the drafter's paged context cache
            (DSpark update_context, src/mlx_dspark/model.py:253-256 and :126-128;
            DFlash KV injection, src/mlx_dspark/dflash_model.py:100-124)
  block   : [pending, mask x (k-1)] -> embed -> layers (q from the block, K/V = [ctx; block],
            no mask) -> final norm (model.py:130-156,258-262; dflash_model.py:125-134,197-205)
The block K/V are written after the committed context for the duration of one draft; the
context update of the accepted rows overwrites them.

DSparkDrafter — drop-in for DSparkDrafter (model.py:220-320): own or shared embedding / head,
head over the first cap rows, then the sequential Markov head (greedy, or temperature drafts
with the q distributions kept for the acceptance test).
DFlashDrafter — drop-in for DFlashDraftModel (dflash_model.py:167-208) bound to a target: the
target's embedding and head, logits read from block row 1 on (logits_start = 1), greedy
argmax or temperature drafts; batch 1 like the reference's dflash_generate.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops
from ._lib import EPI_RESIDUAL_BF16, EPI_SILU_MUL_F16, EPI_STORE_BF16
from .config import DFlashConfig, DSparkConfig
from .kvcache import PAGE, CacheState, CtxCaches, PagePool
from .target import PREFILL_CHUNK, PackedLayer, Target, rope_inv_freq
from .weights import DFlashWeights, DSparkWeights, pack


@dataclass
class Sampling:
    """Temperature / nucleus / top-k parameters of a sampled decode (temperature > 0)."""

    temperature: float
    top_p: float = 1.0
    top_k: int = 0

    @property
    def active(self) -> bool:
        return self.temperature > 0.0


class _Markov:
    """Marker with the reference attribute name (markov_head is not None => sequential head)."""

    def __init__(self, w1, w2, rank):
        self.w1, self.w2, self.rank = w1, w2, rank


class _ConfidenceHead:
    """The confidence head's projection (model.py:211-217): bf16 weight row [H (+ R)] and bf16
    bias [1]; with_markov: its input also holds the previous token's Markov embedding."""

    def __init__(self, w, b, with_markov: bool):
        self.w, self.b, self.with_markov = w, b, with_markov


class DraftBuffers:
    def __init__(self, cfg, B: int, k: int, ctx_rows: int, device):
        H, I = cfg.hidden_size, cfg.intermediate_size
        q_dim = cfg.num_attention_heads * cfg.head_dim
        kv_dim = cfg.num_key_value_heads * cfg.head_dim
        M = B * k
        self.B, self.k, self.M = B, k, M
        self.h = torch.zeros(M, H, dtype=torch.bfloat16, device=device)
        self.xn16 = torch.zeros(M, H, dtype=torch.float16, device=device)
        self.qkv = torch.zeros(M, q_dim + 2 * kv_dim, dtype=torch.bfloat16, device=device)
        self.q = torch.zeros(M, q_dim, dtype=torch.bfloat16, device=device)
        self.attn16 = torch.zeros(M, q_dim, dtype=torch.float16, device=device)
        self.act16 = torch.zeros(M, I, dtype=torch.float16, device=device)
        self.base = torch.zeros(M, cfg.vocab_size, dtype=torch.bfloat16, device=device)
        self.ids = torch.zeros(M, dtype=torch.int32, device=device)
        # context update (rows of the verify block)
        self.ctx_h = torch.zeros(ctx_rows, H, dtype=torch.bfloat16, device=device)
        self.ctx_x16 = torch.zeros(ctx_rows, H, dtype=torch.float16, device=device)
        self.ctx_kv = torch.zeros(ctx_rows, 2 * kv_dim, dtype=torch.bfloat16, device=device)
        # per-128-column-tile row sums of squares for the RMSNorms fused into the next GEMM
        self.sumsq = torch.zeros(M, H // 128, dtype=torch.float32, device=device)
        self.ctx_sumsq = torch.zeros(H // 128 * ctx_rows, dtype=torch.float32, device=device)


class BlockDrafter:
    """Context update and block backbone shared by the DSpark and DFlash drafters."""

    logits_start = 0

    def __init__(self, cfg, fc, hidden_norm, norm, layer_weights, device, own_embed=None,
                 own_head=None):
        self.config = cfg
        self.block_size = cfg.block_size
        self.mask_token_id = cfg.mask_token_id
        self.device = torch.device(device)
        # the drafter's own embedding / head when its checkpoint carries them; otherwise it
        # shares the target's, which bind() attaches
        self._own_embed, self._own_head = own_embed, own_head
        self.target = None
        self.scratch = None
        self.embed_w, self.head_w = own_embed, own_head
        self.fc = pack(fc, device=device)
        self.hidden_norm = hidden_norm.to(device)
        self.norm = norm.to(device)
        self.layers = []
        for lw in layer_weights:
            pl = PackedLayer(lw, device)
            pl.kv = pack(lw.wk, lw.wv, device=device)
            self.layers.append(pl)
        self.inv_freq = rope_inv_freq(cfg.head_dim, cfg.rope_theta, device)
        self._bufs = {}
        self.rng = ops.rng_state(0, self.device)

    def bind(self, target: Target):
        """Attach the drafter to the target whose hidden states condition its drafts: the
        target's workspaces, and its embedding and head where the drafter has none of its own
        (DFlashDraftModel.bind, dflash_model.py:168-184; a DSpark drafter with shared
        embeddings the same way). Returns self; binding again to another target re-attaches."""
        if self.target is target:
            return self
        if getattr(target, "cfg", None) is not None and \
                target.cfg.hidden_size != self.config.hidden_size:
            raise ValueError(f"drafter hidden_size {self.config.hidden_size} does not match the "
                             f"target's {target.cfg.hidden_size}")
        self.target = target
        self.scratch = target.scratch
        self.embed_w = target.embed if self._own_embed is None else self._own_embed
        self.head_w = target.draft_head if self._own_head is None else self._own_head
        self._bufs = {}
        return self

    def _need_target(self) -> None:
        if self.target is None:
            raise RuntimeError("the drafter is not bound to a target: call drafter.bind(target) "
                               "(the generate loops do this)")

    def seed(self, seed: int) -> None:
        """Seed the device Philox stream used by host-API draws (mx.random.seed)."""
        self.rng.copy_(ops.rng_state(int(seed), self.device))

    # ------------------------------------------------------------------ caches / buffers
    def new_pool(self, max_tokens: int, rows: int = 1) -> PagePool:
        c = self.config
        pages = rows * ((max_tokens + PAGE - 1) // PAGE)
        return PagePool(len(self.layers), pages, c.num_key_value_heads, c.head_dim, False,
                        self.device)

    def make_ctx_cache(self, max_tokens: int = 4096) -> CtxCaches:
        """Per-layer context caches of one sequence (model.py:250-251) over a paged pool."""
        return CtxCaches(CacheState(self.new_pool(max_tokens), 1, max_tokens, self.device),
                         len(self.layers))

    def buffers(self, B: int, k: int, ctx_rows: int) -> DraftBuffers:
        self._need_target()
        key = (B, k, ctx_rows)
        b = self._bufs.get(key)
        if b is None:
            b = DraftBuffers(self.config, B, k, ctx_rows, self.device)
            self._bufs[key] = b
        return b

    # ------------------------------------------------------------------ device paths
    def update_context_dev(self, fused16: torch.Tensor, B: int, T: int, ctx: CacheState,
                           buf: DraftBuffers) -> None:
        """fused [B*T, n_tap*H] (fp16) -> fc -> hidden_norm -> per layer k_norm/RoPE K and V
        written at ctx positions seq_len[b] + t."""
        c, sc = self.config, self.scratch
        M = B * T
        eps = c.rms_norm_eps
        # fc -> (hidden_norm fused into each layer's k|v GEMM, whose epilogue runs k_norm + RoPE
        # and writes K/V into the context cache)
        ss = buf.ctx_sumsq[:c.hidden_size // 128 * M].view(M, c.hidden_size // 128)
        ops.gemm(fused16, self.fc, buf.ctx_h, epilogue=EPI_STORE_BF16, scratch=sc, M=M,
                 sumsq_out=ss)
        hn = ops.RowNorm(self.hidden_norm, eps, ss)
        for l, L in enumerate(self.layers):
            ops.gemm_qkv_rope(buf.ctx_h, L.kv, T=T, Hq=0, Hkv=c.num_key_value_heads,
                              hd=c.head_dim, q_norm=None, k_norm=L.k_norm, eps=eps,
                              inv_freq=self.inv_freq, pos0=ctx.seq_len, q_out=None,
                              kv=ctx.layout(l), scratch=sc, M=M, norm=hn)

    def update_context_wide(self, fused16: torch.Tensor, T: int, ctx) -> None:
        """update_context_dev for a prefill chunk: T tapped rows of row 0 of ctx through the
        large-M GEMM (model.py:253-256 over one 2048-row chunk, generate.py:646-647). The
        hidden norm runs as its own kernel here; the only difference from the fused form is
        the fp32 summation order of the squares."""
        c, sc = self.config, self.scratch
        eps = c.rms_norm_eps
        pb = self._prefill_rows(T)
        h, x16, kvo = pb["h"][:T], pb["x16"][:T], pb["kv"][:T]
        ops.gemm_wide(fused16, self.fc, h, epilogue=EPI_STORE_BF16, scratch=sc, M=T)
        ops.rmsnorm(h, self.hidden_norm, eps, y16=x16, M=T)
        for l, L in enumerate(self.layers):
            ops.gemm_wide(x16, L.kv, kvo, epilogue=EPI_STORE_BF16, scratch=sc, M=T)
            ops.qkv_rope_kv_write(kvo, 1, T, 0, c.num_key_value_heads, c.head_dim, None,
                                  L.k_norm, eps, self.inv_freq, ctx.seq_len[:1], None,
                                  ctx.layout(l))

    def _prefill_rows(self, T: int) -> dict:
        """Context-update buffers for prefill chunks, kept at the largest T asked for."""
        pb = self._bufs.get("prefill")
        if pb is None or pb["cap"] < T:
            c = self.config
            H, kv_dim = c.hidden_size, c.num_key_value_heads * c.head_dim
            self._bufs.pop("prefill", None)
            pb = {"cap": T,
                  "h": torch.zeros(T, H, dtype=torch.bfloat16, device=self.device),
                  "x16": torch.zeros(T, H, dtype=torch.float16, device=self.device),
                  "kv": torch.zeros(T, 2 * kv_dim, dtype=torch.bfloat16, device=self.device)}
            self._bufs["prefill"] = pb
        return pb

    def backbone_dev(self, pending: torch.Tensor, B: int, ctx: CacheState, buf: DraftBuffers,
                     splits: int, final_norm: bool = True) -> None:
        """Block [pending, mask x (k-1)] of each row at positions seq_len[b] + i -> layers over
        [ctx; block] -> final norm into buf.xn16 (fp16, the head GEMM input). With
        final_norm=False the block's hidden states stay in buf.h with their row sums of squares
        in buf.sumsq, for a head GEMM that fuses the final norm (final_head_norm())."""
        c, sc = self.config, self.scratch
        k = self.block_size
        M = B * k
        eps = c.rms_norm_eps
        ss = buf.sumsq
        ops.embed_block(pending, B, k, self.mask_token_id, self.embed_w, buf.h, buf.ids)
        for l, L in enumerate(self.layers):
            kv = ctx.layout(l)
            if l == 0:
                ops.rmsnorm(buf.h, L.input_ln, eps, y16=buf.xn16, M=M)
                x, nrm = buf.xn16, None
            else:
                x, nrm = buf.h, ops.RowNorm(L.input_ln, eps, ss)
            ops.gemm_qkv_rope(x, L.qkv, T=k, Hq=c.num_attention_heads,
                              Hkv=c.num_key_value_heads, hd=c.head_dim, q_norm=L.q_norm,
                              k_norm=L.k_norm, eps=eps, inv_freq=self.inv_freq, pos0=ctx.seq_len,
                              q_out=buf.q, kv=kv, scratch=sc, M=M, norm=nrm)
            ops.attention(buf.q, B, k, c.num_attention_heads, kv, ctx.seq_len, False, c.scaling,
                          buf.attn16, splits, sc)
            ops.gemm(buf.attn16, L.o, buf.h, epilogue=EPI_RESIDUAL_BF16, residual=buf.h,
                     scratch=sc, M=M, sumsq_out=ss)
            ops.gemm(buf.h, L.gu, buf.act16, epilogue=EPI_SILU_MUL_F16, scratch=sc, M=M,
                     norm=ops.RowNorm(L.post_ln, eps, ss))
            ops.gemm(buf.act16, L.down, buf.h, epilogue=EPI_RESIDUAL_BF16, residual=buf.h,
                     scratch=sc, M=M, sumsq_out=ss)
        if final_norm:
            ops.rmsnorm(buf.h, self.norm, eps, y16=buf.xn16, M=M)

    def final_head_norm(self, buf: DraftBuffers) -> "ops.RowNorm":
        """The final norm of a backbone_dev(final_norm=False) block, for the head GEMM."""
        return ops.RowNorm(self.norm, self.config.rms_norm_eps, buf.sumsq)

    # ------------------------------------------------------------------ reference API
    def update_context(self, target_hidden_cat, ctx_offset, ctx_caches) -> None:
        """fused [1, n, n_tap*H] at context positions ctx_offset.. (model.py:253-256)."""
        self._need_target()
        ctx_caches = getattr(ctx_caches, "state", ctx_caches)
        fused = target_hidden_cat.reshape(-1, target_hidden_cat.shape[-1])
        n = fused.shape[0]
        ctx_caches.grow(ctx_offset + n + self.block_size)
        ctx_caches.ensure(0, ctx_offset + n + self.block_size)
        pos = 0
        T = self.target.chunk_len(1)
        while pos < n:
            wide = n - pos > self.target.wide_min_tokens
            t = min(PREFILL_CHUNK if wide else T, n - pos)
            f16 = fused[pos:pos + t].to(torch.float16).contiguous()
            ctx_caches.set_len(0, ctx_offset + pos)
            if wide:
                self.update_context_wide(f16, t, ctx_caches)
            else:
                self.update_context_dev(f16, 1, t, ctx_caches, self.buffers(1, self.block_size, t))
            pos += t
        ctx_caches.set_len(0, ctx_offset + n)

    def embed(self, ids):
        """ids [1, L] -> [1, L, H] bf16 (model.py:244-245)."""
        self._need_target()
        ids = torch.as_tensor(ids, dtype=torch.int32).reshape(-1).to(self.device)
        out = torch.empty(ids.numel(), self.config.hidden_size, dtype=torch.bfloat16,
                          device=self.device)
        ops.embed(ids, self.embed_w, out)
        return out[None]


class DSparkDrafter(BlockDrafter):
    def __init__(self, weights: DSparkWeights, target: Target | None = None, device="cuda"):
        cfg = weights.cfg
        self.softcap = cfg.final_logit_softcapping
        if self.softcap is not None:
            raise NotImplementedError("logit softcapping (gemma4 drafters) is not built")
        if cfg.norm_style != "qwen":
            raise NotImplementedError("only the qwen3 drafter family is built")
        own_embed = None if weights.embed is None else pack(weights.embed, device=device)
        own_head = None if weights.lm_head is None else pack(weights.lm_head, device=device)
        super().__init__(cfg, weights.fc, weights.hidden_norm, weights.norm, weights.layers,
                         device, own_embed, own_head)
        self.markov_head = None
        if weights.markov_w1 is not None:
            self.markov_head = _Markov(pack(weights.markov_w1, device=device),
                                       pack(weights.markov_w2, device=device), cfg.markov_rank)
        self.confidence_head = None
        if weights.conf_w is not None:
            with_markov = cfg.confidence_head_with_markov and self.markov_head is not None
            self.confidence_head = _ConfidenceHead(
                weights.conf_w.to(device, torch.bfloat16).reshape(-1).contiguous(),
                weights.conf_b.to(device, torch.bfloat16).reshape(-1).contiguous(), with_markov)
        if target is not None:
            self.bind(target)

    def confidence_dev(self, buf: DraftBuffers, pending: torch.Tensor, draft: torch.Tensor,
                       cap: int, conf: torch.Tensor) -> None:
        """Survival probabilities of batch row 0's cap drafted positions into conf[:cap]
        (generate.py:875-880): from the backbone's pre-norm block rows left in buf.h by
        draft_dev, the pending token and the draft (prev_0 = pending, prev_i = draft[i-1])."""
        ch = self.confidence_head
        ops.confidence(buf.h, cap, ch.w, ch.b, conf, norm_w=self.norm,
                       eps=self.config.rms_norm_eps,
                       w1=self.markov_head.w1 if ch.with_markov else None,
                       first_prev=pending, prev_rest=draft.view(-1) if cap > 1 else None)

    def confidence_logits(self, block_hidden, prev_token_ids):
        """Confidence-head logits of normalised block hidden states [cap, H] (or [1, cap, H])
        and their previous tokens [cap] (model.py:311-320); None without a confidence head."""
        ch = self.confidence_head
        if ch is None:
            return None
        H = self.config.hidden_size
        h = block_hidden.reshape(-1, H).to(self.device, torch.bfloat16).contiguous()
        prev = torch.as_tensor(prev_token_ids, dtype=torch.int32).reshape(-1).to(self.device)
        n = h.shape[0]
        conf = torch.empty(n, dtype=torch.float32, device=self.device)
        logit = torch.empty(n, dtype=torch.float32, device=self.device)
        ops.confidence(h, n, ch.w, ch.b, conf,
                       w1=self.markov_head.w1 if ch.with_markov else None,
                       first_prev=prev[:1], prev_rest=prev[1:] if n > 1 else None, logit=logit)
        return logit

    def draft_dev(self, pending: torch.Tensor, B: int, cap: int, ctx: CacheState,
                  buf: DraftBuffers, draft: torch.Tensor, verify_ids: torch.Tensor | None,
                  splits: int, sampling: Sampling | None = None, rng: torch.Tensor | None = None,
                  q_probs: torch.Tensor | None = None) -> None:
        """Block -> backbone -> head over the first cap positions -> Markov head, greedy
        (generate.py:846-852,910) or a temperature draft keeping q (model.py:283-309)."""
        sc = self.scratch
        k = self.block_size
        self.backbone_dev(pending, B, ctx, buf, splits, final_norm=False)
        head_rows = cap if B == 1 else B * k
        ops.gemm(buf.h, self.head_w, buf.base, epilogue=EPI_STORE_BF16, scratch=sc,
                 M=head_rows, norm=self.final_head_norm(buf))
        rows_per_b = cap if B == 1 else k
        sampled = sampling is not None and sampling.active
        m = self.markov_head
        if m is not None and not sampled:
            ops.markov_sample_block(buf.base, rows_per_b, B, cap, m.w1, m.w2, pending, draft,
                                    verify_ids, sc)
        elif m is not None:
            ops.markov_sample_block_probs(buf.base, rows_per_b, B, cap, m.w1, m.w2, pending, draft,
                                          verify_ids, sampling.temperature, sampling.top_p,
                                          sampling.top_k, rng, q_probs, sc)
        else:
            # no sequential head: every position is an independent argmax / draw
            vids = None if verify_ids is None else verify_ids.view(B, cap + 1)
            if vids is not None:
                vids[:, 0].copy_(pending[:B])
            for b in range(B):
                base_b = buf.base[b * rows_per_b:b * rows_per_b + cap]
                v2 = None if vids is None else vids[b, 1:]
                if sampled:
                    ops.sample_rows(base_b, 1, cap, sampling.temperature, sampling.top_p,
                                    sampling.top_k, rng[b:b + 1], draft.view(B, cap)[b],
                                    stream_id=1, probs=q_probs[b * cap:(b + 1) * cap],
                                    tokens2=v2, temp_mode=1)
                else:
                    ops.argmax_rows(base_b, cap, draft.view(B, cap)[b], 1, v2, 1)

    # ------------------------------------------------------------------ reference API
    def sample_block(self, base_logits, first_prev_token: int):
        """base [cap, V] -> [cap] greedy tokens with the Markov head (model.py:270-281)."""
        self._need_target()
        base = base_logits.reshape(-1, base_logits.shape[-1]).to(torch.bfloat16).contiguous()
        cap = base.shape[0]
        if self.markov_head is None:
            return base.float().argmax(-1)
        prev = torch.tensor([int(first_prev_token)], dtype=torch.int32, device=self.device)
        draft = torch.empty(cap, dtype=torch.int32, device=self.device)
        ops.markov_sample_block(base, cap, 1, cap, self.markov_head.w1, self.markov_head.w2,
                                prev, draft, None, self.scratch)
        return draft

    def sample_block_probs(self, base_logits, first_prev_token: int, temperature: float,
                           top_p: float = 1.0, top_k: int = 0):
        """Temperature draft (model.py:283-309): (tokens [cap], probs [cap, V]). Draws come from
        this drafter's Philox stream (seed()); the stream does not advance (the acceptance
        step advances it in a decode loop)."""
        self._need_target()
        base = base_logits.reshape(-1, base_logits.shape[-1]).to(torch.bfloat16).contiguous()
        cap, V = base.shape
        draft = torch.empty(cap, dtype=torch.int32, device=self.device)
        probs = torch.zeros(cap, V, dtype=torch.float32, device=self.device)
        prev = torch.tensor([int(first_prev_token)], dtype=torch.int32, device=self.device)
        s = Sampling(temperature, top_p, top_k)
        if self.markov_head is not None:
            ops.markov_sample_block_probs(base, cap, 1, cap, self.markov_head.w1,
                                          self.markov_head.w2, prev, draft, None, temperature,
                                          top_p, top_k, self.rng, probs, self.scratch)
        else:
            ops.sample_rows(base, 1, cap, s.temperature, s.top_p, s.top_k, self.rng, draft,
                            stream_id=1, probs=probs, temp_mode=1)
        return draft, probs

    def weight_bytes_per_draft(self, cap: int) -> int:
        n = self.fc.nbytes()
        for L in self.layers:
            n += L.qkv.nbytes() + L.o.nbytes() + L.gu.nbytes() + L.down.nbytes() + L.kv.nbytes()
        n += self.head_w.nbytes()
        if self.markov_head is not None:
            n += cap * self.markov_head.w2.nbytes()
        return n


class DFlashDrafter(BlockDrafter):
    """DFlash block-diffusion drafter bound to a target (dflash_model.py:167-208)."""

    logits_start = 1

    def __init__(self, weights: DFlashWeights, target: Target | None = None, device="cuda"):
        cfg: DFlashConfig = weights.cfg
        if any(t != "full_attention" for t in cfg.layer_types):
            raise NotImplementedError("sliding-window DFlash layers are not built")
        if cfg.final_logit_softcapping is not None:
            raise NotImplementedError("logit softcapping is not built")
        super().__init__(cfg, weights.fc, weights.hidden_norm, weights.norm, weights.layers,
                         device)
        self.markov_head = None
        self.confidence_head = None
        if target is not None:
            self.bind(target)

    def make_cache(self, max_tokens: int = 4096) -> CtxCaches:
        return self.make_ctx_cache(max_tokens)

    def draft_dev(self, pending: torch.Tensor, B: int, cap: int, ctx: CacheState,
                  buf: DraftBuffers, draft: torch.Tensor, verify_ids: torch.Tensor | None,
                  splits: int, sampling: Sampling | None = None, rng: torch.Tensor | None = None,
                  q_probs: torch.Tensor | None = None) -> None:
        """Block -> backbone -> target head over block rows 1..cap -> argmax or draws
        (generate.py:537-549,561-565)."""
        if B != 1:
            raise NotImplementedError("DFlash drafts one request at a time (as dflash_generate)")
        assert cap <= self.block_size - 1
        self.backbone_dev(pending, 1, ctx, buf, splits)
        x = buf.xn16[self.logits_start:self.logits_start + cap]
        ops.gemm(x, self.head_w, buf.base, epilogue=EPI_STORE_BF16, scratch=self.scratch, M=cap)
        base = buf.base[:cap]
        v2 = None
        if verify_ids is not None:
            verify_ids.view(-1)[:1].copy_(pending[:1])
            v2 = verify_ids.view(-1)[1:]
        if sampling is not None and sampling.active:
            ops.sample_rows(base, 1, cap, sampling.temperature, sampling.top_p, sampling.top_k,
                            rng, draft.view(-1), stream_id=1, probs=q_probs[:cap], tokens2=v2,
                            temp_mode=0)
        else:
            ops.argmax_rows(base, cap, draft.view(-1), 1, v2, 1)

    def __call__(self, inputs, target_hidden, cache, logits_start: int = 0):
        """Reference forward: inputs [1, L] block ids, target_hidden [1, S, n_tap*H] new context
        rows appended at the cache's length; returns logits [1, L - logits_start, V]."""
        cache = getattr(cache, "state", cache)
        ids = torch.as_tensor(inputs, dtype=torch.int32).reshape(-1).to(self.device)
        L = ids.numel()
        assert L == self.block_size and int(ids[1:].eq(self.mask_token_id).all())
        if target_hidden is not None and target_hidden.numel():
            n0 = int(cache.seq_len[0])
            self.update_context(target_hidden, n0, cache)
        cache.ensure(0, int(cache.seq_len[0]) + self.block_size)
        buf = self.buffers(1, self.block_size, 1)
        self.backbone_dev(ids[:1], 1, cache, buf, self.target.attn_splits(1, cache.max_pages))
        rows = L - logits_start
        out = torch.zeros(rows, self.config.vocab_size, dtype=torch.bfloat16, device=self.device)
        ops.gemm(buf.xn16[logits_start:], self.head_w, out, epilogue=EPI_STORE_BF16,
                 scratch=self.scratch, M=rows)
        return out[None]
