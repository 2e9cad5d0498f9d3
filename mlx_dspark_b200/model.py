"""GPU DSpark drafter (qwen3 family) on the sm_100a kernels.

Drop-in for DSparkDrafter (src/mlx_dspark/model.py:348-437): embed, fuse_target,
make_ctx_cache, update_context, backbone, compute_logits, sample_block, config,
block_size, mask_token_id, markov_head, confidence_head. The drafter context (the
per-layer K/V of the fused target hidden states, model.py:176-208) lives in a paged pool of
its own; the block K/V are written after the committed context for the duration of one
draft (the attention of model.py:258-283 reads [ctx; block] with no mask), and the context
update of the accepted rows overwrites them.
"""
from __future__ import annotations

import torch

from . import ops
from ._lib import EPI_RESIDUAL_BF16, EPI_SILU_MUL_F16, EPI_STORE_BF16
from .config import DSparkConfig, TargetConfig
from .kvcache import PAGE, CacheState, PagePool
from .target import PackedLayer, Target, rope_inv_freq
from .weights import DSparkWeights, pack


class _Markov:
    """Marker with the reference attribute name (markov_head is not None => sequential head)."""

    def __init__(self, w1, w2, rank):
        self.w1, self.w2, self.rank = w1, w2, rank


class DraftBuffers:
    def __init__(self, cfg: DSparkConfig, B: int, k: int, ctx_rows: int, n_tap: int, device):
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


class DSparkDrafter:
    def __init__(self, weights: DSparkWeights, target: Target, device="cuda"):
        cfg = weights.cfg
        self.config = cfg
        self.block_size = cfg.block_size
        self.mask_token_id = cfg.mask_token_id
        self.softcap = cfg.final_logit_softcapping
        if self.softcap is not None:
            raise NotImplementedError("logit softcapping (gemma4 drafters) is not built")
        if cfg.norm_style != "qwen":
            raise NotImplementedError("only the qwen3 drafter family is built")
        self.device = torch.device(device)
        self.target = target
        self.embed_w = target.embed if weights.embed is None else pack(weights.embed, device=device)
        self.head_w = target.head if weights.lm_head is None else pack(weights.lm_head, device=device)
        self.fc = pack(weights.fc, device=device)
        self.hidden_norm = weights.hidden_norm.to(device)
        self.norm = weights.norm.to(device)
        self.layers = []
        for lw in weights.layers:
            pl = PackedLayer(lw, device)
            pl.kv = pack(lw.wk, lw.wv, device=device)
            self.layers.append(pl)
        self.markov_head = None
        if weights.markov_w1 is not None:
            self.markov_head = _Markov(pack(weights.markov_w1, device=device),
                                       pack(weights.markov_w2, device=device), cfg.markov_rank)
        self.confidence_head = None
        self.inv_freq = rope_inv_freq(cfg.head_dim, cfg.rope_theta, device)
        self.scratch = target.scratch
        self._bufs = {}

    # ------------------------------------------------------------------ caches / buffers
    def new_pool(self, max_tokens: int, rows: int = 1) -> PagePool:
        c = self.config
        pages = rows * ((max_tokens + PAGE - 1) // PAGE)
        return PagePool(len(self.layers), pages, c.num_key_value_heads, c.head_dim, False,
                        self.device)

    def make_ctx_cache(self, max_tokens: int = 4096) -> CacheState:
        return CacheState(self.new_pool(max_tokens), 1, max_tokens, self.device)

    def buffers(self, B: int, k: int, ctx_rows: int) -> DraftBuffers:
        key = (B, k, ctx_rows)
        b = self._bufs.get(key)
        if b is None:
            b = DraftBuffers(self.config, B, k, ctx_rows, len(self.config.target_layer_ids),
                             self.device)
            self._bufs[key] = b
        return b

    # ------------------------------------------------------------------ device paths
    def update_context_dev(self, fused16: torch.Tensor, B: int, T: int, ctx: CacheState,
                           buf: DraftBuffers) -> None:
        """fused [B*T, n_tap*H] (fp16) -> fc -> hidden_norm -> per layer k_norm/RoPE K and V
        written at ctx positions seq_len[b] + t (model.py:381-384, update_ctx :254-256)."""
        c, sc = self.config, self.scratch
        M = B * T
        ops.gemm(fused16, self.fc, buf.ctx_h, epilogue=EPI_STORE_BF16, scratch=sc, M=M)
        ops.rmsnorm(buf.ctx_h, self.hidden_norm, c.rms_norm_eps, y16=buf.ctx_x16, M=M)
        for l, L in enumerate(self.layers):
            ops.gemm(buf.ctx_x16, L.kv, buf.ctx_kv, epilogue=EPI_STORE_BF16, scratch=sc, M=M)
            ops.qkv_rope_kv_write(buf.ctx_kv, B, T, 0, c.num_key_value_heads, c.head_dim, None,
                                  L.k_norm, c.rms_norm_eps, self.inv_freq, ctx.seq_len, None,
                                  ctx.layout(l))

    def draft_dev(self, pending: torch.Tensor, B: int, cap: int, ctx: CacheState,
                  buf: DraftBuffers, draft: torch.Tensor, verify_ids: torch.Tensor | None,
                  splits: int) -> None:
        """Block [pending, mask x (k-1)] -> backbone over [ctx; block] -> head over the first
        cap positions -> Markov sequential argmax (generate.py:846-852,910; model.py:386-409)."""
        c, sc = self.config, self.scratch
        k = self.block_size
        M = B * k
        ops.embed_block(pending, B, k, self.mask_token_id, self.embed_w, buf.h, buf.ids)
        for l, L in enumerate(self.layers):
            kv = ctx.layout(l)
            ops.rmsnorm(buf.h, L.input_ln, c.rms_norm_eps, y16=buf.xn16, M=M)
            ops.gemm(buf.xn16, L.qkv, buf.qkv, epilogue=EPI_STORE_BF16, scratch=sc, M=M)
            ops.qkv_rope_kv_write(buf.qkv, B, k, c.num_attention_heads, c.num_key_value_heads,
                                  c.head_dim, L.q_norm, L.k_norm, c.rms_norm_eps, self.inv_freq,
                                  ctx.seq_len, buf.q, kv)
            ops.attention(buf.q, B, k, c.num_attention_heads, kv, ctx.seq_len, False, c.scaling,
                          buf.attn16, splits, sc)
            ops.gemm(buf.attn16, L.o, buf.h, epilogue=EPI_RESIDUAL_BF16, residual=buf.h,
                     scratch=sc, M=M)
            ops.rmsnorm(buf.h, L.post_ln, c.rms_norm_eps, y16=buf.xn16, M=M)
            ops.gemm(buf.xn16, L.gu, buf.act16, epilogue=EPI_SILU_MUL_F16, scratch=sc, M=M)
            ops.gemm(buf.act16, L.down, buf.h, epilogue=EPI_RESIDUAL_BF16, residual=buf.h,
                     scratch=sc, M=M)
        ops.rmsnorm(buf.h, self.norm, c.rms_norm_eps, y16=buf.xn16, M=M)
        head_rows = cap if B == 1 else M
        ops.gemm(buf.xn16, self.head_w, buf.base, epilogue=EPI_STORE_BF16, scratch=sc,
                 M=head_rows)
        rows_per_b = cap if B == 1 else k
        if self.markov_head is not None:
            ops.markov_sample_block(buf.base, rows_per_b, B, cap, self.markov_head.w1,
                                    self.markov_head.w2, pending, draft, verify_ids, sc)
        else:
            raise NotImplementedError("drafters without a Markov head use markov_rank > 0 here")

    # ------------------------------------------------------------------ reference API
    def embed(self, ids):
        """ids [1, L] -> [1, L, H] bf16 (model.py:372-373)."""
        ids = torch.as_tensor(ids, dtype=torch.int32).reshape(-1).to(self.device)
        out = torch.empty(ids.numel(), self.config.hidden_size, dtype=torch.bfloat16,
                          device=self.device)
        ops.embed(ids, self.embed_w, out)
        return out[None]

    def update_context(self, target_hidden_cat, ctx_offset, ctx_caches: CacheState) -> None:
        """fused [1, n, n_tap*H] at context positions ctx_offset.. (model.py:381-384)."""
        fused = target_hidden_cat.reshape(-1, target_hidden_cat.shape[-1])
        n = fused.shape[0]
        ctx_caches.ensure(0, ctx_offset + n + self.block_size)
        pos = 0
        T = self.target.chunk_len(1)
        while pos < n:
            t = min(T, n - pos)
            buf = self.buffers(1, self.block_size, t)
            f16 = fused[pos:pos + t].to(torch.float16).contiguous()
            ctx_caches.set_len(0, ctx_offset + pos)
            self.update_context_dev(f16, 1, t, ctx_caches, buf)
            pos += t
        ctx_caches.set_len(0, ctx_offset + n)

    def sample_block(self, base_logits, first_prev_token: int):
        """base [cap, V] -> [cap] greedy tokens with the Markov head (model.py:398-409)."""
        base = base_logits.reshape(-1, base_logits.shape[-1]).to(torch.bfloat16).contiguous()
        cap = base.shape[0]
        prev = torch.tensor([int(first_prev_token)], dtype=torch.int32, device=self.device)
        draft = torch.empty(cap, dtype=torch.int32, device=self.device)
        if self.markov_head is None:
            return base.float().argmax(-1)
        ops.markov_sample_block(base, cap, 1, cap, self.markov_head.w1, self.markov_head.w2,
                                prev, draft, None, self.scratch)
        return draft

    def weight_bytes_per_draft(self, cap: int) -> int:
        n = self.fc.nbytes()
        for L in self.layers:
            n += L.qkv.nbytes() + L.o.nbytes() + L.gu.nbytes() + L.down.nbytes() + L.kv.nbytes()
        n += self.head_w.nbytes()
        if self.markov_head is not None:
            n += cap * self.markov_head.w2.nbytes()
        return n
