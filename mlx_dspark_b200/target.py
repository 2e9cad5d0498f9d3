"""GPU Qwen3 target: make_cache / run (hidden-state tap) / plain, on the sm_100a kernels.

Drop-in for src/mlx_dspark/target.py:16-81 (Target.make_cache, run(ids, cache, tap) ->
(logits, fused), plain(ids, cache) -> logits; attributes model/tokenizer/kv_bits/is_vlm/
_tied). A forward over T tokens of B rows runs, per layer:

  rmsnorm -> W8 GEMM (q|k|v) -> q/k norm + RoPE + paged KV write -> paged GQA attention
  -> W8 GEMM (o, + residual) -> rmsnorm -> W8 GEMM (gate|up, SiLU*up) -> W8 GEMM (down, + residual)
  [-> bf16->fp16 copy of the residual stream into the fused tap buffer]

then the final norm and the W8 head. All launches go to the current stream with
programmatic dependent launch, from static per-(B, T) buffers, so the sequence can be
captured into a CUDA graph by the decode loops.
"""
from __future__ import annotations

import math

import torch

from . import ops
from ._lib import EPI_RESIDUAL_BF16, EPI_SILU_MUL_F16, EPI_STORE_BF16
from .config import TargetConfig
from .kvcache import PAGE, CacheState, PagePool, TargetCache
from .weights import PackedLinear, TargetWeights, pack

MAX_M = 64          # rows per W8A16 GEMM launch
MAX_ATTN_ROWS = 128  # query rows per kv head per attention CTA
PREFILL_CHUNK = 2048  # tokens per prefill chunk (the reference's PREFILL_CHUNK, generate.py:613)


def rope_inv_freq(head_dim: int, theta: float, device) -> torch.Tensor:
    i = torch.arange(0, head_dim, 2, dtype=torch.float64)
    return (theta ** (-i / head_dim)).to(torch.float32).to(device)


class PackedLayer:
    def __init__(self, lw, device):
        self.input_ln = lw.input_ln.to(device)
        self.post_ln = lw.post_ln.to(device)
        self.q_norm = lw.q_norm.to(device)
        self.k_norm = lw.k_norm.to(device)
        self.qkv = pack(lw.wq, lw.wk, lw.wv, device=device)
        self.kv = None  # drafters pack k|v separately for the context update
        self.o = pack(lw.wo, device=device)
        self.gu = pack(lw.gate, lw.up, interleave64=True, device=device)
        self.down = pack(lw.down, device=device)


class Buffers:
    """Static activations of one (B, T) forward shape."""

    def __init__(self, cfg: TargetConfig, B: int, T: int, n_tap: int, device, logits=True):
        M = B * T
        H, I = cfg.hidden_size, cfg.intermediate_size
        self.B, self.T, self.M = B, T, M
        self.ids = torch.zeros(M, dtype=torch.int32, device=device)
        self.h = torch.zeros(M, H, dtype=torch.bfloat16, device=device)
        self.xn16 = torch.zeros(M, H, dtype=torch.float16, device=device)
        self.qkv = torch.zeros(M, cfg.qkv_dim, dtype=torch.bfloat16, device=device)
        self.q = torch.zeros(M, cfg.q_dim, dtype=torch.bfloat16, device=device)
        self.attn16 = torch.zeros(M, cfg.q_dim, dtype=torch.float16, device=device)
        self.act16 = torch.zeros(M, I, dtype=torch.float16, device=device)
        self.fused16 = (torch.zeros(M, n_tap * H, dtype=torch.float16, device=device)
                        if n_tap else None)
        self.logits = (torch.zeros(M, cfg.vocab_size, dtype=torch.bfloat16, device=device)
                       if logits else None)
        # per-128-column-tile row sums of squares of h, written by the residual GEMMs for the
        # RMSNorm fused into the next GEMM
        self.sumsq = torch.zeros(M, H // 128, dtype=torch.float32, device=device)


class PrefillBuffers:
    """Activations of a prefill chunk of up to `cap` tokens of one row (the large-M GEMM path);
    rows(T) views the first T rows of each."""

    def __init__(self, cfg: TargetConfig, T: int, n_tap: int, device, all_logits: bool = False):
        H, I = cfg.hidden_size, cfg.intermediate_size
        self.T = self.cap = T
        self.all_logits = all_logits
        self.ids = torch.zeros(T, dtype=torch.int32, device=device)
        self.h = torch.zeros(T, H, dtype=torch.bfloat16, device=device)
        self.xn16 = torch.zeros(T, H, dtype=torch.float16, device=device)
        self.qkv = torch.zeros(T, cfg.qkv_dim, dtype=torch.bfloat16, device=device)
        self.q = torch.zeros(T, cfg.q_dim, dtype=torch.bfloat16, device=device)
        self.attn16 = torch.zeros(T, cfg.q_dim, dtype=torch.float16, device=device)
        self.act16 = torch.zeros(T, I, dtype=torch.float16, device=device)
        self.fused16 = (torch.zeros(T, n_tap * H, dtype=torch.float16, device=device)
                        if n_tap else None)
        # the last row's logits (prefill), or every row's (the run() API)
        self.logits = torch.zeros(T if all_logits else 1, cfg.vocab_size, dtype=torch.bfloat16,
                                  device=device)

    def rows(self, T: int) -> "PrefillBuffers":
        """The same buffers cut to the first T rows (shared storage)."""
        assert 1 <= T <= self.cap
        v = object.__new__(PrefillBuffers)
        v.__dict__.update(self.__dict__)
        v.T = T
        for f in ("ids", "h", "xn16", "qkv", "q", "attn16", "act16", "fused16"):
            t = getattr(self, f)
            setattr(v, f, None if t is None else t[:T])
        if self.all_logits:
            v.logits = self.logits[:T]
        return v


class Target:
    """GPU W8 Qwen3 target with a hidden-state tap (see module docstring)."""

    def __init__(self, weights: TargetWeights, tokenizer=None, *, kv_bits: int | None = None,
                 device="cuda", scratch: ops.Scratch | None = None):
        if kv_bits not in (None, 8):
            raise ValueError("kv_bits must be None (bf16 KV) or 8")
        self.cfg: TargetConfig = weights.cfg
        self.tokenizer = tokenizer
        self.kv_bits = kv_bits
        self.kv_group_size = 64
        self.is_vlm = False
        self.family = "qwen3"
        self._tied = weights.lm_head is None
        self.device = torch.device(device)
        c = self.cfg
        if c.head_dim not in (64, 128):
            raise ValueError("head_dim must be 64 or 128")
        self.embed = pack(weights.embed, device=device)
        self.layers = [PackedLayer(l, device) for l in weights.layers]
        self.norm = weights.norm.to(device)
        self.head = self.embed if self._tied else pack(weights.lm_head, device=device)
        self.inv_freq = rope_inv_freq(c.head_dim, c.rope_theta, device)
        self.scale = c.head_dim ** -0.5
        self.scratch = scratch or ops.Scratch(device)
        self._bufs: dict[tuple, Buffers] = {}
        self.model = self  # reference code reaches target.model for embed/lm_head binding
        self.group = c.num_attention_heads // c.num_key_value_heads
        self.draft_head = self.head  # the head a drafter shares (full vocabulary)

    capturable = True  # a round of this target can be captured into one CUDA graph

    def greedy_accept(self, logits, B, T, verify_ids, argmax, kv_len, commit, pending, plan):
        """Greedy acceptance of B verify blocks (dspark_accept_greedy)."""
        ops.accept_greedy(logits, B, T, verify_ids, argmax, kv_len, commit, pending, plan,
                          self.scratch)

    def argmax_row(self, row: torch.Tensor) -> int:
        return int(row.float().argmax())

    # ------------------------------------------------------------------ caches
    def new_pool(self, max_tokens: int, rows: int = 1, extra_pages: int = 0) -> PagePool:
        pages = rows * ((max_tokens + PAGE - 1) // PAGE) + extra_pages
        return PagePool(self.cfg.num_hidden_layers, pages, self.cfg.num_key_value_heads,
                        self.cfg.head_dim, self.kv_bits == 8, self.device)

    def make_cache(self, max_tokens: int = 4096) -> TargetCache:
        """Per-layer cache views over a fresh page pool (mlx-lm make_prompt_cache shape;
        QuantizedKVCache semantics when kv_bits == 8)."""
        pool = self.new_pool(max_tokens)
        state = CacheState(pool, 1, max_tokens, self.device)
        kind = "QuantizedKVCache" if self.kv_bits == 8 else "KVCache"
        return TargetCache(state, self.cfg.num_hidden_layers, kind)

    # ------------------------------------------------------------------ buffers
    def buffers(self, B: int, T: int, n_tap: int, logits: bool = True) -> Buffers:
        key = (B, T, n_tap, logits)
        b = self._bufs.get(key)
        if b is None:
            b = Buffers(self.cfg, B, T, n_tap, self.device, logits)
            self._bufs[key] = b
        return b

    def attn_splits(self, B: int, max_pages: int) -> int:
        s = max(1, (2 * 148) // (B * self.cfg.num_key_value_heads))
        return max(1, min(s, max_pages))

    def chunk_len(self, B: int = 1) -> int:
        """Largest T with B*T <= 64 GEMM rows and G*T <= 128 attention rows."""
        return max(1, min(MAX_M // B, MAX_ATTN_ROWS // self.group))

    # prefill chunks longer than this run through the large-M GEMM (prefill_chunk); shorter
    # ones through the verify forward
    wide_min_tokens = MAX_M

    def prefill_buffers(self, T: int, n_tap: int, all_logits: bool = False) -> PrefillBuffers:
        """Buffers for a T-token prefill chunk: one set per (n_tap, all_logits) kept at the
        largest T asked for so far, viewed at T rows."""
        key = ("prefill", n_tap, all_logits)
        b = self._bufs.get(key)
        if b is None or b.cap < T:
            self._bufs.pop(key, None)
            b = PrefillBuffers(self.cfg, T, n_tap, self.device, all_logits)
            self._bufs[key] = b
        return b.rows(T)

    def prefill_chunk(self, buf: PrefillBuffers, state: CacheState, tap=(), *,
                      logits: str | None = "last") -> None:
        """One prefill chunk of row 0 of `state` (ids in buf.ids) at positions seq_len[0] + t,
        through the large-M W8 GEMM (Target.run over one chunk, target.py:51-75, as
        _prefill_tapped drives it, generate.py:632-656). Writes the chunk's KV and taps;
        logits "last" (the last row, into buf.logits[0]), "all" or None. Does not advance
        seq_len. Attention runs the chunk's queries as rows of 128 // G tokens each: row v sees
        the keys before position seq_len + v * (128 // G) plus its own causal block, so the
        verify attention kernel serves the whole chunk in one launch (two when T is not a
        multiple of the row length)."""
        c, sc = self.cfg, self.scratch
        T = buf.T
        H, eps = c.hidden_size, c.rms_norm_eps
        Hq, Hkv, hd = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        tap_idx = {l: j for j, l in enumerate(tap)}
        tq = MAX_ATTN_ROWS // self.group
        V, rem = divmod(T, tq)
        pos0 = state.seq_len[:1]
        if V:
            bt_v = state.block_table[:1].expand(V, -1).contiguous()
            kvl_v = pos0 + torch.arange(V, dtype=torch.int32, device=self.device) * tq
            # key splits only while the grid is under two CTAs per SM: measured on a 1024-token
            # Qwen3-8B prefill, 1/2/4/8 splits took 20.9/21.6/22.0/23.1 ms (2048: 36.0/38.3/
            # 40.3/42.5) - the partials and the merge cost more than the causal imbalance
            splits_v = max(1, min(state.max_pages, (2 * 148) // (V * Hkv)))
        if rem:
            kvl_r = pos0 + V * tq
            splits_r = self.attn_splits(1, state.max_pages)
        ops.embed(buf.ids, self.embed, buf.h, T)
        for l, L in enumerate(self.layers):
            kv = state.layout(l)
            ops.rmsnorm(buf.h, L.input_ln, eps, y16=buf.xn16, M=T)
            ops.gemm_wide(buf.xn16, L.qkv, buf.qkv, epilogue=EPI_STORE_BF16, scratch=sc, M=T)
            ops.qkv_rope_kv_write(buf.qkv, 1, T, Hq, Hkv, hd, L.q_norm, L.k_norm, eps,
                                  self.inv_freq, pos0, buf.q, kv)
            if V:
                ops.attention(buf.q, V, tq, Hq, state.pool.layout(l, bt_v), kvl_v, True,
                              self.scale, buf.attn16, splits_v, sc)
            if rem:
                ops.attention(buf.q[V * tq:], 1, rem, Hq, kv, kvl_r, True, self.scale,
                              buf.attn16[V * tq:], splits_r, sc)
            self._wide_residual(buf.attn16, L.o, buf.h, T)
            ops.rmsnorm(buf.h, L.post_ln, eps, y16=buf.xn16, M=T)
            ops.gemm_wide(buf.xn16, L.gu, buf.act16, epilogue=EPI_SILU_MUL_F16, scratch=sc, M=T)
            tap16 = buf.fused16[:, tap_idx[l] * H:(tap_idx[l] + 1) * H] if l in tap_idx else None
            self._wide_residual(buf.act16, L.down, buf.h, T, tap16)
        if logits == "last":
            ops.rmsnorm(buf.h[T - 1:], self.norm, eps, y16=buf.xn16[T - 1:], M=1)
            ops.gemm(buf.xn16[T - 1:], self.head, buf.logits[:1], epilogue=EPI_STORE_BF16,
                     scratch=sc, M=1)
        elif logits == "all":
            assert buf.logits.shape[0] == T
            ops.rmsnorm(buf.h, self.norm, eps, y16=buf.xn16, M=T)
            ops.gemm_wide(buf.xn16, self.head, buf.logits, epilogue=EPI_STORE_BF16, scratch=sc,
                          M=T)

    def _wide_residual(self, x16: torch.Tensor, w: PackedLinear, h: torch.Tensor, T: int,
                       copy16: torch.Tensor | None = None) -> None:
        """h += x16 @ W^T (bf16 residual add in the GEMM epilogue), optionally also into the
        fp16 tap `copy16`."""
        ops.gemm_wide(x16, w, h, epilogue=EPI_RESIDUAL_BF16, residual=h, scratch=self.scratch,
                      M=T, copy16=copy16)

    # ------------------------------------------------------------------ the forward
    # the q|k|v GEMM runs the per-head norm + RoPE + KV write in its epilogue (one launch
    # instead of two; bit-identical outputs)
    fuse_qkv_rope = True
    # every RMSNorm but the first layer's input norm runs inside the GEMM that consumes it (the
    # residual GEMM before it writes per-tile sums of squares); the only difference from the
    # separate norm kernel is the fp32 summation order of the squares
    fuse_norm = True

    def forward(self, buf: Buffers, state: CacheState, tap=(), *, splits: int | None = None,
                with_logits: bool = True) -> None:
        """Run B x T tokens (ids already in buf.ids) at positions state.seq_len[b] + t.
        Writes KV for all T positions; does not advance seq_len."""
        c, sc = self.cfg, self.scratch
        B, T, M = buf.B, buf.T, buf.M
        splits = splits or self.attn_splits(B, state.max_pages)
        tap_idx = {l: j for j, l in enumerate(tap)}
        H = c.hidden_size
        n_layers = len(self.layers)
        eps = c.rms_norm_eps
        fuse = self.fuse_norm
        ss = buf.sumsq if fuse else None
        ops.embed(buf.ids, self.embed, buf.h, M, sumsq=ss)
        for l, L in enumerate(self.layers):
            kv = state.layout(l)
            # each GEMM warms L2 with the next GEMM's weights (the head after the last layer)
            nxt = self.layers[l + 1].qkv if l + 1 < n_layers else (self.head if with_logits else None)
            if fuse:
                self._qkv_rope(buf, L, kv, state, B, T, M, x=buf.h,
                               norm=ops.RowNorm(L.input_ln, eps, ss))
            else:
                ops.rmsnorm(buf.h, L.input_ln, eps, y16=buf.xn16, M=M)
                self._qkv_rope(buf, L, kv, state, B, T, M)
            ops.attention(buf.q, B, T, c.num_attention_heads, kv, state.seq_len, True,
                          self.scale, buf.attn16, splits, sc)
            ops.gemm(buf.attn16, L.o, buf.h, epilogue=EPI_RESIDUAL_BF16, residual=buf.h,
                     scratch=sc, M=M, prefetch=L.gu, sumsq_out=ss)
            if fuse:
                ops.gemm(buf.h, L.gu, buf.act16, epilogue=EPI_SILU_MUL_F16, scratch=sc, M=M,
                         prefetch=L.down, norm=ops.RowNorm(L.post_ln, eps, ss))
            else:
                ops.rmsnorm(buf.h, L.post_ln, eps, y16=buf.xn16, M=M)
                ops.gemm(buf.xn16, L.gu, buf.act16, epilogue=EPI_SILU_MUL_F16, scratch=sc, M=M,
                         prefetch=L.down)
            # the drafter's tap of this layer's output is written by the same epilogue
            tap16 = buf.fused16[:M, tap_idx[l] * H:(tap_idx[l] + 1) * H] if l in tap_idx else None
            ops.gemm(buf.act16, L.down, buf.h, epilogue=EPI_RESIDUAL_BF16, residual=buf.h,
                     scratch=sc, M=M, prefetch=nxt, sumsq_out=ss, copy16=tap16)
        if with_logits:
            if fuse:
                ops.gemm(buf.h, self.head, buf.logits, epilogue=EPI_STORE_BF16, scratch=sc, M=M,
                         norm=ops.RowNorm(self.norm, eps, ss))
            else:
                ops.rmsnorm(buf.h, self.norm, eps, y16=buf.xn16, M=M)
                ops.gemm(buf.xn16, self.head, buf.logits, epilogue=EPI_STORE_BF16, scratch=sc, M=M)

    def _qkv_rope(self, buf: Buffers, L, kv, state: CacheState, B: int, T: int, M: int,
                  x: torch.Tensor | None = None, norm: "ops.RowNorm | None" = None) -> None:
        """q|k|v projection of x (buf.xn16, or the bf16 residual stream with its fused input
        norm), per-head q/k norm + RoPE at state.seq_len, q into buf.q and K/V into the layer's
        paged cache."""
        c, sc = self.cfg, self.scratch
        x = buf.xn16 if x is None else x
        if self.fuse_qkv_rope:
            ops.gemm_qkv_rope(x, L.qkv, T=T, Hq=c.num_attention_heads,
                              Hkv=c.num_key_value_heads, hd=c.head_dim, q_norm=L.q_norm,
                              k_norm=L.k_norm, eps=c.rms_norm_eps, inv_freq=self.inv_freq,
                              pos0=state.seq_len, q_out=buf.q, kv=kv, scratch=sc, M=M,
                              prefetch=L.o, norm=norm)
            return
        ops.gemm(x, L.qkv, buf.qkv, epilogue=EPI_STORE_BF16, scratch=sc, M=M, prefetch=L.o,
                 norm=norm)
        ops.qkv_rope_kv_write(buf.qkv, B, T, c.num_attention_heads, c.num_key_value_heads,
                              c.head_dim, L.q_norm, L.k_norm, c.rms_norm_eps, self.inv_freq,
                              state.seq_len, buf.q, kv)

    # ------------------------------------------------------------------ reference API
    def run(self, ids, cache: TargetCache, tap):
        """ids [1, L] -> (logits [1, L, V] bf16, fused [1, L, n_tap*H] bf16)."""
        return self._run(ids, cache, list(tap))

    def plain(self, ids, cache: TargetCache):
        return self._run(ids, cache, [])[0]

    def _run(self, ids, cache: TargetCache, tap: list[int]):
        ids = torch.as_tensor(ids, dtype=torch.int32).reshape(-1).to(self.device)
        Ltot = ids.numel()
        st = cache.state
        off = cache.sync_to_device()
        st.ensure(0, off + Ltot)
        T = self.chunk_len(1)
        V, H = self.cfg.vocab_size, self.cfg.hidden_size
        logits = torch.empty(Ltot, V, dtype=torch.bfloat16, device=self.device)
        fused = (torch.empty(Ltot, len(tap) * H, dtype=torch.bfloat16, device=self.device)
                 if tap else None)
        pos = 0
        while pos < Ltot:
            if Ltot - pos > self.wide_min_tokens:
                t = min(PREFILL_CHUNK, Ltot - pos)
                buf = self.prefill_buffers(t, len(tap), all_logits=True)
                buf.ids.copy_(ids[pos:pos + t])
                self.prefill_chunk(buf, st, tap, logits="all")
            else:
                t = min(T, Ltot - pos)
                buf = self.buffers(1, t, len(tap))
                buf.ids.copy_(ids[pos:pos + t])
                self.forward(buf, st, tap)
            logits[pos:pos + t].copy_(buf.logits)
            if tap:
                fused[pos:pos + t].copy_(buf.fused16)
            pos += t
            st.seq_len.add_(t)
        cache.advance(Ltot)
        return logits[None], (None if fused is None else fused[None])

    def weight_bytes(self) -> int:
        n = self.embed.nbytes() + (0 if self._tied else self.head.nbytes())
        for L in self.layers:
            n += L.qkv.nbytes() + L.o.nbytes() + L.gu.nbytes() + L.down.nbytes()
        return n

    def verify_tap(self) -> None:
        """The tap is computed inside the same forward as the logits (no replicated loop
        to validate, unlike target.py:84-128); nothing to probe."""
        return None
