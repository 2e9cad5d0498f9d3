"""Typed wrappers over the C ABI: torch tensors in, device pointers and shapes out.

Every wrapper launches on the current torch CUDA stream and raises ``DsparkError`` on a
nonzero status. ``Scratch`` owns the caller-side workspaces (one per kernel family, since
each family keeps self-resetting counters at the start of its buffer) and the device
status word that bounded device waits report into.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import KvLayout, call, lib
from .weights import PackedLinear


def _p(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("dspark_b200 kernels take CUDA tensors only (no CPU fallback)")


class Scratch:
    """Zero-filled, grow-only workspaces per kernel family plus a device status word."""

    FAMILIES = ("gemm", "attention", "accept", "markov", "accept_sample", "markov_probs")

    def __init__(self, device="cuda"):
        self.device = torch.device(device)
        self.bufs: dict[str, torch.Tensor] = {}
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.version = 0  # bumped when a buffer moves (captured graphs hold the addresses)
        # pinned copy of the status word, allocated here: a pinned allocation inside a CUDA
        # graph capture (the first read_status_async of a captured round) invalidates it
        self._status_host = (torch.zeros(1, dtype=torch.int32, pin_memory=True)
                             if self.device.type == "cuda" else None)

    def get(self, family: str, nbytes: int) -> torch.Tensor:
        b = self.bufs.get(family)
        if b is None or b.numel() < nbytes:
            b = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=self.device)
            self.bufs[family] = b
            self.version += 1
        return b

    def reserve(self, family: str, nbytes: int) -> None:
        self.get(family, nbytes)

    def read_status_async(self) -> None:
        """Enqueue a copy of the status word into pinned host memory on the current stream
        (inside a captured round it becomes part of the graph). The decode loops call it
        next to their per-round plan read and raise_on_status() after that round's sync, so a
        bounded device wait that ran out fails the round instead of letting it commit tokens
        computed from stale data."""
        self._status_host.copy_(self.status, non_blocking=True)

    def raise_on_status(self) -> None:
        """After the stream synchronised past read_status_async(): raise DsparkError (and
        reset the workspaces, as check_status does) if a kernel reported an error."""
        if self._status_host is not None and int(self._status_host[0]) != 0:
            self._status_host.zero_()
            self.check_status()

    def check_status(self) -> None:
        s = int(self.status.item())
        if s != 0:
            self.status.zero_()
            for b in self.bufs.values():  # counters may be left mid-count after a timeout
                b.zero_()
            raise _lib.DsparkError("device", s, "a kernel reported an error on the device")


# ----------------------------------------------------------------------------------------
def gemm_workspace_bytes(M: int, N: int, K: int) -> int:
    return int(lib().dspark_w8a16_gemm_workspace_bytes(M, N, K))


PREFETCH_LIMIT = 8 << 20  # bytes of the next weights warmed in L2 (C2 layer GEMMs: 0 MB 80.6 us, 8 MB 79.7, 16 MB 80.6, 32 MB 82.5)


class RowNorm:
    """An RMSNorm fused into the GEMM that consumes it: the weights, eps, and the per-tile row
    sums of squares [M, N/128] (fp32) written by the GEMM that produced the input."""

    __slots__ = ("w", "eps", "sumsq")

    def __init__(self, w: torch.Tensor, eps: float, sumsq: torch.Tensor):
        self.w, self.eps, self.sumsq = w, float(eps), sumsq  # sumsq [rows, N/128 tiles]


def _opts(prefetch: PackedLinear | None, norm: RowNorm | None,
          sumsq_out: torch.Tensor | None, copy16: torch.Tensor | None = None) -> _lib.GemmOpts:
    o = _lib.GemmOpts()
    if copy16 is not None:
        assert copy16.dtype == torch.float16 and copy16.stride(1) == 1
        o.copy_f16 = copy16.data_ptr()
        o.copy_f16_ld = copy16.stride(0)
    if prefetch is not None and PREFETCH_LIMIT > 0:
        # q is row-major [N, K]: a prefix of it is whole 128-row tiles. sb is [K/64, N] (1/16 of
        # q's bytes), so any prefix covers a few groups of every row: warm all of it, up to
        # limit / 8.
        o.prefetch[0] = prefetch.q.data_ptr()
        o.prefetch_bytes[0] = min(prefetch.q.numel(), PREFETCH_LIMIT)
        o.prefetch[1] = prefetch.sb.data_ptr()
        o.prefetch_bytes[1] = min(prefetch.sb.numel() * 4, PREFETCH_LIMIT // 8)
    if norm is not None:
        o.norm_w = norm.w.data_ptr()
        o.norm_sumsq = norm.sumsq.data_ptr()
        o.norm_tiles = norm.sumsq.shape[1]
        o.norm_eps = norm.eps
        o.norm_ld = norm.sumsq.stride(0)
    if sumsq_out is not None:
        o.row_sumsq = sumsq_out.data_ptr()
    return o


def gemm(x16: torch.Tensor, w: PackedLinear, y: torch.Tensor, *, epilogue=_lib.EPI_STORE_BF16,
         residual: torch.Tensor | None = None, scratch: Scratch, M: int | None = None,
         prefetch: PackedLinear | None = None, norm: RowNorm | None = None,
         sumsq_out: torch.Tensor | None = None, copy16: torch.Tensor | None = None) -> torch.Tensor:
    """y = x16 @ W^T with the chosen epilogue (see include/dspark_b200.h). `prefetch`: the next
    projection's weights, warmed in L2 (up to PREFETCH_LIMIT bytes) during this GEMM's tail.
    `norm`: x16 is the bf16 residual stream and the GEMM consumes its RMSNorm. `sumsq_out`
    (STORE_BF16 / RESIDUAL_BF16): per-tile row sums of squares of y for the next fused norm.
    `copy16` (RESIDUAL_BF16): an fp16 view [M, N] that also receives y (the hidden-state tap)."""
    _require_cuda(x16, y)
    M = x16.shape[0] if M is None else M
    K = w.K
    want = torch.bfloat16 if norm is not None else torch.float16
    assert x16.dtype == want and x16.shape[-1] >= K
    if sumsq_out is not None:  # written as a packed [M, N/128] block
        assert sumsq_out.is_contiguous() and tuple(sumsq_out.shape) == (M, w.N // 128)
    ws = scratch.get("gemm", gemm_workspace_bytes(M, w.N, K))
    if norm is None and sumsq_out is None and copy16 is None and \
            (prefetch is None or PREFETCH_LIMIT <= 0):
        call("dspark_w8a16_gemm", _p(x16), x16.stride(0), _p(w.q), _p(w.sb), M, w.N, K, _p(y),
             y.stride(0), _p(residual), residual.stride(0) if residual is not None else 0,
             epilogue, _p(ws), ws.numel(), _p(scratch.status), _stream())
        return y
    opts = _opts(prefetch, norm, sumsq_out, copy16)
    call("dspark_w8a16_gemm_ex", _p(x16), x16.stride(0), _p(w.q), _p(w.sb), M, w.N, K, _p(y),
         y.stride(0), _p(residual), residual.stride(0) if residual is not None else 0, epilogue,
         ctypes.byref(opts), _p(ws), ws.numel(), _p(scratch.status), _stream())
    return y


def gemm_peer(x16: torch.Tensor, w: PackedLinear, ar, *, scratch: Scratch,
              M: int | None = None) -> None:
    """This rank's row-split product x16 @ W^T sent to every rank's receive buffer, slot
    (ar.epoch & 1), with the tiles' epoch flags (dspark_w8a16_gemm_peer)."""
    _require_cuda(x16)
    M = x16.shape[0] if M is None else M
    assert x16.dtype == torch.float16 and x16.shape[-1] >= w.K
    ws = scratch.get("gemm", gemm_workspace_bytes(M, w.N, w.K))
    call("dspark_w8a16_gemm_peer", _p(x16), x16.stride(0), _p(w.q), _p(w.sb), M, w.N, w.K,
         ctypes.byref(ar), _p(ws), ws.numel(), _p(scratch.status), _stream())


def peer_reduce_residual(h: torch.Tensor, ar, M: int, scratch: Scratch,
                         timeout_ns: int = 2_000_000_000) -> None:
    """h[:M] = bf16(h + bf16(sum over ranks, in order, of this epoch's partials)), after a
    bounded wait for every rank's flags (DSPARK_ERR_TIMEOUT in scratch.status on expiry)."""
    _require_cuda(h)
    call("dspark_peer_reduce_residual", _p(h), h.stride(0), M, ctypes.byref(ar), int(timeout_ns),
         _p(scratch.status), _stream())


def gemm_wide(x16: torch.Tensor, w: PackedLinear, y: torch.Tensor, *,
              epilogue=_lib.EPI_STORE_BF16, residual: torch.Tensor | None = None,
              scratch: Scratch, M: int | None = None,
              copy16: torch.Tensor | None = None) -> torch.Tensor:
    """y = x16 @ W^T for a prefill chunk (any M; the persistent large-M tcgen05 kernel), with
    the epilogues of gemm(). `copy16` (RESIDUAL_BF16): an fp16 view [M, N] that also receives
    y (the hidden-state tap)."""
    _require_cuda(x16, y)
    M = x16.shape[0] if M is None else M
    K = w.K
    assert x16.dtype == torch.float16 and x16.shape[-1] >= K
    call("dspark_w8a16_gemm_wide", _p(x16), x16.stride(0), _p(w.q), _p(w.sb), M, w.N, K, epilogue,
         _p(y), y.stride(0), _p(residual), residual.stride(0) if residual is not None else 0,
         _p(copy16), copy16.stride(0) if copy16 is not None else 0, _p(scratch.status),
         _stream())
    return y


def gemm_wide_bn(bn: int) -> None:
    """Force the prefill GEMM's tokens per tile (128 / 256), or 0 to pick by M."""
    call("dspark_w8a16_gemm_wide_bn", int(bn))


def gemm_wide_plan(M: int, N: int, K: int) -> dict:
    bn, grid = ctypes.c_int(), ctypes.c_int()
    call("dspark_w8a16_gemm_wide_plan", M, N, K, ctypes.byref(bn), ctypes.byref(grid))
    return {"bn": bn.value, "grid": grid.value}


def gemm_qkv_rope(x16: torch.Tensor, w: PackedLinear, *, T: int, Hq: int, Hkv: int, hd: int,
                  q_norm: torch.Tensor | None, k_norm: torch.Tensor, eps: float,
                  inv_freq: torch.Tensor, pos0: torch.Tensor, q_out: torch.Tensor | None,
                  kv: KvLayout, scratch: Scratch, M: int | None = None,
                  prefetch: PackedLinear | None = None, norm: RowNorm | None = None) -> None:
    """The q|k|v GEMM with the per-head norm + RoPE + q / paged K/V writes in its epilogue
    (one launch; equals gemm(STORE_BF16) + qkv_rope_kv_write). `norm` as in gemm()."""
    _require_cuda(x16)
    M = x16.shape[0] if M is None else M
    K = w.K
    want = torch.bfloat16 if norm is not None else torch.float16
    assert x16.dtype == want and x16.shape[-1] >= K and w.N == (Hq + 2 * Hkv) * hd
    ws = scratch.get("gemm", gemm_workspace_bytes(M, w.N, K))
    opts = _opts(prefetch, norm, None)
    call("dspark_w8a16_gemm_qkv_rope", _p(x16), x16.stride(0), _p(w.q), _p(w.sb), M, K, T, Hq,
         Hkv, hd, _p(q_norm), _p(k_norm), float(eps), _p(inv_freq), _p(pos0), _p(q_out), kv,
         ctypes.byref(opts), _p(ws), ws.numel(), _p(scratch.status), _stream())


def embed(ids: torch.Tensor, w: PackedLinear, out: torch.Tensor, M: int | None = None,
          sumsq: torch.Tensor | None = None) -> torch.Tensor:
    """`sumsq` [M, H/128] fp32: also write the per-tile row sums of squares of the output (for
    the first layer's fused input norm)."""
    _require_cuda(ids, out)
    M = ids.numel() if M is None else M
    if sumsq is not None:
        assert sumsq.is_contiguous() and tuple(sumsq.shape) == (M, w.K // 128)
        call("dspark_embed_w8_sumsq", _p(ids), M, _p(w.q), _p(w.sb), w.N, w.K, _p(out),
             out.stride(0), _p(sumsq), _stream())
        return out
    call("dspark_embed_w8", _p(ids), M, _p(w.q), _p(w.sb), w.N, w.K, _p(out), out.stride(0), _stream())
    return out


def embed_block(pending: torch.Tensor, B: int, k: int, mask_id: int, w: PackedLinear,
                out: torch.Tensor, ids_out: torch.Tensor | None = None) -> torch.Tensor:
    call("dspark_embed_block_w8", _p(pending), B, k, mask_id, _p(w.q), _p(w.sb), w.N, w.K,
         _p(out), out.stride(0), _p(ids_out), _stream())
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, y: torch.Tensor | None = None,
            y16: torch.Tensor | None = None, M: int | None = None) -> None:
    _require_cuda(x, w)
    M = x.shape[0] if M is None else M
    H = w.numel()
    call("dspark_rmsnorm", _p(x), x.stride(0), _p(w), M, H, float(eps), _p(y),
         y.stride(0) if y is not None else 0, _p(y16), y16.stride(0) if y16 is not None else 0,
         _stream())


def kv_page_bytes(page_size: int, num_kv_heads: int, head_dim: int, kv8: bool) -> int:
    return int(lib().dspark_kv_page_bytes(page_size, num_kv_heads, head_dim, int(kv8)))


def kv_layout(pool: torch.Tensor, block_table: torch.Tensor, page_size: int, num_kv_heads: int,
              head_dim: int, kv8: bool) -> KvLayout:
    return KvLayout(pool.data_ptr(), block_table.data_ptr(), block_table.shape[1], page_size,
                    num_kv_heads, head_dim, int(kv8), 0,
                    kv_page_bytes(page_size, num_kv_heads, head_dim, kv8))


def qkv_rope_kv_write(qkv: torch.Tensor, B: int, T: int, Hq: int, Hkv: int, hd: int,
                      q_norm: torch.Tensor | None, k_norm: torch.Tensor, eps: float,
                      inv_freq: torch.Tensor, pos0: torch.Tensor, q_out: torch.Tensor | None,
                      kv: KvLayout) -> None:
    call("dspark_qkv_rope_kv_write", _p(qkv), qkv.stride(0), B, T, Hq, Hkv, hd, _p(q_norm),
         _p(k_norm), float(eps), _p(inv_freq), _p(pos0), _p(q_out), kv, _stream())


def attention_workspace_bytes(B, T, Hq, Hkv, hd, splits) -> int:
    return int(lib().dspark_attention_workspace_bytes(B, T, Hq, Hkv, hd, splits))


def attention(q: torch.Tensor, B: int, T: int, Hq: int, kv: KvLayout, kv_len: torch.Tensor,
              causal: bool, scale: float, out: torch.Tensor, splits: int, scratch: Scratch) -> None:
    ws = scratch.get("attention", attention_workspace_bytes(B, T, Hq, kv.num_kv_heads,
                                                            kv.head_dim, splits))
    call("dspark_attention", _p(q), B, T, Hq, kv, _p(kv_len), int(causal), float(scale), _p(out),
         out.stride(0), splits, _p(ws), ws.numel(), _p(scratch.status), _stream())


def accept_greedy(logits: torch.Tensor, B: int, T: int, verify_ids: torch.Tensor,
                  argmax: torch.Tensor, kv_len: torch.Tensor | None, commit: bool,
                  pending: torch.Tensor, plan: torch.Tensor, scratch: Scratch) -> None:
    V = logits.shape[-1]
    ws = scratch.get("accept", int(lib().dspark_accept_workspace_bytes(B * T, V)))
    call("dspark_accept_greedy", _p(logits), logits.stride(0), B, T, V, _p(verify_ids),
         _p(argmax), _p(kv_len), int(commit), _p(pending), _p(plan), _p(ws), ws.numel(), _stream())


def commit_lengths(plan: torch.Tensor, B: int, a: torch.Tensor, b: torch.Tensor | None = None):
    call("dspark_commit_lengths", _p(plan), plan.stride(0), B, _p(a), _p(b), _stream())


def draft_override(B, cap, V, ref, agree, round_ctr, kv_len, prompt_len, verify_ids):
    call("dspark_draft_override", B, cap, V, _p(ref), ref.shape[-1], _p(agree), agree.shape[1],
         _p(round_ctr), _p(kv_len), _p(prompt_len), _p(verify_ids), _stream())


def markov_sample_block(base: torch.Tensor, rows_per_b: int, B: int, cap: int, w1: PackedLinear,
                        w2: PackedLinear,
                        first_prev: torch.Tensor, draft: torch.Tensor,
                        verify_ids: torch.Tensor | None, scratch: Scratch) -> None:
    V = w2.N
    ws = scratch.get("markov", int(lib().dspark_markov_workspace_bytes(B, V)))
    call("dspark_markov_sample_block", _p(base), base.stride(0), rows_per_b, B, cap, V, w2.K, _p(w1.q),
         _p(w1.sb), _p(w2.q), _p(w2.sb), _p(first_prev), _p(draft), _p(verify_ids), _p(ws),
         ws.numel(), _p(scratch.status), _stream())


def bf16_to_f16(src: torch.Tensor, dst: torch.Tensor, rows: int, cols: int,
                status: torch.Tensor | None = None) -> None:
    """dst[:rows, :cols] = fp16(src); a value past the fp16 range sets DSPARK_ERR_RANGE in
    `status` (a Scratch.status word)."""
    call("dspark_bf16_to_f16", _p(src), src.stride(0), _p(dst), dst.stride(0), rows, cols,
         _p(status), _stream())


def apply_penalties(logits: torch.Tensor, B: int, T: int, counts: torch.Tensor,
                    verify_ids: torch.Tensor | None, presence: float, frequency: float) -> None:
    """In-place presence / frequency penalties on B verify blocks of T rows (_Penalizer)."""
    _require_cuda(logits, counts)
    call("dspark_apply_penalties", _p(logits), logits.stride(0), B, T, logits.shape[-1],
         _p(counts), _p(verify_ids), float(presence), float(frequency), _stream())


def penalty_counts_add(counts: torch.Tensor, plan: torch.Tensor, B: int) -> None:
    """counts[b] += the committed tokens of plan row b."""
    call("dspark_penalty_counts_add", _p(counts), B, counts.shape[-1], _p(plan), plan.stride(0),
         _stream())


def argmax_rows(logits: torch.Tensor, rows: int, tokens: torch.Tensor, tok_stride: int = 1,
                tokens2: torch.Tensor | None = None, tok2_stride: int = 1, *,
                values: torch.Tensor | None = None, index_offset: int = 0,
                V: int | None = None) -> torch.Tensor:
    """First-index argmax of each row over its first V columns (the greedy draft of a head-less
    block drafter; with values/index_offset, one vocabulary shard's maxima)."""
    _require_cuda(logits, tokens)
    call("dspark_argmax_rows", _p(logits), logits.stride(0), rows,
         logits.shape[-1] if V is None else int(V), _p(tokens), int(tok_stride), _p(tokens2),
         int(tok2_stride), _p(values), int(index_offset), _stream())
    return tokens


def logprobs(logits: torch.Tensor, rows: int, ids: torch.Tensor, ids_ld: int, T: int, top_k: int,
             logp: torch.Tensor, top_ids: torch.Tensor | None = None,
             top_logp: torch.Tensor | None = None, V: int | None = None) -> None:
    """Raw log-softmax entry of each row's token (row r's token is ids[(r // T) * ids_ld + r % T])
    into logp[r], and with top_k > 0 the row's top_k entries, descending, into top_ids /
    top_logp [rows, top_k] (_logprobs_for_block, generate.py:149-176)."""
    _require_cuda(logits, ids, logp, top_ids, top_logp)
    call("dspark_logprobs", _p(logits), logits.stride(0), rows,
         logits.shape[-1] if V is None else int(V), _p(ids), int(ids_ld), int(T), int(top_k),
         _p(logp), _p(top_ids), _p(top_logp), _stream())


def confidence(hidden: torch.Tensor, rows: int, proj_w: torch.Tensor, proj_b: torch.Tensor,
               conf: torch.Tensor, *, norm_w: torch.Tensor | None = None, eps: float = 1e-6,
               w1: PackedLinear | None = None, first_prev: torch.Tensor | None = None,
               prev_rest: torch.Tensor | None = None, logit: torch.Tensor | None = None) -> None:
    """Confidence-head survival probabilities of `rows` drafted positions (dspark_confidence):
    conf[i] = bf16(sigmoid(proj([norm(hidden_i), w1[prev_i]]))), prev_0 = first_prev[0],
    prev_i = prev_rest[i - 1]; without norm_w the rows are taken as already normalised."""
    _require_cuda(hidden, proj_w, proj_b, conf, norm_w, first_prev, prev_rest, logit)
    H = hidden.shape[-1]
    call("dspark_confidence", _p(hidden), hidden.stride(0), rows, H, _p(norm_w), float(eps),
         None if w1 is None else _p(w1.q), None if w1 is None else _p(w1.sb),
         0 if w1 is None else w1.N, 0 if w1 is None else w1.K, _p(first_prev), _p(prev_rest),
         _p(proj_w), _p(proj_b), _p(logit), _p(conf), _stream())


def residual_add_f32(h: torch.Tensor, summed: torch.Tensor, M: int) -> None:
    """h[:M] = bf16(h + bf16(summed)) (row-split projection after its all-reduce)."""
    call("dspark_residual_add_f32", _p(h), h.stride(0), _p(summed), summed.stride(0), M,
         h.shape[-1], _stream())


def accept_greedy_sharded(values: torch.Tensor, indices: torch.Tensor, B: int, T: int,
                          verify_ids: torch.Tensor, kv_len: torch.Tensor | None, commit: bool,
                          pending: torch.Tensor, plan: torch.Tensor) -> None:
    """Greedy acceptance from every vocabulary shard's (max, global argmax) per row."""
    call("dspark_accept_greedy_sharded", _p(values), _p(indices), values.shape[0], B, T,
         _p(verify_ids), _p(kv_len), int(commit), _p(pending), _p(plan), _stream())


# ----------------------------------------------------------------------------------------
# lossless speculative sampling (K9)
def rng_state(seeds, device="cuda") -> torch.Tensor:
    """Device {seed, offset} pairs, one per request (int64 storage of the u64 words)."""
    seeds = [seeds] if isinstance(seeds, int) else list(seeds)
    words = [((int(s) & 0xFFFFFFFFFFFFFFFF) ^ (1 << 63)) - (1 << 63) for s in seeds]
    t = torch.zeros(len(words), 2, dtype=torch.int64)
    t[:, 0] = torch.tensor(words, dtype=torch.int64)
    return t.to(device)


def sample_rows(logits: torch.Tensor, groups: int, rows: int, temperature: float, top_p: float,
                top_k: int, rng: torch.Tensor, tokens: torch.Tensor, *, stream_id: int = 2,
                row_base: int = 0, tok_stride: int = 1, probs: torch.Tensor | None = None,
                tokens2: torch.Tensor | None = None, tok2_stride: int = 1,
                temp_mode: int = 0) -> torch.Tensor:
    """Draw one token per row of truncate(softmax(logits / T)) (dspark_sample_rows)."""
    _require_cuda(logits, rng, tokens)
    assert logits.dtype == torch.bfloat16
    V = logits.shape[-1]
    call("dspark_sample_rows", _p(logits), logits.stride(0), groups, rows, V, float(temperature),
         int(temp_mode), float(top_p), int(top_k or 0), _p(rng), int(stream_id), int(row_base),
         _p(probs), probs.stride(0) if probs is not None else 0, _p(tokens), int(tok_stride),
         _p(tokens2), int(tok2_stride), _stream())
    return tokens


def accept_sample(logits: torch.Tensor, B: int, T: int, verify_ids: torch.Tensor,
                  q_probs: torch.Tensor | None, temperature: float, top_p: float, top_k: int,
                  rng: torch.Tensor, kv_len: torch.Tensor | None, commit: bool,
                  pending: torch.Tensor, plan: torch.Tensor, scratch: Scratch, *,
                  q_onehot: bool = False, temp_mode: int = 0) -> None:
    """Rejection-sampling acceptance of B blocks (dspark_accept_sample); advances rng offsets."""
    _require_cuda(logits, verify_ids, rng, pending, plan)
    V = logits.shape[-1]
    ws = scratch.get("accept_sample", int(lib().dspark_accept_sample_workspace_bytes(B, T)))
    ld_q = q_probs.shape[-1] if q_probs is not None else 0
    call("dspark_accept_sample", _p(logits), logits.stride(0), B, T, V, _p(verify_ids),
         _p(q_probs), ld_q, int(q_onehot), float(temperature), int(temp_mode), float(top_p),
         int(top_k or 0), _p(rng), _p(kv_len), int(commit), _p(pending), _p(plan), _p(ws),
         ws.numel(), _stream())


def markov_sample_block_probs(base: torch.Tensor, rows_per_b: int, B: int, cap: int,
                              w1: PackedLinear, w2: PackedLinear, first_prev: torch.Tensor,
                              draft: torch.Tensor, verify_ids: torch.Tensor | None,
                              temperature: float, top_p: float, top_k: int, rng: torch.Tensor,
                              q_probs: torch.Tensor, scratch: Scratch) -> None:
    """DSpark temperature draft: Markov step + draw per position (model.py:283-309)."""
    V = w2.N
    ws = scratch.get("markov_probs", int(lib().dspark_markov_probs_workspace_bytes(B, V)))
    call("dspark_markov_sample_block_probs", _p(base), base.stride(0), rows_per_b, B, cap, V,
         w2.K, _p(w1.q), _p(w1.sb), _p(w2.q), _p(w2.sb), _p(first_prev), _p(draft),
         _p(verify_ids), float(temperature), float(top_p), int(top_k or 0), _p(rng), _p(q_probs),
         q_probs.shape[-1], _p(ws), ws.numel(), _stream())
