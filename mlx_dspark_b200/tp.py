"""Tensor parallelism of the verify forward for targets past one GPU's budget (BASELINE C5:
Qwen3-32B at TP 2/4/8). The reference runs on one device; this is the B200 counterpart of its
target forward (src/mlx_dspark/target.py:58-75) spread over `world` ranks, one process per
GPU, NCCL over NVLink for the exchanges.

Split (Megatron-style, by head and by MLP slice):
  q/k/v      column-split by head: rank r owns q heads [r*Hq/w, (r+1)*Hq/w) and kv heads
             [r*Hkv/w, (r+1)*Hkv/w) (GQA groups stay whole), its slice of the paged KV cache
  o_proj     row-split over the same q heads -> fp32 partial [M, H] -> all-reduce -> residual
  gate/up    column-split over the intermediate dimension (I/w per rank)
  down_proj  row-split over I/w -> fp32 partial -> all-reduce -> residual
  lm_head    vocabulary-parallel: rank r owns rows [r*Vs, (r+1)*Vs) (padded to 128-row tiles);
             greedy acceptance all-gathers each rank's (row max, global argmax) pair — 8 bytes
             per row per rank — and merges them (ties to the smallest index, the mx.argmax rule)
  embedding, norms, the drafter: replicated (the drafter reads the replicated hidden taps and a
             replicated copy of the head)
The residual epilogue rounds once after the sum, bf16(h + bf16(sum of partials)), the same
rounding point as the single-device RESIDUAL_BF16 epilogue; only the fp32 summation order of
the partials differs from TP = 1.
"""
from __future__ import annotations

from dataclasses import replace

import torch
import torch.distributed as dist

import ctypes

from . import _lib, ops
from ._lib import EPI_SILU_MUL_F16, EPI_STORE_BF16, EPI_STORE_F32
from .target import Target
from .weights import GROUP, LayerWeights, QTensor, TargetWeights, pack

TILE = 128


def shard_rows(qt: QTensor, r0: int, r1: int) -> QTensor:
    return QTensor(qt.q[r0:r1].contiguous(), qt.scales[r0:r1].contiguous(),
                   qt.biases[r0:r1].contiguous())


def shard_cols(qt: QTensor, k0: int, k1: int) -> QTensor:
    assert k0 % GROUP == 0 and k1 % GROUP == 0
    return QTensor(qt.q[:, k0:k1].contiguous(), qt.scales[:, k0 // GROUP:k1 // GROUP].contiguous(),
                   qt.biases[:, k0 // GROUP:k1 // GROUP].contiguous())


def pad_rows(qt: QTensor, n: int) -> QTensor:
    """Append zero rows (q = 0, scale = 0, bias = 0) up to n rows."""
    extra = n - qt.q.shape[0]
    if extra <= 0:
        return qt
    z = lambda t: torch.zeros((extra,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)  # noqa: E731
    return QTensor(torch.cat([qt.q, z(qt.q)]), torch.cat([qt.scales, z(qt.scales)]),
                   torch.cat([qt.biases, z(qt.biases)]))


def vocab_shard(V: int, world: int) -> tuple[int, int]:
    """(rows per rank, rows per rank padded to whole 128-row GEMM tiles)."""
    vs = (V + world - 1) // world
    return vs, (vs + TILE - 1) // TILE * TILE


def check_divisible(cfg, world: int) -> None:
    H, I = cfg.hidden_size, cfg.intermediate_size
    if cfg.num_key_value_heads % world or cfg.num_attention_heads % world:
        raise ValueError(f"TP {world}: heads {cfg.num_attention_heads}/{cfg.num_key_value_heads} "
                         "do not split evenly")
    if (I // world) % TILE or I % world:
        raise ValueError(f"TP {world}: intermediate {I} does not split into 128-row tiles")
    if ((cfg.num_attention_heads + 2 * cfg.num_key_value_heads) // world * cfg.head_dim) % TILE:
        raise ValueError(f"TP {world}: the per-rank q|k|v width is not a multiple of 128")
    if (cfg.num_attention_heads // world * cfg.head_dim) % TILE:
        raise ValueError(f"TP {world}: the per-rank o_proj depth is not a multiple of 128")
    if H % TILE:
        raise ValueError("hidden size must be a multiple of 128")


def shard_target(tw: TargetWeights, rank: int, world: int):
    """Rank `rank`'s weights: (TargetWeights with the per-rank config, vocab offset, valid
    vocabulary rows of the head shard)."""
    cfg = tw.cfg
    check_divisible(cfg, world)
    hd = cfg.head_dim
    qh, kvh, I = cfg.num_attention_heads // world, cfg.num_key_value_heads // world, \
        cfg.intermediate_size // world
    q0, kv0, i0 = rank * qh * hd, rank * kvh * hd, rank * I
    layers = []
    for L in tw.layers:
        layers.append(LayerWeights(
            L.input_ln, L.post_ln, L.q_norm, L.k_norm,
            shard_rows(L.wq, q0, q0 + qh * hd), shard_rows(L.wk, kv0, kv0 + kvh * hd),
            shard_rows(L.wv, kv0, kv0 + kvh * hd), shard_cols(L.wo, q0, q0 + qh * hd),
            shard_rows(L.gate, i0, i0 + I), shard_rows(L.up, i0, i0 + I),
            shard_cols(L.down, i0, i0 + I)))
    V = cfg.vocab_size
    vs, vpad = vocab_shard(V, world)
    v0 = rank * vs
    valid = max(0, min(vs, V - v0))
    head = pad_rows(shard_rows(tw.head, v0, v0 + valid), vpad)
    rcfg = replace(cfg, num_attention_heads=qh, num_key_value_heads=kvh, intermediate_size=I,
                   vocab_size=vpad, tie_word_embeddings=False)
    return TargetWeights(rcfg, tw.embed, layers, tw.norm, head), v0, valid


class PeerAllReduce:
    """The buffers of the fused one-shot all-reduce (dspark_w8a16_gemm_peer +
    dspark_peer_reduce_residual): this rank's receive buffer [2][world][m_cap][n] fp32 and flags
    [2][world][n/128] int32, their CUDA IPC handles exchanged over the process group, and every
    peer's pair mapped here. Every rank builds it at the same point (a collective) and takes
    epochs in the same order."""

    def __init__(self, rank: int, world: int, group, m_cap: int, n: int):
        if not 2 <= world <= 8:
            raise ValueError("the fused all-reduce takes 2..8 ranks")
        L = _lib.lib()
        self.world, self.rank, self.m_cap, self.n = world, rank, m_cap, n
        self._own, self._mapped = [], []
        mine = []
        for nbytes in (2 * world * m_cap * n * 4, 2 * world * (n // 128) * 4):
            p = ctypes.c_void_p()
            _lib.check(L.dspark_peer_alloc(nbytes, ctypes.byref(p)), "dspark_peer_alloc")
            self._own.append(p.value)
            h = ctypes.create_string_buffer(64)
            _lib.check(L.dspark_ipc_handle(p.value, h), "dspark_ipc_handle")
            mine.append(h.raw)
        handles = [None] * world
        dist.all_gather_object(handles, mine, group=group)
        self.ar = _lib.PeerAR()
        for r in range(world):
            for j, field in enumerate(("recv", "flags")):
                if r == rank:
                    ptr = self._own[j]
                else:
                    p = ctypes.c_void_p()
                    _lib.check(L.dspark_ipc_open(handles[r][j], ctypes.byref(p)), "dspark_ipc_open")
                    self._mapped.append(p.value)
                    ptr = p.value
                getattr(self.ar, field)[r] = ptr
        self.ar.world, self.ar.rank, self.ar.m_cap, self.ar.n = world, rank, m_cap, n
        # device-resident epoch (dspark_peer_ar.epoch_dev): the calls take their numbers on the
        # device, so a CUDA graph of a round replays with fresh epochs on every rank
        dev = torch.device("cuda", torch.cuda.current_device())
        self.epoch_dev = torch.zeros(4, dtype=torch.int32, device=dev)
        self.ar.epoch_dev = self.epoch_dev.data_ptr()
        self.epoch = 0  # calls issued from the host (eager or captured)

    def next(self):
        self.epoch += 1
        self.ar.epoch = self.epoch
        return self.ar

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after every rank is done with them)."""
        L = _lib.lib()
        for p in self._mapped:
            L.dspark_ipc_close(p)
        for p in self._own:
            L.dspark_peer_free(p)
        self._mapped, self._own = [], []


class TPTarget(Target):
    """One rank's share of a tensor-parallel target. The process group must be NCCL (one
    process per GPU) for device tensors; every rank runs the same decode loop."""

    capturable = True  # a round, collectives included, is captured into one CUDA graph
    # o_proj / down_proj all-reduce of verify-sized calls (M <= 64): True, the fused GEMM
    # epilogue over NVLink peer memory (dspark_w8a16_gemm_peer + dspark_peer_reduce_residual,
    # partials summed in rank order: the same bits whatever the call's M); False, NCCL. Prefill
    # chunks (M > 64) always use NCCL.
    fused_allreduce = True

    def __init__(self, weights: TargetWeights, rank: int, world: int, group=None, tokenizer=None,
                 *, kv_bits: int | None = None, device="cuda"):
        shard, self.vocab_offset, self.vocab_valid = shard_target(weights, rank, world)
        super().__init__(shard, tokenizer, kv_bits=kv_bits, device=device)
        self.full_cfg = weights.cfg
        self.rank, self.world, self.pg = rank, world, group  # (self.group is the GQA group)
        # the drafters index the whole vocabulary: a replicated copy of the full head
        self.draft_head = self.embed if weights.lm_head is None else pack(weights.lm_head,
                                                                          device=device)
        self._partials: dict[int, torch.Tensor] = {}
        self._shard: dict[int, tuple] = {}
        self.peer: PeerAllReduce | None = None

    def _partial(self, M: int) -> torch.Tensor:
        p = self._partials.get(M)
        if p is None:
            p = torch.zeros(M, self.cfg.hidden_size, dtype=torch.float32, device=self.device)
            self._partials[M] = p
        return p

    def _all_reduce(self, t: torch.Tensor) -> None:
        dist.all_reduce(t, group=self.pg)

    def _row_parallel(self, x16: torch.Tensor, w, h: torch.Tensor, M: int) -> None:
        """h[:M] += all-reduce over ranks of x16 @ W^T (this rank's K-slice)."""
        if self.fused_allreduce and M <= 64:
            if self.peer is None:
                self.peer = PeerAllReduce(self.rank, self.world, self.pg, 64, self.cfg.hidden_size)
            ar = self.peer.next()
            ops.gemm_peer(x16, w, ar, scratch=self.scratch, M=M)
            ops.peer_reduce_residual(h, ar, M, self.scratch)
            return
        part = self._partial(M)
        ops.gemm(x16, w, part, epilogue=EPI_STORE_F32, scratch=self.scratch, M=M)
        self._all_reduce(part)
        ops.residual_add_f32(h, part, M)

    def release_peer(self) -> None:
        """Free the fused all-reduce's buffers; every rank calls it together (a barrier first,
        so no rank unmaps memory a peer may still write)."""
        if self.peer is not None:
            torch.cuda.synchronize()
            dist.barrier(group=self.pg)
            self.peer.close()
            self.peer = None

    def forward(self, buf, state, tap=(), *, splits: int | None = None,
                with_logits: bool = True) -> None:
        c, sc = self.cfg, self.scratch
        B, T, M = buf.B, buf.T, buf.M
        splits = splits or self.attn_splits(B, state.max_pages)
        tap_idx = {l: j for j, l in enumerate(tap)}
        H = c.hidden_size
        ops.embed(buf.ids, self.embed, buf.h, M)
        for l, L in enumerate(self.layers):
            kv = state.layout(l)
            ops.rmsnorm(buf.h, L.input_ln, c.rms_norm_eps, y16=buf.xn16, M=M)
            self._qkv_rope(buf, L, kv, state, B, T, M)
            ops.attention(buf.q, B, T, c.num_attention_heads, kv, state.seq_len, True,
                          self.scale, buf.attn16, splits, sc)
            self._row_parallel(buf.attn16, L.o, buf.h, M)
            ops.rmsnorm(buf.h, L.post_ln, c.rms_norm_eps, y16=buf.xn16, M=M)
            ops.gemm(buf.xn16, L.gu, buf.act16, epilogue=EPI_SILU_MUL_F16, scratch=sc, M=M)
            self._row_parallel(buf.act16, L.down, buf.h, M)
            if l in tap_idx:
                j = tap_idx[l]
                ops.bf16_to_f16(buf.h, buf.fused16[:, j * H:(j + 1) * H], M, H, sc.status)
        if with_logits:
            ops.rmsnorm(buf.h, self.norm, c.rms_norm_eps, y16=buf.xn16, M=M)
            ops.gemm(buf.xn16, self.head, buf.logits, epilogue=EPI_STORE_BF16, scratch=sc, M=M)

    def _wide_residual(self, x16, w, h, T, copy16=None) -> None:
        """The row-parallel projection of a prefill chunk: fp32 partial, NCCL all-reduce, then
        the bf16 residual add (as forward())."""
        part = self._partial(T)
        ops.gemm_wide(x16, w, part, epilogue=EPI_STORE_F32, scratch=self.scratch, M=T)
        self._all_reduce(part)
        ops.residual_add_f32(h, part, T)
        if copy16 is not None:
            ops.bf16_to_f16(h, copy16, T, h.shape[1], self.scratch.status)

    # ------------------------------------------------------------------ vocab-parallel argmax
    def _shard_bufs(self, rows: int):
        b = self._shard.get(rows)
        if b is None:
            dev = self.device
            b = (torch.zeros(rows, dtype=torch.float32, device=dev),
                 torch.zeros(rows, dtype=torch.int32, device=dev),
                 torch.zeros(self.world, rows, dtype=torch.float32, device=dev),
                 torch.zeros(self.world, rows, dtype=torch.int32, device=dev))
            self._shard[rows] = b
        return b

    def _gather_maxima(self, logits: torch.Tensor, rows: int):
        v, i, va, ia = self._shard_bufs(rows)
        ops.argmax_rows(logits, rows, i, values=v, index_offset=self.vocab_offset,
                        V=self.vocab_valid)
        dist.all_gather_into_tensor(va, v, group=self.pg)
        dist.all_gather_into_tensor(ia, i, group=self.pg)
        return va, ia

    def greedy_accept(self, logits, B, T, verify_ids, argmax, kv_len, commit, pending, plan):
        va, ia = self._gather_maxima(logits, B * T)
        ops.accept_greedy_sharded(va, ia, B, T, verify_ids, kv_len, commit, pending, plan)

    def argmax_row(self, row: torch.Tensor) -> int:
        va, ia = self._gather_maxima(row.view(1, -1), 1)
        vals, idx = va[:, 0].tolist(), ia[:, 0].tolist()
        best = max(range(self.world), key=lambda s: (vals[s], -idx[s]))
        return int(idx[best])


def init_process_group(backend: str = "nccl", timeout_s: int = 120):
    """One process per GPU from torchrun's environment; returns (rank, world, device)."""
    import datetime
    import os
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local) if backend == "nccl" else torch.device("cpu")
    if backend == "nccl":
        torch.cuda.set_device(dev)
    if not dist.is_initialized():
        dist.init_process_group(backend, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s),
                                **({"device_id": dev} if backend == "nccl" else {}))
    return rank, world, dev


__all__ = ["TPTarget", "shard_target", "shard_rows", "shard_cols", "vocab_shard",
           "init_process_group"]
