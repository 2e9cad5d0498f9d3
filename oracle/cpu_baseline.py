"""Timed CPU baseline: plain greedy decode of the W8 Qwen3 target on the host cores.
TEST / BENCHMARK INFRASTRUCTURE ONLY (bench.py's cpu_baseline leg and --impl reference).

The reference's MLX CPU backend cannot run here (mlx is not installed), so this is the
oracle port of greedy_generate's per-token work (src/mlx_dspark/generate.py:433-450: one
target forward of one token over the KV cache, then argmax), written for speed on CPU:
weights stay int8 + bf16 scale/bias and every linear is one pass over them in C
(oracle/cpu_gemv.c: the group's scale and bias applied to its partial dot product, as MLX's
CPU qmv does, threads over rows); the rest is fp32 torch with the oracle's bf16 rounding
points. Without the built C library the linears fall back to torch, dequantizing row chunks.
"""
from __future__ import annotations

import os
import time

import torch

from .qwen3 import F32, bf, inv_freq, rms_norm, rope, silu

_GEMV = None


def _gemv_lib():
    """oracle/_build/libcpu_gemv.so (oracle/build_cpu.py), or None when it is not built."""
    global _GEMV
    if _GEMV is None:
        import ctypes
        from pathlib import Path
        path = Path(__file__).resolve().parent / "_build" / "libcpu_gemv.so"
        if not path.exists():
            try:
                from .build_cpu import build
                build()
            except Exception:  # noqa: BLE001 - the torch path still works
                _GEMV = False
                return None
        lib = ctypes.CDLL(str(path))
        P = ctypes.c_void_p
        lib.dspark_cpu_w8_gemv.argtypes = [P, P, P, P, P, ctypes.c_int, ctypes.c_int, P,
                                           ctypes.c_int]
        lib.dspark_cpu_w8_gemv.restype = None
        _GEMV = lib
    return _GEMV or None


def linear_kind() -> str:
    """How the timed decode computes its W8 linears (for the baseline's sample description)."""
    if _gemv_lib() is not None:
        return ("int8 weights read once per step by the threaded AVX2 C group-64 GEMV of "
                "oracle/cpu_gemv.c; the small ops between products in torch on one thread")
    return "int8 weights dequantized per step in torch (oracle/cpu_gemv.c not built)"


class StreamingDecoder:
    """One-token decode of a TargetWeights on the CPU with a dense per-layer KV cache."""

    def __init__(self, w, max_ctx: int, threads: int | None = None, chunk_rows: int = 2048):
        self.w, self.cfg = w, w.cfg
        # the cores this process may run on (an affinity mask can hold fewer than the host has)
        usable = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else None
        self.threads = threads or usable or os.cpu_count() or 1
        # the C GEMV runs its own pool of self.threads threads, which spin between the
        # products; torch's thread pool beside it would fight them for the cores during the
        # small ops in between (on an 8-core host, 2.6 tok/s with one torch thread against
        # 1.0 with eight), so torch gets one thread when the C GEMV is there
        torch.set_num_threads(1 if _gemv_lib() is not None else self.threads)
        c = self.cfg
        self.freqs = inv_freq(c.head_dim, c.rope_theta)
        self.chunk = chunk_rows
        L, Hkv, hd = c.num_hidden_layers, c.num_key_value_heads, c.head_dim
        self.K = torch.zeros(L, Hkv, max_ctx, hd)
        self.V = torch.zeros(L, Hkv, max_ctx, hd)
        self.len = 0

    def fill_random_context(self, n: int, seed: int = 0) -> None:
        """Stand-in context of n positions (timing sample: the attention work of a real
        context of that length, without paying for a CPU prefill)."""
        g = torch.Generator().manual_seed(seed)
        self.K[:, :, :n].normal_(0, 1, generator=g)
        self.V[:, :, :n].normal_(0, 1, generator=g)
        self.len = n

    def _lin(self, x, qt):
        N, K = qt.q.shape
        lib = _gemv_lib()
        if lib is not None and qt.scales.dtype == torch.bfloat16 and qt.biases.dtype == torch.bfloat16:
            import ctypes
            xc = x.to(F32).contiguous()
            out = torch.empty(N, dtype=F32)
            xs = torch.empty(K // 64, dtype=F32)
            q, sc, bi = qt.q.contiguous(), qt.scales.contiguous(), qt.biases.contiguous()
            P = ctypes.c_void_p
            lib.dspark_cpu_w8_gemv(P(q.data_ptr()), P(sc.data_ptr()), P(bi.data_ptr()),
                                   P(xc.data_ptr()), P(out.data_ptr()), N, K, P(xs.data_ptr()),
                                   self.threads)
            return bf(out)
        out = torch.empty(N, dtype=F32)
        for r0 in range(0, N, self.chunk):
            r1 = min(N, r0 + self.chunk)
            w = qt.q[r0:r1].to(F32).view(r1 - r0, K // 64, 64)
            w.mul_(qt.scales[r0:r1].to(F32)[..., None]).add_(qt.biases[r0:r1].to(F32)[..., None])
            out[r0:r1] = w.view(r1 - r0, K) @ x
        return bf(out)

    def step(self, token: int) -> int:
        c, W = self.cfg, self.w
        e = W.embed
        h = bf(e.scales[token].to(F32).repeat_interleave(64) * e.q[token].to(F32)
               + e.biases[token].to(F32).repeat_interleave(64))
        pos = self.len
        p = torch.tensor([pos])
        for i, L in enumerate(W.layers):
            x = rms_norm(h, L.input_ln, c.rms_norm_eps)
            q = self._lin(x, L.wq).view(c.num_attention_heads, 1, c.head_dim)
            k = self._lin(x, L.wk).view(c.num_key_value_heads, 1, c.head_dim)
            v = self._lin(x, L.wv).view(c.num_key_value_heads, 1, c.head_dim)
            q = rope(rms_norm(q, L.q_norm, c.rms_norm_eps), p, self.freqs)
            k = rope(rms_norm(k, L.k_norm, c.rms_norm_eps), p, self.freqs)
            self.K[i, :, pos] = k[:, 0]
            self.V[i, :, pos] = v[:, 0]
            # GQA as a batched product per kv head: query heads j*rep .. j*rep+rep-1 read kv
            # head j (no repeated copy of the context)
            rep = c.num_attention_heads // c.num_key_value_heads
            qg = q.reshape(c.num_key_value_heads, rep, c.head_dim)
            Kc, Vc = self.K[i, :, :pos + 1], self.V[i, :, :pos + 1]
            s = (qg @ Kc.transpose(1, 2)) * c.head_dim ** -0.5
            a = bf(torch.softmax(s, -1) @ Vc).reshape(-1)
            h = bf(h + self._lin(a, L.wo))
            x = rms_norm(h, L.post_ln, c.rms_norm_eps)
            act = bf(bf(silu(self._lin(x, L.gate))) * self._lin(x, L.up))
            h = bf(h + self._lin(act, L.down))
        hn = rms_norm(h, W.norm, c.rms_norm_eps)
        logits = self._lin(hn, W.head)
        self.len += 1
        return int(logits.argmax())


def time_greedy_decode(w, context: int, budget_s: float = 20.0, min_steps: int = 1,
                       max_steps: int = 64, threads: int | None = None):
    """Decode until the time budget is spent; returns (tokens_per_s, steps, seconds, threads)."""
    prev_threads = torch.get_num_threads()
    try:
        dec = StreamingDecoder(w, context + max_steps + 1, threads)
        dec.fill_random_context(context)
        tok = 1
        tok = dec.step(tok)  # untimed warm-up (allocator, thread pool)
        t0 = time.perf_counter()
        n = 0
        while n < max_steps and (n < min_steps or time.perf_counter() - t0 < budget_s):
            tok = dec.step(tok)
            n += 1
        dt = time.perf_counter() - t0
        return n / dt, n, dt, dec.threads
    finally:
        torch.set_num_threads(prev_threads)
