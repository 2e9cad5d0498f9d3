#!/usr/bin/env python
"""Benchmark of the speculative verify step (BASELINE.json metric: accepted tok/s on
Qwen3-8B W8 with a DSpark drafter; verify-step us; HBM GB/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: Qwen3-8B-arch target, random-init W8 g64 weights (seed 1),
1-layer DSpark drafter with block 8, batch 1, a 1024-token random prompt, greedy decoding,
draft tokens overridden from a seeded Bernoulli(0.7) agree mask over the target's own
greedy continuation (so the mean accept length is set by the mask, as the config asks).

A step is one speculative round: draft (drafter forward + Markov head) -> verify (target
forward over 9 tokens) -> fused acceptance -> drafter context update -> KV commit, replayed
from one CUDA graph. `value` = committed tokens / device time over exactly K rounds with
everything resident in HBM. `e2e` = the same metric through the public
speculative_generate() call, whose host loop copies each round's input token host->device
and reads each round's commit plan device->host. Multi-GPU: one process per GPU, each an
independent replica of the request (request-parallel, no collective), value = sum of
tokens / max over ranks of the device time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "source": "measured"}
    return dict(PEAKS_FALLBACK, source="fallback")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="C2")
    ap.add_argument("--prompt-len", type=int, default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="small run for ncu: short prompt, random reference tokens, no extras")
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    ap.add_argument("--layers", type=int, default=None,
                    help="depth-reduced target (same widths) for profiling captures")
    ap.add_argument("--tp-allreduce", action="store_true",
                    help="under torchrun (2..8 ranks): one row-split projection of the Qwen3-32B "
                         "shapes at M = 9, the fused peer all-reduce against NCCL, one JSON line")
    ap.add_argument("--attention-sweep", action="store_true",
                    help="verify attention alone at 1k/5k/16.9k context (bf16 and KV8), one JSON line")
    ap.add_argument("--serve", action="store_true",
                    help="the continuous-batching workload (C4 shapes: 32 requests, 4 slots per GPU, "
                         "a shared 2048-token prefix, 8-bit KV) over --gpus replicas, one JSON line "
                         "(run as one process; it starts a worker process per GPU)")
    ap.add_argument("--profile-prefill", action="store_true",
                    help="small run for ncu: two prefills of --prompt-len tokens (default 2048) "
                         "through the large-M GEMM, nothing else")
    return ap.parse_args()


# ----------------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def allreduce_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_all(obj, world: int) -> list:
    """Every rank's `obj` (a small JSON-able value), in rank order."""
    if world == 1:
        return [obj]
    import torch.distributed as dist
    out = [None] * world
    dist.all_gather_object(out, obj)
    return out


def cpu_model() -> str:
    """The host CPU's model name (lscpu / /proc/cpuinfo)."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def allreduce_sum(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ----------------------------------------------------------------------------------------
def build_models(wl, seed, layers=None, keep_cpu=True):
    from mlx_dspark_b200.config import TARGETS, dspark_for, with_layers
    from mlx_dspark_b200.model import DSparkDrafter
    from mlx_dspark_b200.target import Target
    from mlx_dspark_b200.weights import generate_dspark, generate_target

    tcfg = TARGETS[wl.target]
    if layers:
        tcfg = with_layers(tcfg, layers)
    dcfg = dspark_for(tcfg, block_size=wl.block_size)
    tw = generate_target(tcfg, seed, "cuda")
    dw = generate_dspark(dcfg, seed, "cuda")
    target = Target(tw, kv_bits=wl.kv_bits)
    drafter = DSparkDrafter(dw, target)
    # the kernels hold packed copies; keep the canonical tensors on the host only
    tw_cpu = tw.to("cpu") if keep_cpu else None
    del tw, dw
    torch.cuda.empty_cache()
    return tw_cpu, target, drafter, dcfg


def gemm_roofline(target, M, reps=5):
    """Time the verify's W8 GEMMs alone (every layer's qkv, o, gate/up, down and the head at
    M rows) with CUDA events; returns (GB/s, algorithmic bytes per pass, us per pass, launches)."""
    from mlx_dspark_b200 import ops
    from mlx_dspark_b200._lib import EPI_RESIDUAL_BF16, EPI_SILU_MUL_F16, EPI_STORE_BF16

    c = target.cfg
    dev = target.device
    x = torch.randn(M, max(c.hidden_size, c.intermediate_size, c.q_dim), device=dev).to(torch.float16)
    h = torch.zeros(M, c.hidden_size, dtype=torch.bfloat16, device=dev)
    qkv = torch.zeros(M, c.qkv_dim, dtype=torch.bfloat16, device=dev)
    act = torch.zeros(M, c.intermediate_size, dtype=torch.float16, device=dev)
    logits = torch.zeros(M, c.vocab_size, dtype=torch.bfloat16, device=dev)
    sc = target.scratch
    H, I = c.hidden_size, c.intermediate_size
    # the residual stream the norm-fused GEMMs read, and its per-tile row sums of squares
    hin = torch.randn(M, H, device=dev).to(torch.bfloat16)
    ss = torch.full((M, H // 128), 128.0, dtype=torch.float32, device=dev)
    eps = c.rms_norm_eps

    def one_pass():
        # the verify forward's GEMM sequence and variants (input RMSNorm fused into q|k|v,
        # gate|up and the head; row sums of squares out of o and down), each warming L2 with the
        # next one's weights
        n = len(target.layers)
        for l, L in enumerate(target.layers):
            nxt = target.layers[l + 1].qkv if l + 1 < n else target.head
            ops.gemm(hin, L.qkv, qkv, epilogue=EPI_STORE_BF16, scratch=sc, M=M, prefetch=L.o,
                     norm=ops.RowNorm(L.input_ln, eps, ss))
            ops.gemm(x[:, :c.q_dim], L.o, h, epilogue=EPI_RESIDUAL_BF16, residual=h, scratch=sc,
                     M=M, prefetch=L.gu, sumsq_out=ss)
            ops.gemm(hin, L.gu, act, epilogue=EPI_SILU_MUL_F16, scratch=sc, M=M,
                     prefetch=L.down, norm=ops.RowNorm(L.post_ln, eps, ss))
            ops.gemm(x[:, :I], L.down, h, epilogue=EPI_RESIDUAL_BF16, residual=h, scratch=sc, M=M,
                     prefetch=nxt, sumsq_out=ss)
        ops.gemm(hin, target.head, logits, epilogue=EPI_STORE_BF16, scratch=sc, M=M,
                 norm=ops.RowNorm(target.norm, eps, ss))

    wbytes = sum(L.qkv.nbytes() + L.o.nbytes() + L.gu.nbytes() + L.down.nbytes()
                 for L in target.layers) + target.head.nbytes()
    act_bytes = 0
    for L in target.layers:
        act_bytes += M * (H * 2 + c.qkv_dim * 2)            # x in, qkv out
        act_bytes += M * (c.q_dim * 2 + H * 2 * 2)          # x in, residual in + out
        act_bytes += M * (H * 2 + I * 2)                    # x in, act out
        act_bytes += M * (I * 2 + H * 2 * 2)
    act_bytes += M * (H * 2 + c.vocab_size * 2)
    one_pass()
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        one_pass()
    e.record()
    torch.cuda.synchronize()
    us = s.elapsed_time(e) * 1000.0 / reps
    total = wbytes + act_bytes
    return total / (us * 1e-6) / 1e9, total, us, 4 * len(target.layers) + 1


def verify_step_us(target, sess, reps=30):
    """Device time of the verify forward + fused acceptance alone (one CUDA graph)."""
    from mlx_dspark_b200 import ops
    from mlx_dspark_b200.generate import capture_graph

    t = target
    B, T = sess.B, sess.T

    def launch():
        t.forward(sess.vbuf, sess.tstate, sess.tap, splits=sess.splits_t)
        ops.accept_greedy(sess.vbuf.logits, B, T, sess.vbuf.ids, sess.argmax, None, False,
                          sess.pending, sess.plan, t.scratch)

    launch()
    torch.cuda.synchronize()
    g = capture_graph(launch)
    g.replay()
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        g.replay()
    e.record()
    torch.cuda.synchronize()
    del g
    return s.elapsed_time(e) * 1000.0 / reps


def read_traffic():
    """Per-launch DRAM traffic of the W8 GEMM from the committed ncu summary, if present."""
    p = os.path.join(ROOT, "profiles", "w8a16_gemm_qwen3_8b_verify.md")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        for line in f:
            if line.strip().startswith("traffic_bytes_per_pass_scaled:"):
                try:
                    return float(line.split(":", 1)[1].strip().split()[0])
                except ValueError:
                    return None
    return None


def cpu_baseline(tw, prompt_len, budget):
    from oracle.cpu_baseline import linear_kind, time_greedy_decode

    cw = tw.to("cpu")
    tps, n, dt, threads = time_greedy_decode(cw, prompt_len, budget_s=budget)
    return {"value": round(tps, 4), "unit": "tok/s", "cores": threads, "kind": "port",
            "cpu": cpu_model(), "os_cpu_count": os.cpu_count(),
            "sample": f"{n} plain greedy decode steps of the Qwen3-8B W8 target at a "
                      f"{prompt_len}-token context (oracle port, fp32 math, {linear_kind()}; "
                      f"KV of the context filled synthetically), {dt:.1f} s"}


def prefill_measure(target, drafter, prompt, reps=2):
    """Prefill of the prompt (target chunks + the drafter's context update, as the decode loops
    run it) timed with CUDA events, and the large-M GEMMs of one chunk timed alone: every
    layer's q|k|v, o, gate|up and down at M = min(prompt, PREFILL_CHUNK) rows (tensor roofline:
    2*M*N*K FLOPs per GEMM)."""
    from mlx_dspark_b200 import ops
    from mlx_dspark_b200._lib import EPI_RESIDUAL_BF16, EPI_SILU_MUL_F16, EPI_STORE_BF16
    from mlx_dspark_b200.generate import SpecSession, prefill_rows
    from mlx_dspark_b200.target import PREFILL_CHUNK

    n = len(prompt)
    times = []
    for _ in range(reps):
        sess = SpecSession(target, drafter, 1, drafter.block_size, n + 64)
        torch.cuda.synchronize()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        prefill_rows(target, prompt, sess.tstate, sess.tap, drafter, sess.cstate)
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
        sess.release()
    target.scratch.check_status()
    c, dev, sc = target.cfg, target.device, target.scratch
    M = min(n, PREFILL_CHUNK)
    H, I = c.hidden_size, c.intermediate_size
    x = torch.randn(M, max(H, I, c.q_dim), device=dev).to(torch.float16)
    h = torch.zeros(M, H, dtype=torch.bfloat16, device=dev)
    qkv = torch.zeros(M, c.qkv_dim, dtype=torch.bfloat16, device=dev)
    act = torch.zeros(M, I, dtype=torch.float16, device=dev)

    def one_pass():
        for L in target.layers:
            ops.gemm_wide(x[:, :H], L.qkv, qkv, epilogue=EPI_STORE_BF16, scratch=sc, M=M)
            ops.gemm_wide(x[:, :c.q_dim], L.o, h, epilogue=EPI_RESIDUAL_BF16, residual=h,
                          scratch=sc, M=M)
            ops.gemm_wide(x[:, :H], L.gu, act, epilogue=EPI_SILU_MUL_F16, scratch=sc, M=M)
            ops.gemm_wide(x[:, :I], L.down, h, epilogue=EPI_RESIDUAL_BF16, residual=h,
                          scratch=sc, M=M)

    flops = 2.0 * M * sum(L.qkv.N * L.qkv.K + L.o.N * L.o.K + L.gu.N * L.gu.K + L.down.N * L.down.K
                          for L in target.layers)
    one_pass()
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    one_pass()
    e.record()
    torch.cuda.synchronize()
    target.scratch.check_status()
    us = s.elapsed_time(e) * 1000.0
    peaks = load_peaks()
    tf = flops / (us * 1e-6) / 1e12
    ms = min(times)
    return {"tokens": n, "ms": round(ms, 2), "tok_s": round(n / (ms / 1000.0), 1),
            "chunk": M, "gemm_us_per_pass": round(us, 1),
            "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peaks["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": round(tf / peaks["bf16_tflops"], 4),
                         "kernel": f"w8a16_wide_kernel (all layers' q|k|v, o, gate|up, down at M={M})",
                         "peak_source": peaks["source"] + " (MEASURED_PEAKS.json bf16_tflops, burst: "
                                        "the GEMMs are timed alone)"}}


def run_tp_allreduce(world, rank):
    """o_proj and down_proj of Qwen3-32B split over `world` ranks at M = 9: GEMM + all-reduce +
    residual add, the fused peer form (dspark_w8a16_gemm_peer + dspark_peer_reduce_residual)
    against GEMM + NCCL all-reduce + dspark_residual_add_f32. 50 calls back to back, twice per
    form, CUDA events, max over ranks."""
    import torch.distributed as dist
    from mlx_dspark_b200 import ops
    from mlx_dspark_b200._lib import EPI_STORE_F32
    from mlx_dspark_b200.tp import PeerAllReduce
    from mlx_dspark_b200.weights import pack, quantize_w8g64

    if world < 2:
        raise SystemExit("--tp-allreduce runs under torchrun with 2..8 ranks")
    dev = torch.device("cuda", torch.cuda.current_device())
    H, M = 5120, 9
    shapes = {"o_proj": (H, 8192 // world), "down_proj": (H, 25600 // world)}
    sc = ops.Scratch(dev)
    peer = PeerAllReduce(rank, world, None, 64, H)
    res = {}
    try:
        for name, (N, K) in shapes.items():
            g = torch.Generator(device=dev).manual_seed(rank * 7 + K)
            w = pack(quantize_w8g64(torch.randn(N, K, generator=g, device=dev) * 0.02), device=dev)
            x = torch.randn(M, K, device=dev, generator=g).to(torch.float16)
            h = torch.zeros(M, H, dtype=torch.bfloat16, device=dev)
            part = torch.zeros(M, H, dtype=torch.float32, device=dev)

            def fused():
                ar = peer.next()
                ops.gemm_peer(x, w, ar, scratch=sc, M=M)
                ops.peer_reduce_residual(h, ar, M, sc)

            def nccl():
                ops.gemm(x, w, part, epilogue=EPI_STORE_F32, scratch=sc, M=M)
                dist.all_reduce(part)
                ops.residual_add_f32(h, part, M)

            for label, fn in (("fused", fused), ("nccl", nccl)) * 2:
                for _ in range(5):
                    fn()
                torch.cuda.synchronize()
                dist.barrier()
                torch.cuda.synchronize()
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                a.record()
                for _ in range(50):
                    fn()
                b.record()
                torch.cuda.synchronize()
                us = torch.tensor([a.elapsed_time(b) * 1000 / 50], device=dev)
                dist.all_reduce(us, op=dist.ReduceOp.MAX)
                res[f"{name}/{label}"] = round(float(us), 2)   # the second pass is kept
            sc.check_status()
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        peer.close()
    if rank == 0:
        print(json.dumps({"metric": "us per row-split projection + all-reduce + residual (M=9)",
                          "unit": "us", "higher_is_better": False, "n_gpus": world,
                          "config": {"model": "Qwen3-32B shapes", "tp": world},
                          "data": "synthetic: random W8 weights and activations", **res}), flush=True)
    import torch.distributed as _d
    _d.destroy_process_group()
    return 0


def run_tp(args, world, rank):
    """C5: one Qwen3-32B W8 request tensor-parallel over the `world` ranks (one process per
    GPU; o_proj / down_proj row-split with an all-reduce after each), DSpark drafting
    replicated on every rank. The same session is timed with the fused peer all-reduce (the
    default) and with NCCL, eager rounds (rounds with collectives are not captured), CUDA
    events, max over ranks."""
    from mlx_dspark_b200 import _lib
    from mlx_dspark_b200.config import TARGETS, WORKLOADS, dspark_for, with_layers
    from mlx_dspark_b200.generate import SpecSession, greedy_generate, prefill_rows, speculative_generate
    from mlx_dspark_b200.model import DSparkDrafter
    from mlx_dspark_b200.tp import TPTarget
    from mlx_dspark_b200.weights import generate_dspark, generate_target

    wl = WORKLOADS[args.workload]
    K, W = args.steps, args.warmup
    dev = torch.device("cuda", torch.cuda.current_device())
    tcfg = TARGETS[wl.target]
    if args.layers:
        tcfg = with_layers(tcfg, args.layers)
    dcfg = dspark_for(tcfg, block_size=wl.block_size)
    tw = generate_target(tcfg, wl.seed, "cuda")
    target = TPTarget(tw, rank, world, kv_bits=wl.kv_bits, device=dev)
    del tw
    drafter = DSparkDrafter(generate_dspark(dcfg, wl.seed, "cuda"), target)
    torch.cuda.empty_cache()
    cap = wl.block_size
    prompt_len = args.prompt_len or wl.prompt_len
    V = tcfg.vocab_size
    prompt = torch.randint(0, V, (prompt_len,), generator=torch.Generator().manual_seed(wl.seed)).tolist()
    rounds = 3 * (K + W) + 4
    ref_len = rounds * (cap + 1) + 16
    ref = greedy_generate(target, None, prompt_ids=prompt, max_new_tokens=ref_len).token_ids
    p_agree = wl.accept_p or 0.7
    agree = (torch.rand(1, max(rounds, 256), cap, generator=torch.Generator().manual_seed(7))
             < p_agree).to(torch.uint8)
    override = {"ref": torch.tensor([ref]), "agree": agree, "prompt_len": [prompt_len]}
    sess = SpecSession(target, drafter, 1, cap, prompt_len + ref_len + 64, override=override)
    last = prefill_rows(target, prompt, sess.tstate, sess.tap, drafter, sess.cstate)
    sess.pending.fill_(target.argmax_row(last))   # (the whole vocabulary's argmax under TP)
    torch.cuda.synchronize()
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    modes, launches = {}, 0
    try:
        for mode in ("fused_graph", "nccl_graph", "fused_eager"):
            # fused_graph (the default): the whole round as one CUDA graph with the fused peer
            # all-reduce; nccl_graph: the same with NCCL all-reduces captured in it;
            # fused_eager: the default's launches without the graph
            target.fused_allreduce = mode.startswith("fused")
            graph = mode.endswith("_graph")
            if graph:
                sess.step(use_graph=False)
                torch.cuda.synchronize()
                barrier(world)
                sess.capture()
            for _ in range(W):
                sess.step(use_graph=graph)
            torch.cuda.synchronize()
            barrier(world)
            len0 = int(sess.tstate.seq_len[0])
            n0 = _lib.LAUNCHES["n"]
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(K):
                sess.step(use_graph=graph)
            b.record()
            torch.cuda.synchronize()
            ms = allreduce_max(a.elapsed_time(b), world)
            tokens = int(sess.tstate.seq_len[0]) - len0
            launches = _lib.LAUNCHES["n"] - n0 if mode == "fused_eager" else launches
            modes[mode] = {"tok_s": round(tokens / (ms / 1000.0), 2),
                           "round_us": round(ms * 1000.0 / K, 1),
                           "mean_accept_len": round(tokens / K, 3)}
        target.scratch.check_status()
        target.fused_allreduce = True
        sess.graph = None
        res = speculative_generate(target, None, drafter, lookup_drafts=False, prompt_ids=prompt,
                                   max_new_tokens=min(128, ref_len - 16), max_draft_tokens=cap,
                                   draft_override=override)
    finally:
        clk = clocks.stop()
        sess.graph = None        # a graph holding NCCL calls goes before the process group
        torch.cuda.synchronize()
        sess.release()
        target.release_peer()
    e2e_tps = allreduce_max((res.num_tokens - 1) / res.decode_seconds, world)
    per_rank = gather_all({"rank": rank, "sm_mhz": clk.get("sm_mhz"), "reasons": clk.get("reasons")},
                          world)
    f = modes["fused_graph"]
    return {
        "metric": "accepted tok/s Qwen3-32B W8 DSpark, one request tensor-parallel over N GPUs",
        "value": f["tok_s"], "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(f["round_us"] / 1000.0, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "w8a16 (int8 weights, fp16 MMA, fp32 accumulate, bf16 activations)",
        "data": "synthetic: random-init W8 g64 weights (seed 1), random prompt ids, "
                "Bernoulli(0.7) draft-agree mask over the target's own greedy continuation",
        "config": {"workload": wl.name, "model": f"Qwen3-32B-arch W8 g64 ({tcfg.num_hidden_layers} "
                   f"layers) + DSpark 1-layer block 8", "global_batch": 1, "prompt_len": prompt_len,
                   "draft_cap": cap, "parallelism": f"tp{world}",
                   "l2": "inputs larger than L2 (32 GB of weights / N per GPU per round)"},
        "round_us": f["round_us"], "mean_accept_len": f["mean_accept_len"],
        "allreduce": {"fused_peer_graph": f, "nccl_graph": modes["nccl_graph"],
                      "fused_peer_eager": modes["fused_eager"]},
        "gpu_launches": launches, "clocks": clk, "per_rank": per_rank,
        "e2e": {"value": round(e2e_tps, 2), "unit": "tok/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4 * (cap + 3),
                "api": "mlx_dspark_b200.speculative_generate (host loop, captured rounds)",
                "rounds": res.num_rounds, "mean_accept_len": round(res.mean_accept_len, 3)},
    }


def run_c3(args, world, rank):
    """C3: Qwen3-4B W8 with the DFlash drafter (2 layers, block 16), sampled at T 1.0,
    top-p 0.95, top-k 50, one request per GPU (replicas under torchrun). Device time of K
    captured rounds (the rejection-sampling acceptance and every draw on the device), then
    the public dflash_generate loop end to end. With random weights the drafter's q and the
    target's p are unrelated, so few drafts are accepted: the line measures the sampled
    round's machinery (draft, verify, accept, residual draws), not speculation."""
    from mlx_dspark_b200 import _lib
    from mlx_dspark_b200.config import TARGETS, WORKLOADS, dflash_for, with_layers
    from mlx_dspark_b200.generate import SpecSession, _pick_first, dflash_generate, prefill_rows
    from mlx_dspark_b200.model import DFlashDrafter, Sampling
    from mlx_dspark_b200.target import Target
    from mlx_dspark_b200.weights import generate_dflash, generate_target

    wl = WORKLOADS["C3"]
    K, W = args.steps, args.warmup
    tcfg = TARGETS[wl.target]
    if args.layers:
        tcfg = with_layers(tcfg, args.layers)
    fcfg = dflash_for(tcfg, block_size=wl.block_size)
    tw = generate_target(tcfg, wl.seed, "cuda")
    target = Target(tw, kv_bits=wl.kv_bits)
    del tw
    drafter = DFlashDrafter(generate_dflash(fcfg, wl.seed, "cuda"), target)
    torch.cuda.empty_cache()
    cap = wl.block_size - 1
    prompt_len = args.prompt_len or wl.prompt_len
    prompt = torch.randint(0, tcfg.vocab_size, (prompt_len,),
                           generator=torch.Generator().manual_seed(wl.seed + rank)).tolist()
    sm = Sampling(wl.temperature, wl.top_p, wl.top_k)
    sess = SpecSession(target, drafter, 1, cap, prompt_len + (K + W + 2) * (cap + 1) + 64,
                       sampling=sm, seeds=[wl.seed + rank])
    last = prefill_rows(target, prompt, sess.tstate, sess.tap, drafter, sess.cstate)
    sess.pending.fill_(_pick_first(target, last, sm, sess.rng))
    n0 = _lib.LAUNCHES["n"]
    sess.step(use_graph=False)
    launches = _lib.LAUNCHES["n"] - n0
    sess.capture()
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    for _ in range(max(0, W - 1)):
        sess.graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    len0 = int(sess.tstate.seq_len[0])
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(K):
        sess.graph.replay()
    b.record()
    torch.cuda.synchronize()
    tokens = int(sess.tstate.seq_len[0]) - len0
    clk = clocks.stop()
    target.scratch.check_status()
    sess.release()
    ms = allreduce_max(a.elapsed_time(b), world)
    value = allreduce_sum(float(tokens), world) / (ms / 1000.0)
    res = dflash_generate(target, None, drafter, prompt_ids=prompt, max_new_tokens=wl.new_tokens,
                          temperature=wl.temperature, top_p=wl.top_p, top_k=wl.top_k,
                          seed=wl.seed + rank)
    e2e = allreduce_sum((res.num_tokens - 1) / res.decode_seconds, world)
    return {
        "metric": "accepted tok/s Qwen3-4B W8 DFlash block 16, sampled (T 1.0, top-p 0.95, top-k 50)",
        "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(ms / K, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "w8a16 (int8 weights, fp16 MMA, fp32 accumulate, bf16 activations)",
        "data": "synthetic: random-init W8 g64 weights (seed 0), random prompt ids; drafts and "
                "acceptance sampled on the device (Philox)",
        "config": {"workload": wl.name, "model": f"Qwen3-4B-arch W8 g64 ({tcfg.num_hidden_layers} "
                   "layers) + DFlash 2-layer block 16", "global_batch": world, "prompt_len": prompt_len,
                   "draft_cap": cap, "parallelism": f"request-parallel x{world} (replicas)",
                   "l2": "inputs larger than L2 (4.4 GB of weights streamed per round)"},
        "round_us": round(ms * 1000.0 / K, 1), "mean_accept_len": round(tokens / K, 3),
        "gpu_launches": launches * K, "clocks": clk,
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 4 * (cap + 3),
                "api": "mlx_dspark_b200.dflash_generate (host loop, one sync per round)",
                "rounds": res.num_rounds, "mean_accept_len": round(res.mean_accept_len, 3)},
    }


def run_attention_sweep(args):
    """Verify attention alone (C2 shape: 1 row, 9 block tokens, 32 q / 8 kv heads, hd 128),
    causal, at 1k, 5k and 16.9k tokens of context, bf16 and 8-bit pages: CUDA events over 200
    back-to-back calls (after 20), µs per call and the KV bytes read per call over that time
    against the measured HBM copy peak."""
    from mlx_dspark_b200 import ops
    from mlx_dspark_b200.kvcache import CacheState, PagePool

    dev = torch.device("cuda", torch.cuda.current_device())
    B, T, Hq, Hkv, hd = 1, 9, 32, 8, 128
    peaks = load_peaks()
    out = {"metric": "verify attention us per call (B 1, T 9, 32q/8kv, hd 128)", "unit": "us",
           "higher_is_better": False, "n_gpus": 1, "data": "synthetic: random q and KV pages",
           "peak_gbs": peaks["hbm_gbs"], "rows": []}
    g = torch.Generator(device=dev).manual_seed(3)
    for kv8 in (False, True):
        for ctx in (1024, 5120, 16896):
            tokens = ctx + T
            pool = PagePool(1, (tokens + 63) // 64 + 1, Hkv, hd, kv8, dev)
            st = CacheState(pool, B, tokens, dev)
            st.ensure(0, tokens)
            if not kv8:  # (8-bit pages stay zero-filled: codes and scales of a valid cache)
                d = pool.data.view(torch.bfloat16)
                d.copy_(torch.randn(d.shape, generator=g, device=dev).to(torch.bfloat16))
            st.seq_len.fill_(ctx)
            q = torch.randn(B * T, Hq * hd, generator=g, device=dev).to(torch.bfloat16)
            o = torch.zeros(B * T, Hq * hd, dtype=torch.float16, device=dev)
            sc = ops.Scratch(dev)
            splits = max(1, min(256, 296 // (B * Hkv)))

            def call():
                ops.attention(q, B, T, Hq, st.layout(0), st.seq_len, True, hd ** -0.5, o, splits, sc)

            for _ in range(20):
                call()
            torch.cuda.synchronize()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(200):
                call()
            b.record()
            torch.cuda.synchronize()
            sc.check_status()
            us = a.elapsed_time(b) * 1000.0 / 200
            per_tok = 2 * Hkv * (hd + (hd // 64) * 4 if kv8 else hd * 2)
            byts = tokens * per_tok
            out["rows"].append({"context": ctx, "kv8": kv8, "us": round(us, 2),
                                "kv_bytes": byts, "gbs": round(byts / us / 1e3, 1),
                                "frac": round(byts / us / 1e3 / peaks["hbm_gbs"], 4)})
            st.release()
    print(json.dumps(out), flush=True)
    return 0


def run_serve(args):
    """C4 continuous batching: 32 requests (a shared random 2048-token prefix plus a random
    64-2048-token suffix, 128-1024 output tokens) over N GPUs, one ReplicaPool worker process
    per GPU (its own Qwen3-8B W8 replica with the 8-bit KV cache, a 4-slot BatchEngine, DSpark
    cap 8, no collective), each request sent to the least-loaded replica. Value = generated
    tokens / wall time from the first submit to the last result, after one warm-up request per
    replica. With random weights the drafts are rejected, so the figure measures the batched
    verify, admission and prefill machinery, not speculation."""
    import functools

    from mlx_dspark_b200.config import TARGETS, WORKLOADS
    from mlx_dspark_b200.engine import ReplicaPool, serving_replica

    wl = WORKLOADS["C4"]
    n = max(1, args.gpus)
    V = TARGETS[wl.target].vocab_size
    g = torch.Generator().manual_seed(4)
    prefix = torch.randint(0, V, (wl.prompt_len,), generator=g).tolist()
    reqs = []
    for _ in range(32):
        sfx = int(torch.randint(64, 2049, (1,), generator=g))
        out = int(torch.randint(128, 1025, (1,), generator=g))
        reqs.append((prefix + torch.randint(0, V, (sfx,), generator=g).tolist(), out))
    slot_tokens = max(len(p) + m for p, m in reqs) + 2 * wl.block_size + 64
    factory = functools.partial(serving_replica, target=wl.target, seed=wl.seed,
                                kv_bits=wl.kv_bits, block_size=wl.block_size,
                                max_batch=wl.batch, slot_tokens=slot_tokens,
                                max_draft_tokens=wl.block_size)
    pool = ReplicaPool(factory, list(range(n)))
    try:
        warm = [pool.submit(prefix[:300], max_tokens=16, temperature=0.0) for _ in range(n)]
        for f in warm:
            f.result()
        pool.assigned = [0] * n
        t0 = time.time()
        futs = [pool.submit(p, max_tokens=m, temperature=0.0) for p, m in reqs]
        res = [f.result() for f in futs]
        dt = time.time() - t0
        assigned = list(pool.assigned)
    finally:
        pool.close()
    toks = sum(r.num_tokens for r in res)
    rounds = sum(r.num_rounds for r in res)
    print(json.dumps({
        "metric": "served tok/s, continuous batching (C4 shapes)", "value": round(toks / dt, 1),
        "unit": "tok/s", "higher_is_better": True, "n_gpus": n, "scaling": "strong",
        "config": {"workload": wl.name, "requests": len(reqs), "slots_per_gpu": wl.batch,
                   "kv_bits": wl.kv_bits, "draft_cap": wl.block_size,
                   "shared_prefix": wl.prompt_len, "dispatch": "least outstanding tokens",
                   "parallelism": f"request-parallel x{n} (one process per GPU)"},
        "data": "synthetic: random-init W8 weights (seed 1), random prompt ids; drafts rejected",
        "tokens": toks, "seconds": round(dt, 2), "requests_per_gpu": assigned,
        "mean_accept_len": round(toks / max(1, rounds), 3),
        "prompt_tokens": sum(len(p) for p, _ in reqs),
        "replicas": {str(k): v.get("batching") for k, v in sorted(pool.replica_metrics.items())},
        "prefix_cache": {str(k): v.get("prefix_cache") for k, v in sorted(pool.replica_metrics.items())}}),
        flush=True)
    return 0


def run_profile_prefill(args):
    """Two prefills of a random prompt (target chunks + drafter context) on one GPU: the
    second one's w8a16_wide launches are the ones an ncu capture skips to."""
    from mlx_dspark_b200.config import WORKLOADS
    from mlx_dspark_b200.generate import SpecSession, prefill_rows

    wl = WORKLOADS[args.workload]
    _, target, drafter, _ = build_models(wl, wl.seed, args.layers, keep_cpu=False)
    n = args.prompt_len or 2048
    prompt = torch.randint(0, target.cfg.vocab_size, (n,),
                           generator=torch.Generator().manual_seed(wl.seed)).tolist()
    for _ in range(2):
        sess = SpecSession(target, drafter, 1, drafter.block_size, n + 64)
        prefill_rows(target, prompt, sess.tstate, sess.tap, drafter, sess.cstate)
        torch.cuda.synchronize()
        sess.release()
    target.scratch.check_status()
    print(json.dumps({"profile_prefill": n, "layers": len(target.layers)}), flush=True)
    return 0


# ----------------------------------------------------------------------------------------
def run_ours(args, world, rank):
    from mlx_dspark_b200 import _lib
    from mlx_dspark_b200.config import WORKLOADS
    from mlx_dspark_b200.generate import SpecSession, greedy_generate, prefill_rows, speculative_generate

    wl = WORKLOADS[args.workload]
    K, W = args.steps, args.warmup
    prompt_len = args.prompt_len or (128 if args.profile else wl.prompt_len)
    cap = wl.block_size
    want_cpu = rank == 0 and world == 1 and not args.no_cpu_baseline and not args.profile
    tw, target, drafter, dcfg = build_models(wl, wl.seed, args.layers, keep_cpu=want_cpu)
    V = target.cfg.vocab_size
    g = torch.Generator().manual_seed(wl.seed)
    prompt = torch.randint(0, V, (prompt_len,), generator=g).tolist()
    rounds = K + W + 2
    ref_len = (K + W + 2) * (cap + 1) + 16
    if args.profile:
        ref = torch.randint(0, V, (ref_len,), generator=g).tolist()
    else:
        ref = greedy_generate(target, None, prompt_ids=prompt, max_new_tokens=ref_len).token_ids
    # one Bernoulli row per round, for the timed rounds and for every round the e2e decode can
    # take (at most one per token); past the last row the override repeats it, which would
    # replace the Bernoulli draw by one fixed pattern. The leading rows do not depend on the count.
    agree_rounds = max(rounds, 512 + cap + 2)
    p_agree = wl.accept_p or 0.7
    expect_len = 1.0 + sum(p_agree ** i for i in range(1, cap + 1))
    agree = (torch.rand(1, agree_rounds, cap, generator=torch.Generator().manual_seed(7)) < p_agree).to(torch.uint8)
    override = {"ref": torch.tensor([ref]), "agree": agree, "prompt_len": [prompt_len]}
    budget = prompt_len + ref_len + 64
    sess = SpecSession(target, drafter, 1, cap, budget, override=override)
    last = prefill_rows(target, prompt, sess.tstate, sess.tap, drafter, sess.cstate)
    sess.pending.fill_(target.argmax_row(last))   # (the whole vocabulary's argmax under TP)
    torch.cuda.synchronize()
    # one eager round (counts launches, sizes every workspace), then capture
    n0 = _lib.LAUNCHES["n"]
    sess.step(use_graph=False)
    launches_per_round = _lib.LAUNCHES["n"] - n0
    sess.capture()
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    for _ in range(max(0, W - 1)):
        sess.graph.replay()
    torch.cuda.synchronize()
    len0 = int(sess.tstate.seq_len[0])
    barrier(world)
    torch.cuda.synchronize()
    ev_s = torch.cuda.Event(enable_timing=True)
    ev_e = torch.cuda.Event(enable_timing=True)
    ev_s.record()
    for _ in range(K):
        sess.graph.replay()
    ev_e.record()
    torch.cuda.synchronize()
    barrier(world)
    ms = ev_s.elapsed_time(ev_e)
    len1 = int(sess.tstate.seq_len[0])
    target.scratch.check_status()
    tokens = len1 - len0
    # verify-step and GEMM roofline (same process, same clocks window)
    vus = verify_step_us(target, sess)
    gbs, gemm_bytes, gemm_us, gemm_launches = gemm_roofline(target, sess.T)
    clk = clocks.stop()
    sess.release()
    max_ms = allreduce_max(ms, world)
    all_tokens = allreduce_sum(float(tokens), world)
    value = all_tokens / (max_ms / 1000.0)
    per_rank = gather_all({"rank": rank, "round_us": round(ms * 1000.0 / K, 1),
                           "accept": round(tokens / K, 3), "verify_us": round(vus, 1),
                           "sm_mhz": clk.get("sm_mhz"), "reasons": clk.get("reasons")}, world)
    peaks = load_peaks()
    out = {
        "metric": "accepted tok/s Qwen3-8B W8 DSpark (1/N GPU); verify-step us; HBM GB/s",
        "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(max_ms / K, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "w8a16 (int8 weights, fp16 MMA, fp32 accumulate, bf16 activations)",
        "data": "synthetic: random-init W8 g64 weights (seed 1), random prompt ids, "
                "Bernoulli(0.7) draft-agree mask over the target's own greedy continuation",
        "config": {"workload": wl.name, "model": "Qwen3-8B-arch W8 g64 + DSpark 1-layer block 8",
                   "global_batch": world, "batch_per_gpu": 1, "prompt_len": prompt_len,
                   "draft_cap": cap, "parallelism": f"request-parallel x{world} (replicas)",
                   "l2": "inputs larger than L2 (8 GB of weights streamed per round)"},
        "mean_accept_len": round(tokens / K, 3),
        "verify_step_us": round(vus, 1),
        "round_us": round(max_ms * 1000.0 / K, 1),
        # tok/s if every round committed the configured expectation, 1 + sum_i p^i over the
        # cap (3.20 at p = 0.7, cap 8): removes the mask sample's noise from the comparison
        "expected_accept_len": round(expect_len, 3),
        "value_at_expected_accept": round(world * expect_len / (max_ms / 1000.0 / K), 2),
        # the north star quotes its targets at a mean accept length of 3.5 (the config's
        # Bernoulli(0.7) mask over cap 8 expects 3.20): tok/s at the measured time per decode
        # round with 3.5 tokens committed per round
        "value_at_accept_3_5": round(world * 3.5 / (max_ms / 1000.0 / K), 2),
        "per_rank": per_rank,
        "verify_hbm_gbs": round(target.weight_bytes() / (vus * 1e-6) / 1e9, 1),
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4),
                     "traffic": read_traffic(), "kernel": "w8a16_tc_kernel (all verify GEMMs, M=9)",
                     "bytes_per_pass": gemm_bytes, "us_per_pass": round(gemm_us, 1),
                     "launches_per_pass": gemm_launches,
                     "peak_source": peaks["source"] + " (MEASURED_PEAKS.json hbm_gbs)"},
        "gpu_launches": launches_per_round * K,
        "clocks": clk,
    }
    if not args.no_e2e and not args.profile:
        res = speculative_generate(target, None, drafter, lookup_drafts=False, prompt_ids=prompt,
                                   max_new_tokens=min(512, ref_len - 16), max_draft_tokens=cap,
                                   draft_override=override)
        e2e_tps = (res.num_tokens - 1) / res.decode_seconds
        e2e_all = allreduce_sum(e2e_tps, world)
        hist = {}
        for n in res.accept_lengths:
            hist[str(n)] = hist.get(str(n), 0) + 1
        out["e2e"] = {"value": round(e2e_all, 2), "unit": "tok/s",
                      "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4 * (cap + 3),
                      "api": "mlx_dspark_b200.speculative_generate (host loop, one sync per round)",
                      "rounds": res.num_rounds, "mean_accept_len": round(res.mean_accept_len, 3),
                      "committed_per_round": dict(sorted(hist.items(), key=lambda kv: int(kv[0]))),
                      "prefill_s": round(res.seconds - res.decode_seconds, 3)}
    if not args.profile:
        out["prefill"] = prefill_measure(target, drafter, prompt)
    if want_cpu:
        out["cpu_baseline"] = cpu_baseline(tw, prompt_len, args.cpu_budget)
    return out


def run_reference(args, world, rank):
    """The reference arm: the reference's CPU implementation of this path on the host cores.
    MLX cannot be installed here, so it is the oracle port (plain greedy decode, the
    north-star's 'plain MLX-CPU decode' baseline); each step is one decode token."""
    if rank != 0:
        return None
    from mlx_dspark_b200.config import TARGETS, WORKLOADS
    from mlx_dspark_b200.weights import generate_target
    from oracle.cpu_baseline import StreamingDecoder, linear_kind

    wl = WORKLOADS[args.workload]
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    tw = generate_target(TARGETS[wl.target], wl.seed, dev).to("cpu")
    if dev == "cuda":
        torch.cuda.empty_cache()
    K = args.steps
    W = min(args.warmup, 1)
    dec = StreamingDecoder(tw, wl.prompt_len + K + W + 2)
    dec.fill_random_context(wl.prompt_len)
    tok = 1
    for _ in range(W):
        tok = dec.step(tok)
    budget = 150.0
    t0 = time.perf_counter()
    n = 0
    while n < K and time.perf_counter() - t0 < budget:
        tok = dec.step(tok)
        n += 1
    dt = time.perf_counter() - t0
    v = n / dt
    return {
        "impl": "reference", "metric": "accepted tok/s Qwen3-8B W8 DSpark (1/N GPU); verify-step us; HBM GB/s",
        "value": round(v, 4), "unit": "tok/s", "n_gpus": world, "steps": n, "steps_requested": K,
        "warmup": W, "ms_per_step": round(dt * 1000 / max(n, 1), 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32 math over int8 + bf16 weights",
        "data": "synthetic (same weights and context length as the GPU arm)",
        "config": {"workload": wl.name, "model": "Qwen3-8B-arch W8 g64 (plain greedy decode)",
                   "global_batch": 1, "prompt_len": wl.prompt_len, "parallelism": "host cores"},
        "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": dec.threads, "kind": "port",
                         "cpu": cpu_model(), "os_cpu_count": os.cpu_count(),
                         "sample": f"{n} greedy decode steps at a {wl.prompt_len}-token context "
                                   f"(mlx absent: oracle port of greedy_generate, "
                                   f"{linear_kind()}), {dt:.1f} s"},
        "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main():
    args = parse()
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        out = run_reference(args, world, rank)
        if out is not None:
            print(json.dumps(out), flush=True)
        return 0
    if args.serve:
        return run_serve(args)       # one process per GPU of its own (ReplicaPool)
    if args.attention_sweep:
        torch.cuda.set_device(0)
        return run_attention_sweep(args)
    world, rank, _ = dist_setup(args.gpus)
    if args.profile_prefill:
        return run_profile_prefill(args)
    if args.tp_allreduce:
        return run_tp_allreduce(world, rank)
    try:
        if args.workload == "C5" and world > 1:
            out = run_tp(args, world, rank)
        elif args.workload == "C3":
            out = run_c3(args, world, rank)
        else:
            out = run_ours(args, world, rank)
        if rank == 0:
            print(json.dumps(out), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
