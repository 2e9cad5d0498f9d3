"""Tensor-parallel host logic on CPU ranks (gloo, world size 2; no GPU).

Each rank takes its shard from mlx_dspark_b200.tp.shard_target (the product's sharding) and
runs the oracle's TP decomposition (oracle.tp.TPRef) with gloo all-reduces; the gathered
vocabulary slices must equal the single-process oracle's logits up to the fp32 order of the
partial sums (one bf16 ulp), and the vocabulary-parallel argmax merge must equal the full
argmax. Also checks shard bookkeeping for the 32B shapes at TP 2/4/8.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mlx_dspark_b200.config import QWEN3_32B, TINY
from mlx_dspark_b200.tp import check_divisible, shard_target, vocab_shard
from mlx_dspark_b200.weights import generate_target


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.qwen3 import Qwen3Ref
        from oracle.tp import TPRef, merge_argmax
        torch.set_num_threads(2)
        tw = generate_target(TINY, 0, "cpu")
        shard, v0, valid = shard_target(tw, rank, world)
        ref = TPRef(shard, dist.all_reduce)
        g = torch.Generator().manual_seed(3)
        prompt = torch.randint(0, TINY.vocab_size, (24,), generator=g).tolist()
        cache = ref.make_cache()
        lg, _ = ref.run(prompt[:16], cache)
        lg2, _ = ref.run(prompt[16:], cache)          # a second chunk through the KV cache
        local = torch.cat([lg, lg2])[:, :valid].contiguous()
        parts = [torch.zeros_like(local) for _ in range(world)]
        dist.all_gather(parts, local)
        vals = [p.max(-1).values.tolist() for p in parts]
        idx = [(p.argmax(-1) + i * vocab_shard(TINY.vocab_size, world)[0]).tolist()
               for i, p in enumerate(parts)]
        if rank == 0:
            full = torch.cat(parts, dim=1)
            exp, _ = Qwen3Ref(tw).run(prompt, Qwen3Ref(tw).make_cache())
            ulp = 2.0 ** (exp.abs().clamp(min=1e-30).log2().floor() - 7)
            bad = int(((full - exp).abs() > ulp + 1e-12).sum())
            merged = merge_argmax(vals, idx)
            q.put((bad, merged == [int(i) for i in exp.argmax(-1)], full.shape))
    finally:
        dist.destroy_process_group()


def test_tp2_gloo_ranks_reproduce_the_single_process_forward():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        bad, argmax_ok, shape = q.get(timeout=300)
    finally:
        for p in procs:
            p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    assert shape == (24, TINY.vocab_size)
    assert bad == 0 and argmax_ok


@pytest.mark.parametrize("world", [2, 4, 8])
def test_32b_shard_shapes(world):
    cfg = QWEN3_32B
    check_divisible(cfg, world)
    vs, vpad = vocab_shard(cfg.vocab_size, world)
    assert vpad % 128 == 0 and vs * world >= cfg.vocab_size
    hd = cfg.head_dim
    assert (cfg.num_attention_heads // world + 2 * cfg.num_key_value_heads // world) * hd % 128 == 0
    assert (cfg.intermediate_size // world) % 128 == 0


def test_shard_target_slices_reassemble():
    tw = generate_target(TINY, 0, "cpu")
    shards = [shard_target(tw, r, 2) for r in range(2)]
    L0 = tw.layers[0]
    wq = torch.cat([s[0].layers[0].wq.dequant() for s in shards])
    wo = torch.cat([s[0].layers[0].wo.dequant() for s in shards], dim=1)
    down = torch.cat([s[0].layers[0].down.dequant() for s in shards], dim=1)
    assert torch.equal(wq, L0.wq.dequant()) and torch.equal(wo, L0.wo.dequant())
    assert torch.equal(down, L0.down.dequant())
    head = torch.cat([s[0].head.dequant()[:s[2]] for s in shards])
    assert torch.equal(head, tw.head.dequant())
    assert [s[1] for s in shards] == [0, TINY.vocab_size // 2]
