"""The persistent multi-GEMM launch (dspark_w8a16_stream) against the separate launches it
replaces: the same grid and work split, with split tiles summed in 64-bit fixed point rather
than ordered fp32. Checked here with a tolerance of a few bf16 ulps of the row scale (2^-6),
and for exact repetition.

Checked on the tiny config through Target.run (bf16 and 8-bit KV, with hidden-state taps,
against the CPU oracle too: bf16 rtol 2e-2 of the row scale) and on a depth-reduced Qwen3-8B-
width target at the verify widths (M = 1, 9 and 36 rows: the BN 16 and BN 48 instances),
comparing logits, taps, q, the new KV rows and the residual stream.

Tile-ready chaining of the single-GEMM launches (each GEMM waits on the previous GEMM's
finished-tile count instead of its grid's completion) changes no arithmetic: its forward must be
bit-identical to the unchained one."""
import pytest
import torch

from mlx_dspark_b200.config import QWEN3_8B, TINY, dspark_for, with_layers
from mlx_dspark_b200.kvcache import CacheState
from mlx_dspark_b200.load import load_target
from mlx_dspark_b200.weights import generate_target
from oracle.qwen3 import Qwen3Ref

pytestmark = pytest.mark.gpu


def _close(a, b, tol=2.0 ** -6):
    a, b = a.float(), b.float()
    scale = b.abs().amax(-1, keepdim=True) + 1e-6
    return float(((a - b).abs() / scale).max()) <= tol


def test_stream_grid_matches_the_single_gemm_grid(cuda):
    from mlx_dspark_b200 import ops
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    assert ops.stream_grid(9) == ops.stream_grid(32) == 2 * sms
    assert ops.stream_grid(36) == ops.stream_grid(64) == sms


@pytest.mark.parametrize("layers,kv", [(1, None), (4, None), (4, 8)])
def test_stream_forward_matches_separate_kernels_and_oracle(cuda, layers, kv):
    cfg = with_layers(TINY, layers)
    tw = generate_target(cfg, 0, "cpu")
    target, _ = load_target(cfg, weights=tw, kv_bits=kv, device=cuda)
    tap = [t for t in dspark_for(TINY).target_layer_ids if t < layers]
    g = torch.Generator().manual_seed(11)
    prompt = torch.randint(0, TINY.vocab_size, (90,), generator=g).tolist()
    out = {}
    for stream in (True, False):
        target.use_stream = stream
        cache = target.make_cache(512)
        parts = [target.run([prompt[a:b]], cache, tap) for a, b in ((0, 40), (40, 49), (49, 90))]
        out[stream] = (torch.cat([p[0][0] for p in parts]).float().cpu(),
                       torch.cat([p[1][0] for p in parts]).float().cpu() if tap else None)
    del target.use_stream
    target.scratch.check_status()
    assert _close(out[True][0], out[False][0])
    if tap:
        assert _close(out[True][1], out[False][1])
    ref = Qwen3Ref(tw)
    rl, rf = ref.run(prompt, ref.make_cache(kv == 8), tap)
    pairs = [("logits", out[True][0], rl)] + ([("taps", out[True][1], rf)] if tap else [])
    for name, a, b in pairs:
        sc = b.abs().amax(-1, keepdim=True)
        err = float(((a - b).abs() / sc).max())
        assert err <= 2e-2, (name, err)


@pytest.mark.parametrize("B,T", [(1, 1), (1, 9), (4, 9)])
def test_stream_bit_identical_at_qwen3_8b_width(cuda, B, T):
    cfg = with_layers(QWEN3_8B, 2)
    tw = generate_target(cfg, 1, "cuda")
    target, _ = load_target(cfg, weights=tw, device=cuda)
    del tw
    tap = [0, 1]
    g = torch.Generator(device=cuda).manual_seed(3)
    ids = torch.randint(0, cfg.vocab_size, (B * T,), generator=g, device=cuda, dtype=torch.int32)
    lens = torch.tensor([37, 64, 100, 5][:B], dtype=torch.int32)
    res = {}
    for mode in ("stream", "chained", "plain"):
        stream = mode == "stream"
        target.use_stream = stream
        target.chain_gemms = mode == "chained"
        st = CacheState(target.new_pool(256, B), B, 256, cuda)
        for b in range(B):
            st.ensure(b, 256)
        # identical random history in the cache of both runs
        gen = torch.Generator(device=cuda).manual_seed(5)
        d = st.pool.data.view(torch.bfloat16)   # bf16 pages: finite random history
        d.copy_(torch.randn(d.shape, generator=gen, device=cuda) * 0.5)
        st.seq_len.copy_(lens.to(cuda))
        buf = target.buffers(B, T, len(tap))
        buf.ids.copy_(ids)
        target.forward(buf, st, tap)
        again = None
        if stream:   # the stream form repeats exactly (its counters are left at zero)
            l0 = buf.logits.clone()
            target.forward(buf, st, tap)
            again = torch.equal(l0, buf.logits)
        torch.cuda.synchronize()
        kv = st.pool.data.view(torch.bfloat16).clone()
        res[mode] = ([t.clone() for t in (buf.logits, buf.fused16, buf.q, buf.h)], kv, again)
        st.release()
    del target.use_stream, target.chain_gemms
    target.scratch.check_status()
    assert res["stream"][2]
    for a, b in zip(res["stream"][0], res["plain"][0]):
        assert _close(a, b)
    for a, b in zip(res["chained"][0], res["plain"][0]):
        assert torch.equal(a, b)
    assert torch.equal(res["chained"][1], res["plain"][1])
    # the cache pages: history untouched, the new rows within the same tolerance
    ka, kb = res["stream"][1], res["plain"][1]
    assert _close(ka.reshape(-1, 128), kb.reshape(-1, 128))
