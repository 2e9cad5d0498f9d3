"""The prefill path on the GPU: the large-M W8A16 GEMM (dspark_w8a16_gemm_wide) against the
fp16-weight bound of the CPU product, its epilogues, and a chunked prefill through it against
the verify-forward prefill and the oracle (prefill chunks, src/mlx_dspark/generate.py:613-656)."""
import pytest
import torch

from mlx_dspark_b200 import generate, ops
from mlx_dspark_b200._lib import (EPI_RESIDUAL_BF16, EPI_SILU_MUL_F16, EPI_STORE_BF16,
                                  EPI_STORE_F32)
from mlx_dspark_b200.config import TINY, dspark_for
from mlx_dspark_b200.generate import SpecSession, prefill_rows
from mlx_dspark_b200.load import drafter_for, load_target
from mlx_dspark_b200.weights import generate_dspark, generate_target, pack, quantize_w8g64
from oracle import qwen3 as oq
from oracle.qwen3 import Qwen3Ref

pytestmark = pytest.mark.gpu


def _qrand(N, K, seed):
    g = torch.Generator().manual_seed(seed)
    return quantize_w8g64(torch.randn(N, K, generator=g) * 0.02)


def _x16(M, K, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed + 7)
    return (torch.randn(M, K, generator=g) * scale).to(torch.bfloat16).to(torch.float32)


WIDE_SHAPES = [
    (1, 128, 64), (65, 256, 128), (129, 384, 640), (300, 256, 4096), (1000, 1024, 1024),
    (2048, 512, 4096), (257, 6144, 256), (511, 128, 12288),
]


@pytest.fixture()
def force_bn():
    """Force the prefill GEMM's tokens per tile for one test, then restore the automatic pick."""
    yield ops.gemm_wide_bn
    ops.gemm_wide_bn(0)


def test_gemm_wide_tile_width_rule():
    """128 tokens per tile for short calls or few tiles, 256 otherwise (measured on B200)."""
    for M, N, want in [(1, 128, 128), (256, 24576, 128), (512, 4096, 128), (512, 6144, 256),
                       (768, 4096, 256), (1024, 4096, 256), (2048, 512, 128), (257, 6144, 256)]:
        assert ops.gemm_wide_plan(M, N, 4096)["bn"] == want, (M, N)


@pytest.mark.parametrize("bn", [128, 256])
@pytest.mark.parametrize("M,N,K", WIDE_SHAPES)
def test_gemm_wide_matches_fp32_bound(cuda, force_bn, M, N, K, bn):
    """fp32 outputs inside the fp16-weight bound (as the verify GEMM's test), deterministic
    across calls, at both tile widths."""
    force_bn(bn)
    qt = _qrand(N, K, seed=M * 31 + N + K)
    w = pack(qt, device=cuda)
    x = _x16(M, K, seed=N + K)
    ref = x @ qt.dequant().t()
    bound = (x.abs() @ qt.dequant().abs().t()) * 2.0 ** -10 + 1e-5
    sc = ops.Scratch(cuda)
    x16 = x.to(torch.float16).to(cuda)
    ys = []
    for _ in range(2):
        y = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
        ops.gemm_wide(x16, w, y, epilogue=EPI_STORE_F32, scratch=sc)
        ys.append(y)
    torch.cuda.synchronize()
    sc.check_status()
    err = (ys[0].cpu() - ref).abs()
    bad = ~(err <= bound)
    if bad.any():
        idx = bad.nonzero()[:8].tolist()
        pytest.fail(f"{int(bad.sum())} of {M*N} outside bound; first {idx}; "
                    f"max err {err.max():.3e}, ref max {ref.abs().max():.3e}")
    assert torch.equal(ys[0], ys[1])
    plan = ops.gemm_wide_plan(M, N, K)
    assert plan["bn"] == bn and plan["grid"] >= 1


@pytest.mark.parametrize("bn", [128, 256])
def test_gemm_wide_kmap_diagnostic(cuda, force_bn, bn):
    """One-hot activation rows read single weight columns, Y[m, n] = W[n, k_m], at rows in
    several token tiles: pins the k <-> TMEM column mapping of the converter, the 64-byte
    swizzle of the weight tile and the activation-row addressing."""
    force_bn(bn)
    N, K = 256, 256
    ks = [0, 1, 2, 7, 8, 15, 16, 31, 32, 47, 63, 64, 65, 100, 127, 128, 191, 200, 255]
    M = 600
    qt = _qrand(N, K, 5)
    w = pack(qt, device=cuda)
    x = torch.zeros(M, K)
    rows = {}
    for i, k in enumerate(ks):
        for m in (i, 255 - i, 256 + 3 * i, M - 1 - i):
            x[m, k] = 1.0
            rows[m] = k
    y = torch.zeros(M, N, dtype=torch.float32, device=cuda)
    ops.gemm_wide(x.to(torch.float16).to(cuda), w, y, epilogue=EPI_STORE_F32,
                  scratch=ops.Scratch(cuda))
    torch.cuda.synchronize()
    Wd = qt.dequant()
    yc = y.cpu()
    for m, k in rows.items():
        err = (yc[m] - Wd[:, k]).abs().max()
        assert err <= Wd.abs().max() * 2 ** -10 + 1e-6, (m, k, float(err))
    zero = [m for m in range(M) if m not in rows]
    assert yc[zero].abs().max() == 0


@pytest.mark.parametrize("M,H,I", [(100, 512, 1536), (700, 1024, 2048), (257, 4096, 1024)])
def test_gemm_wide_epilogues(cuda, M, H, I):
    """SiLU(gate) * up (interleaved pack) -> fp16, then down with the residual add in place and
    the fp16 tap copy, then a bf16 store: the verify GEMM's epilogue arithmetic and bounds."""
    sc = ops.Scratch(cuda)
    g, u, d = _qrand(I, H, 11), _qrand(I, H, 12), _qrand(H, I, 13)
    x = _x16(M, H, 14)
    r = torch.randn(M, H, generator=torch.Generator().manual_seed(19)).to(torch.bfloat16)
    wgu = pack(g, u, interleave64=True, device=cuda)
    act = torch.zeros(M, I, dtype=torch.float16, device=cuda)
    ops.gemm_wide(x.to(torch.float16).to(cuda), wgu, act, epilogue=EPI_SILU_MUL_F16, scratch=sc)
    gg = oq.bf(x @ g.dequant().t())
    uu = oq.bf(x @ u.dequant().t())
    ref_act = oq.bf(oq.bf(oq.silu(gg)) * uu)
    torch.cuda.synchronize()
    got = act.float().cpu()
    bg = (x.abs() @ g.dequant().abs().t()) * 2.0 ** -10 + gg.abs() * 2.0 ** -7
    bu = (x.abs() @ u.dequant().abs().t()) * 2.0 ** -10 + uu.abs() * 2.0 ** -7
    bound = 1.1 * bg * uu.abs() + oq.silu(gg).abs() * bu + bg * bu + ref_act.abs() * 2.0 ** -7 + 1e-6
    assert ((got - ref_act).abs() <= bound).all(), ((got - ref_act).abs() / bound).max()
    wd = pack(d, device=cuda)
    h = r.clone().to(cuda)
    tap = torch.zeros(M, 2 * H, dtype=torch.float16, device=cuda)
    ops.gemm_wide(act, wd, h, epilogue=EPI_RESIDUAL_BF16, residual=h, scratch=sc,
                  copy16=tap[:, H:])
    dd = got @ d.dequant().t()
    ref_h = oq.bf(r.float() + oq.bf(dd))
    torch.cuda.synchronize()
    bh = (got.abs() @ d.dequant().abs().t()) * 2.0 ** -10 + (dd.abs() + ref_h.abs()) * 2.0 ** -7 + 1e-6
    hc = h.float().cpu()
    assert ((hc - ref_h).abs() <= bh).all(), ((hc - ref_h).abs() / bh).max()
    assert torch.equal(tap[:, H:].float().cpu(), hc) and tap[:, :H].abs().max() == 0
    # bf16 store: the rounding of the fp32 product
    yb = torch.zeros(M, I, dtype=torch.bfloat16, device=cuda)
    yf = torch.zeros(M, I, dtype=torch.float32, device=cuda)
    wg = pack(g, device=cuda)
    ops.gemm_wide(x.to(torch.float16).to(cuda), wg, yb, epilogue=EPI_STORE_BF16, scratch=sc)
    ops.gemm_wide(x.to(torch.float16).to(cuda), wg, yf, epilogue=EPI_STORE_F32, scratch=sc)
    torch.cuda.synchronize()
    sc.check_status()
    assert torch.equal(yb.cpu(), yf.cpu().to(torch.bfloat16))


@pytest.fixture(scope="module")
def tiny_pair(cuda):
    tw = generate_target(TINY, 3, "cpu")
    dcfg = dspark_for(TINY)
    dw = generate_dspark(dcfg, 3, "cpu")
    target, _ = load_target(TINY, weights=tw, device=cuda)
    drafter, _ = drafter_for(target, dcfg, weights=dw, device=cuda)
    return tw, target, drafter


def _kv_rows(state, layer: int, n: int):
    """K and V [Hkv, n, hd] (fp32) of row 0's first n positions in a bf16 page pool."""
    pool = state.pool
    assert not pool.kv8
    npg = (n + 63) // 64
    pages = state.block_table[0, :npg].tolist()
    d = pool.data[layer, pages].view(torch.bfloat16).view(npg, 2, pool.num_kv_heads, 64,
                                                          pool.head_dim)
    kv = d.permute(1, 2, 0, 3, 4).reshape(2, pool.num_kv_heads, npg * 64, pool.head_dim)[:, :, :n]
    return kv[0].float().cpu(), kv[1].float().cpu()


@pytest.mark.parametrize("n,chunk", [(600, 256), (572, 256), (130, 2048)])
def test_prefill_wide_matches_verify_forward(tiny_pair, monkeypatch, n, chunk):
    """prefill_rows through the large-M path (chunks of `chunk` tokens; a short tail takes the
    verify forward) against the verify-forward prefill (32-token chunks): the same last-row
    logits, and the same target and drafter-context KV (bf16 roundings of the same sums taken
    in another order). Each path is held to 2e-2 of the row scale against the oracle elsewhere
    (the end-to-end tolerance); two such paths may sit on opposite sides of it, so they are
    compared here at 4e-2 (deep layers measured 0.021: single bf16 ulps accumulated through
    the residual stream)."""
    tw, target, drafter = tiny_pair
    g = torch.Generator().manual_seed(n)
    prompt = torch.randint(0, TINY.vocab_size, (n,), generator=g).tolist()
    out = {}
    for mode in ("wide", "narrow"):
        monkeypatch.setattr(generate, "PREFILL_CHUNK", chunk)
        monkeypatch.setattr(target, "wide_min_tokens", 64 if mode == "wide" else 10 ** 9)
        sess = SpecSession(target, drafter, 1, 8, n + 64)
        last = prefill_rows(target, prompt, sess.tstate, sess.tap, drafter, sess.cstate)
        torch.cuda.synchronize()
        target.scratch.check_status()
        kv = [_kv_rows(sess.tstate, l, n) for l in range(TINY.num_hidden_layers)]
        ckv = [_kv_rows(sess.cstate, l, n) for l in range(len(drafter.layers))]
        out[mode] = (last.float().cpu(), kv, ckv, sess.tstate.seq_len.item(),
                     sess.cstate.seq_len.item())
        sess.release()
    (lw, kw, cw, tw_len, cw_len), (ln, kn, cn, tn_len, cn_len) = out["wide"], out["narrow"]
    assert tw_len == tn_len == n and cw_len == cn_len == n
    sc = ln.abs().max()
    assert ((lw - ln).abs() <= 4e-2 * sc).all(), float((lw - ln).abs().max() / sc)
    for (a, b), (c, d) in zip(kw + cw, kn + cn):
        for x, y in ((a, c), (b, d)):
            s = y.abs().amax(-1, keepdim=True) + 1e-6
            assert ((x - y).abs() <= 4e-2 * s).all(), float(((x - y).abs() / s).max())


def test_prefill_wide_matches_oracle(tiny_pair, monkeypatch):
    """Target.run over 700 tokens (chunks of 256: every chunk on the large-M path) against the
    oracle's chunked prefill: every row's logits within bf16 rtol 2e-2 of the row scale (the
    north star's output tolerance); the taps, hidden states of the residual stream that only
    condition the drafter, within 3e-2 (700 positions of bf16 rounding differences in the
    attention and norm orders accumulate in them)."""
    tw, target, _ = tiny_pair
    import mlx_dspark_b200.target as tmod
    monkeypatch.setattr(tmod, "PREFILL_CHUNK", 256)
    g = torch.Generator().manual_seed(700)
    prompt = torch.randint(0, TINY.vocab_size, (700,), generator=g).tolist()
    tap = (1, 2, 3)
    cache = target.make_cache(1024)
    logits, fused = target.run([prompt], cache, tap)
    ref = Qwen3Ref(tw)
    rc = ref.make_cache()
    rl, rf = ref.run(prompt, rc, tap)
    gl = logits[0].float().cpu()
    s = rl.abs().amax(-1, keepdim=True)
    assert ((gl - rl).abs() <= 2e-2 * s).all(), float(((gl - rl).abs() / s).max())
    gf = fused[0].float().cpu()
    fs = rf.abs().amax(-1, keepdim=True)
    assert ((gf - rf).abs() <= 3e-2 * fs).all(), float(((gf - rf).abs() / fs).max())


def test_prefill_wide_kv8_matches_verify_forward(cuda, monkeypatch):
    """The same comparison with the 8-bit KV cache (C4's cache): chunks quantize K/V on write
    through the same kernel, and the last-row logits of the two prefill paths agree."""
    tw = generate_target(TINY, 4, "cpu")
    target, _ = load_target(TINY, weights=tw, device=cuda, kv_bits=8)
    dcfg = dspark_for(TINY)
    drafter, _ = drafter_for(target, dcfg, weights=generate_dspark(dcfg, 4, "cpu"), device=cuda)
    prompt = torch.randint(0, TINY.vocab_size, (400,),
                           generator=torch.Generator().manual_seed(4)).tolist()
    lasts = {}
    for mode in ("wide", "narrow"):
        monkeypatch.setattr(generate, "PREFILL_CHUNK", 192)
        monkeypatch.setattr(target, "wide_min_tokens", 64 if mode == "wide" else 10 ** 9)
        sess = SpecSession(target, drafter, 1, 8, 464)
        assert sess.tstate.pool.kv8
        lasts[mode] = prefill_rows(target, prompt, sess.tstate, sess.tap, drafter,
                                   sess.cstate).float().cpu()
        torch.cuda.synchronize()
        target.scratch.check_status()
        sess.release()
    sc = lasts["narrow"].abs().max()
    assert ((lasts["wide"] - lasts["narrow"]).abs() <= 4e-2 * sc).all()
