"""GPU parity of each kernel against the CPU oracle (and of the tcgen05 GEMM against a
rigorous per-element bound and the CUDA-core cross-check kernel)."""
import math

import pytest
import torch

from mlx_dspark_b200 import ops
from mlx_dspark_b200._lib import (EPI_RESIDUAL_BF16, EPI_SILU_MUL_F16, EPI_STORE_BF16,
                                  EPI_STORE_F32)
from mlx_dspark_b200.kvcache import PAGE, CacheState, PagePool
from mlx_dspark_b200.weights import pack, quantize_w8g64
from oracle import qwen3 as oq

pytestmark = pytest.mark.gpu


def _qrand(N, K, seed):
    g = torch.Generator().manual_seed(seed)
    return quantize_w8g64(torch.randn(N, K, generator=g) * 0.02)


def _x16(M, K, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed + 7)
    x = (torch.randn(M, K, generator=g) * scale).to(torch.bfloat16).to(torch.float32)
    return x  # bf16 values (exact in fp16)


GEMM_SHAPES = [
    (1, 128, 128), (9, 768, 512), (16, 1024, 4096), (17, 512, 256), (9, 6144, 4096),
    (36, 4096, 1024), (64, 256, 12288), (8, 32768, 512), (3, 128, 6144), (48, 2048, 2048),
]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_w8a16_gemm_tc_matches_fp32_bound(cuda, M, N, K):
    qt = _qrand(N, K, seed=M * 131 + N + K)
    w = pack(qt, device=cuda)
    x = _x16(M, K, seed=N)
    ref = x @ qt.dequant().t()
    # fp16 dequant rounds each weight to half an fp16 ulp (2^-11 relative) and the inputs
    # are exact; fp32 accumulation error is far below that.
    bound = (x.abs() @ qt.dequant().abs().t()) * 2.0 ** -10 + 1e-5
    sc = ops.Scratch(cuda)
    y = torch.zeros(M, N, dtype=torch.float32, device=cuda)
    ops.gemm(x.to(torch.float16).to(cuda), w, y, epilogue=EPI_STORE_F32, scratch=sc)
    torch.cuda.synchronize()
    sc.check_status()
    err = (y.cpu() - ref).abs()
    bad = err > bound
    if bad.any():
        idx = bad.nonzero()[:8].tolist()
        pytest.fail(f"{int(bad.sum())} of {M*N} outside bound; first {idx}; "
                    f"max err {err.max():.3e}, ref max {ref.abs().max():.3e}")
    # second call reuses the workspace counters (left at zero by the first)
    y3 = torch.zeros_like(y)
    ops.gemm(x.to(torch.float16).to(cuda), w, y3, epilogue=EPI_STORE_F32, scratch=sc)
    torch.cuda.synchronize()
    assert torch.equal(y3, y), "stream-K reduction must be deterministic across calls"


def test_w8a16_gemm_kmap_diagnostic(cuda):
    """One-hot activations read single weight columns: Y[m, n] = W[n, k_m]. Pins the
    k <-> TMEM column mapping of the converter and the B-operand swizzle addressing."""
    M, N, K = 16, 256, 256
    qt = _qrand(N, K, 5)
    w = pack(qt, device=cuda)
    ks = [0, 1, 2, 7, 8, 15, 16, 31, 63, 64, 65, 100, 127, 128, 200, 255]
    x = torch.zeros(M, K)
    for m, k in enumerate(ks):
        x[m, k] = 1.0
    y = torch.zeros(M, N, dtype=torch.float32, device=cuda)
    ops.gemm(x.to(torch.float16).to(cuda), w, y, epilogue=EPI_STORE_F32, scratch=ops.Scratch(cuda))
    torch.cuda.synchronize()
    Wd = qt.dequant()
    exp = Wd[:, ks].t()  # [M, N]
    err = (y.cpu() - exp).abs().max(dim=1).values
    assert (err <= exp.abs().max() * 2 ** -10 + 1e-6).all(), f"per-k max err {err.tolist()}"


@pytest.mark.parametrize("M,H,I", [(9, 512, 1536), (36, 1024, 2048), (1, 256, 384),
                                   (9, 4096, 2048)])
def test_gemm_residual_and_silu_epilogues(cuda, M, H, I):
    sc = ops.Scratch(cuda)
    g, u, d = _qrand(I, H, 1), _qrand(I, H, 2), _qrand(H, I, 3)
    x = _x16(M, H, 4)
    r = (torch.randn(M, H, generator=torch.Generator().manual_seed(9))).to(torch.bfloat16)
    # gate/up with SiLU * up (interleaved pack) -> fp16 [M, I]
    wgu = pack(g, u, interleave64=True, device=cuda)
    act = torch.zeros(M, I, dtype=torch.float16, device=cuda)
    ops.gemm(x.to(torch.float16).to(cuda), wgu, act, epilogue=EPI_SILU_MUL_F16, scratch=sc)
    gg = oq.bf(x @ g.dequant().t())
    uu = oq.bf(x @ u.dequant().t())
    ref_act = oq.bf(oq.bf(oq.silu(gg)) * uu)
    torch.cuda.synchronize()
    got = act.float().cpu()
    # per-element bound: the fp16 weight rounding bounds |dg| and |du| by 2^-10 sum|x||w|
    # (as in the GEMM test), each then rounded to bf16; silu' <= 1.1; three bf16 roundings
    bg = (x.abs() @ g.dequant().abs().t()) * 2.0 ** -10 + gg.abs() * 2.0 ** -7
    bu = (x.abs() @ u.dequant().abs().t()) * 2.0 ** -10 + uu.abs() * 2.0 ** -7
    bound = 1.1 * bg * uu.abs() + oq.silu(gg).abs() * bu + bg * bu + ref_act.abs() * 2.0 ** -7 + 1e-6
    assert ((got - ref_act).abs() <= bound).all(), ((got - ref_act).abs() / bound).max()
    # down with the residual epilogue, in place on r
    wd = pack(d, device=cuda)
    h = r.clone().to(cuda)
    ops.gemm(act, wd, h, epilogue=EPI_RESIDUAL_BF16, residual=h, scratch=sc)
    dd = got @ d.dequant().t()
    ref_h = oq.bf(r.float() + oq.bf(dd))
    torch.cuda.synchronize()
    bh = (got.abs() @ d.dequant().abs().t()) * 2.0 ** -10 + (dd.abs() + ref_h.abs()) * 2.0 ** -7 + 1e-6
    assert ((h.float().cpu() - ref_h).abs() <= bh).all(), ((h.float().cpu() - ref_h).abs() / bh).max()


@pytest.mark.parametrize("M,H,N", [(9, 4096, 1024), (1, 1024, 512), (33, 2048, 256),
                                   (64, 512, 384)])
def test_gemm_fused_rmsnorm_and_row_sumsq(cuda, M, H, N):
    """The residual epilogue's per-tile row sums of squares are the sums of the squares of the
    bf16 rows it wrote, and a GEMM fed the raw residual stream with the fused RMSNorm matches
    dspark_rmsnorm + GEMM to one bf16 rounding of its inputs (the squares are summed in another
    fp32 order, so 1/rms may differ in its last bits)."""
    sc = ops.Scratch(cuda)
    Kd = 512
    d = _qrand(H, Kd, 11)
    x = _x16(M, Kd, 3).to(torch.float16).to(cuda)
    r0 = torch.randn(M, H, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    h = r0.clone().to(cuda)
    ss = torch.zeros(M, H // 128, dtype=torch.float32, device=cuda)
    tap = torch.zeros(M, 2 * H, dtype=torch.float16, device=cuda)  # the copy lands in a column slice
    ops.gemm(x, pack(d, device=cuda), h, epilogue=EPI_RESIDUAL_BF16, residual=h, scratch=sc,
             sumsq_out=ss, copy16=tap[:, H:])
    torch.cuda.synchronize()
    sc.check_status()
    hf = h.float().cpu().double()
    ref_ss = (hf ** 2).reshape(M, H // 128, 128).sum(-1)
    assert torch.allclose(ss.cpu().double(), ref_ss, rtol=1e-5, atol=1e-6)
    assert torch.equal(tap[:, H:].cpu(), h.cpu().to(torch.float16))
    assert not tap[:, :H].any()
    eps = 1e-6
    w = (1 + 0.1 * torch.randn(H, generator=torch.Generator().manual_seed(6))).to(torch.bfloat16).to(cuda)
    qt = _qrand(N, H, 12)
    wn = pack(qt, device=cuda)
    xn16 = torch.zeros(M, H, dtype=torch.float16, device=cuda)
    y1 = torch.zeros(M, N, dtype=torch.float32, device=cuda)
    y2 = torch.zeros_like(y1)
    ops.rmsnorm(h, w, eps, y16=xn16, M=M)
    ops.gemm(xn16, wn, y1, epilogue=EPI_STORE_F32, scratch=sc, M=M)
    ops.gemm(h, wn, y2, epilogue=EPI_STORE_F32, scratch=sc, M=M, norm=ops.RowNorm(w, eps, ss))
    torch.cuda.synchronize()
    sc.check_status()
    xn = xn16.float().cpu()
    bound = (xn.abs() @ qt.dequant().abs().t()) * (2.0 ** -8 + 2.0 ** -9) + 1e-5
    diff = (y1.cpu() - y2.cpu()).abs()
    assert (diff <= bound).all(), (diff / bound).max()
    # the fused path is deterministic
    y3 = torch.zeros_like(y1)
    ops.gemm(h, wn, y3, epilogue=EPI_STORE_F32, scratch=sc, M=M, norm=ops.RowNorm(w, eps, ss))
    torch.cuda.synchronize()
    assert torch.equal(y2, y3)


def test_rmsnorm_and_embed(cuda):
    M, H, V = 9, 1024, 4096
    g = torch.Generator().manual_seed(21)
    x = torch.randn(M, H, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
    y = torch.zeros(M, H, dtype=torch.bfloat16, device=cuda)
    y16 = torch.zeros(M, H, dtype=torch.float16, device=cuda)
    ops.rmsnorm(x.to(cuda), w.to(cuda), 1e-6, y=y, y16=y16)
    ref = oq.rms_norm(x.float(), w, 1e-6)
    torch.cuda.synchronize()
    assert torch.allclose(y.float().cpu(), ref, rtol=2 ** -7, atol=1e-6)
    # the fp16 copy is the bf16 value rounded to fp16 (exact except in fp16's subnormal range,
    # below 2^-14, where its absolute error is at most 2^-25)
    assert torch.equal(y16.cpu(), y.cpu().to(torch.float16))
    emb = _qrand(V, H, 11)
    ids = torch.tensor([0, 5, V - 1, 17, 17, 4000, 3, 2, 1], dtype=torch.int32)
    out = torch.zeros(len(ids), H, dtype=torch.bfloat16, device=cuda)
    # the gather with per-tile row sums of squares equals the plain gather
    out_s = torch.zeros_like(out)
    ss = torch.zeros(len(ids), H // 128, dtype=torch.float32, device=cuda)
    ops.embed(ids.to(cuda), pack(emb, device=cuda), out_s, sumsq=ss)
    ops.embed(ids.to(cuda), pack(emb, device=cuda), out)
    torch.cuda.synchronize()
    assert torch.equal(out_s, out)
    ref_ss = (out.float().cpu().double() ** 2).reshape(len(ids), H // 128, 128).sum(-1)
    assert torch.allclose(ss.cpu().double(), ref_ss, rtol=1e-5, atol=1e-6)
    ref = oq.bf(emb.dequant()[ids.long()])
    torch.cuda.synchronize()
    assert torch.allclose(out.float().cpu(), ref, rtol=2 ** -8, atol=1e-7)


def _pool_and_state(cuda, Hkv, hd, kv8, rows, max_tokens, layers=1):
    pool = PagePool(layers, rows * ((max_tokens + PAGE - 1) // PAGE) + 2, Hkv, hd, kv8, cuda)
    st = CacheState(pool, rows, max_tokens, cuda)
    # scatter pages (non-contiguous physical order) to exercise the block table
    for r in range(rows):
        st.ensure(r, max_tokens)
    return pool, st


def _read_kv(pool, st, row, length, Hkv, hd):
    """Dequantized (bf16-valued fp32) K, V [Hkv, length, hd] of a row, read on the host."""
    data = pool.data[0].cpu()
    K = torch.zeros(Hkv, length, hd)
    V = torch.zeros(Hkv, length, hd)
    for p in range((length + PAGE - 1) // PAGE):
        phys = int(st.block_table[row, p])
        page = data[phys]
        n = min(PAGE, length - p * PAGE)
        if not pool.kv8:
            kv = page.view(torch.bfloat16).reshape(2, Hkv, PAGE, hd).float()
            K[:, p * PAGE:p * PAGE + n] = kv[0, :, :n]
            V[:, p * PAGE:p * PAGE + n] = kv[1, :, :n]
        else:
            q = page[: 2 * Hkv * PAGE * hd].reshape(2, Hkv, PAGE, hd).float()
            sb = page[2 * Hkv * PAGE * hd:].view(torch.int32).reshape(2, Hkv, PAGE, hd // 64)
            s = (sb << 16).view(torch.float32).repeat_interleave(64, -1)
            b = (sb & -65536).view(torch.float32).repeat_interleave(64, -1)
            deq = oq.bf(s * q + b)
            K[:, p * PAGE:p * PAGE + n] = deq[0, :, :n]
            V[:, p * PAGE:p * PAGE + n] = deq[1, :, :n]
    return K, V


@pytest.mark.parametrize("hd,kv8", [(128, False), (64, False), (128, True), (64, True)])
def test_qkv_rope_kv_write(cuda, hd, kv8):
    B, T, Hq, Hkv, eps = 2, 5, 8, 2, 1e-6
    pool, st = _pool_and_state(cuda, Hkv, hd, kv8, B, 256)
    pos0 = torch.tensor([60, 3], dtype=torch.int32)  # row 0 straddles a page boundary
    st.seq_len.copy_(pos0.to(cuda))
    g = torch.Generator().manual_seed(hd + 2 * int(kv8))
    qkv = torch.randn(B * T, (Hq + 2 * Hkv) * hd, generator=g).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(hd, generator=g)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(hd, generator=g)).to(torch.bfloat16)
    freqs = oq.inv_freq(hd, 1e6)
    q_out = torch.zeros(B * T, Hq * hd, dtype=torch.bfloat16, device=cuda)
    ops.qkv_rope_kv_write(qkv.to(cuda), B, T, Hq, Hkv, hd, qn.to(cuda), kn.to(cuda), eps,
                          freqs.to(cuda), st.seq_len, q_out, st.layout(0))
    torch.cuda.synchronize()
    for b in range(B):
        rows = qkv[b * T:(b + 1) * T].float()
        pos = torch.arange(int(pos0[b]), int(pos0[b]) + T)
        q = rows[:, : Hq * hd].reshape(T, Hq, hd).transpose(0, 1)
        k = rows[:, Hq * hd:(Hq + Hkv) * hd].reshape(T, Hkv, hd).transpose(0, 1)
        v = rows[:, (Hq + Hkv) * hd:].reshape(T, Hkv, hd).transpose(0, 1)
        q = oq.rope(oq.rms_norm(q, qn, eps), pos, freqs)
        k = oq.rope(oq.rms_norm(k, kn, eps), pos, freqs)
        gq = q_out[b * T:(b + 1) * T].float().cpu().reshape(T, Hq, hd).transpose(0, 1)
        # x*cos - y*sin can cancel: a small output carries the absolute rounding of its terms,
        # so the absolute part of the tolerance follows the head's magnitude
        tol = 2 ** -6 * q.abs() + 2 ** -8 * q.abs().amax(-1, keepdim=True) + 1e-5
        assert ((gq - q).abs() <= tol).all(), (gq - q).abs().max()
        K, V = _read_kv(pool, st, b, int(pos0[b]) + T, Hkv, hd)
        Kn, Vn = K[:, int(pos0[b]):], V[:, int(pos0[b]):]
        if kv8:
            k, v = oq.quantize_kv(k), oq.quantize_kv(v)
            # quantization steps are ~range/255: compare against one step
            tol_k = (k.amax(-1, keepdim=True) - k.amin(-1, keepdim=True)) / 255.0 + 1e-6
            assert ((Kn - k).abs() <= tol_k * 1.01).all()
            assert torch.equal(Vn, v), (Vn - v).abs().max()
        else:
            ktol = 2 ** -6 * k.abs() + 2 ** -8 * k.abs().amax(-1, keepdim=True) + 1e-5
            assert ((Kn - k).abs() <= ktol).all(), (Kn - k).abs().max()
            assert torch.equal(Vn, v)


@pytest.mark.parametrize("hd,kv8,B,T,Hq,Hkv", [(128, False, 1, 9, 32, 8), (128, True, 2, 5, 8, 2),
                                             (64, False, 3, 1, 8, 2), (64, True, 1, 16, 6, 2),
                                             (128, False, 4, 9, 16, 4)])
def test_gemm_qkv_rope_fused_matches_separate(cuda, hd, kv8, B, T, Hq, Hkv):
    """The q|k|v GEMM with the RoPE/KV-write epilogue equals the GEMM followed by the
    standalone RoPE/KV-write kernel bit for bit (q rows and every written cache byte)."""
    H, eps = 1024, 1e-6
    M = B * T
    N = (Hq + 2 * Hkv) * hd
    qt = _qrand(N, H, seed=N + T)
    w = pack(qt, device=cuda)
    x = _x16(M, H, seed=7 + B).to(torch.float16).to(cuda)
    qn = (1 + 0.1 * torch.randn(hd, generator=torch.Generator().manual_seed(1))).to(torch.bfloat16).to(cuda)
    kn = (1 + 0.1 * torch.randn(hd, generator=torch.Generator().manual_seed(2))).to(torch.bfloat16).to(cuda)
    freqs = oq.inv_freq(hd, 1e6).to(cuda)
    pos0 = torch.tensor([60, 3, 127, 0][:B], dtype=torch.int32)  # page-straddling rows
    outs = []
    for fused in (False, True):
        pool, st = _pool_and_state(cuda, Hkv, hd, kv8, B, 256)
        st.seq_len.copy_(pos0.to(cuda))
        sc = ops.Scratch(cuda)
        q_out = torch.zeros(M, Hq * hd, dtype=torch.bfloat16, device=cuda)
        if fused:
            ops.gemm_qkv_rope(x, w, T=T, Hq=Hq, Hkv=Hkv, hd=hd, q_norm=qn, k_norm=kn, eps=eps,
                              inv_freq=freqs, pos0=st.seq_len, q_out=q_out, kv=st.layout(0),
                              scratch=sc, M=M)
        else:
            qkv = torch.zeros(M, N, dtype=torch.bfloat16, device=cuda)
            ops.gemm(x, w, qkv, epilogue=EPI_STORE_BF16, scratch=sc, M=M)
            ops.qkv_rope_kv_write(qkv, B, T, Hq, Hkv, hd, qn, kn, eps, freqs, st.seq_len, q_out,
                                  st.layout(0))
        torch.cuda.synchronize()
        sc.check_status()
        pages = torch.stack([pool.data[0][int(st.block_table[b, p])]
                             for b in range(B) for p in range(st.max_pages)])
        outs.append((q_out.cpu(), pages.cpu()))
    assert torch.equal(outs[0][0], outs[1][0]), "q rows differ"
    assert torch.equal(outs[0][1], outs[1][1]), "cache pages differ"
    assert outs[1][0].float().abs().sum() > 0


@pytest.mark.parametrize("hd,kv8,causal,T,lens", [
    (128, False, True, 9, [1535, 7]),
    (128, False, False, 8, [200, 0]),
    (64, False, True, 9, [127, 64]),
    (128, True, True, 9, [300, 65]),
    (64, True, False, 8, [63, 1]),
    (128, False, True, 1, [4095, 1]),
    (128, False, True, 16, [1000, 31]),
])
def test_attention_paged(cuda, hd, kv8, causal, T, lens):
    B, Hq, Hkv = len(lens), 32 if T <= 9 else 16, 8
    if hd == 64:
        Hq, Hkv = 8, 2
    max_tokens = max(lens) + T + 64
    pool, st = _pool_and_state(cuda, Hkv, hd, kv8, B, max_tokens)
    # fill the cache through the writer kernel (k/v only), then run the block queries
    g = torch.Generator().manual_seed(hd + T)
    for b, L in enumerate(lens):
        tot = L + T
        done = 0
        while done < tot:
            t = min(64, tot - done)
            kvrows = torch.randn(t, 2 * Hkv * hd, generator=g).to(torch.bfloat16)
            view = CacheStateRow(st, b)
            view.seq_len.fill_(done)
            ops.qkv_rope_kv_write(kvrows.to(cuda), 1, t, 0, Hkv, hd, None,
                                  torch.ones(hd, dtype=torch.bfloat16, device=cuda), 1e-6,
                                  oq.inv_freq(hd, 1e6).to(cuda), view.seq_len, None,
                                  view.layout(0))
            done += t
    st.seq_len.copy_(torch.tensor(lens, dtype=torch.int32).to(cuda))
    q = (torch.randn(B * T, Hq * hd, generator=g)).to(torch.bfloat16)
    out = torch.zeros(B * T, Hq * hd, dtype=torch.float16, device=cuda)
    sc = ops.Scratch(cuda)
    splits = max(1, 296 // (B * Hkv))
    ops.attention(q.to(cuda), B, T, Hq, st.layout(0), st.seq_len, causal, hd ** -0.5, out,
                  splits, sc)
    torch.cuda.synchronize()
    # one split (the attention launch writes the output directly): the same arithmetic on
    # other page ranges, so P's bf16 rounding per split differs by a few output ulps
    out3 = torch.zeros_like(out)
    ops.attention(q.to(cuda), B, T, Hq, st.layout(0), st.seq_len, causal, hd ** -0.5, out3,
                  1, sc)
    torch.cuda.synchronize()
    sc.check_status()
    for b, L in enumerate(lens):
        K, V = _read_kv(pool, st, b, L + T, Hkv, hd)
        qb = q[b * T:(b + 1) * T].float().reshape(T, Hq, hd).transpose(0, 1)
        mask = None
        if causal:
            mask = torch.arange(L + T)[None, :] <= (L + torch.arange(T))[:, None]
        ref = oq.sdpa(qb, K, V, hd ** -0.5, mask)
        for o in (out, out3):
            got = o[b * T:(b + 1) * T].float().cpu().reshape(T, Hq, hd).transpose(0, 1)
            # P is rounded to bf16 before P.V on the tensor cores; outputs are bf16
            assert torch.allclose(got, ref, rtol=2 ** -5, atol=2e-3), (b, (got - ref).abs().max())
    # a second call with the same workspace gives the same result
    out2 = torch.zeros_like(out)
    ops.attention(q.to(cuda), B, T, Hq, st.layout(0), st.seq_len, causal, hd ** -0.5, out2,
                  splits, sc)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)


class CacheStateRow:
    def __init__(self, st, r):
        from mlx_dspark_b200.kvcache import RowView
        v = RowView(st, r)
        self.seq_len, self.layout = v.seq_len, v.layout


def test_accept_greedy_fused(cuda):
    B, T, V = 3, 5, 70000
    g = torch.Generator().manual_seed(3)
    logits = torch.randn(B * T, V, generator=g).to(torch.bfloat16)
    tt = logits.float().argmax(-1).view(B, T).int()
    # row 0: all drafts agree; row 1: first draft rejected; row 2: two accepted
    vid = torch.zeros(B, T, dtype=torch.int32)
    vid[0, 1:] = tt[0, :T - 1]
    vid[1, 1:] = (tt[1, :T - 1] + 1) % V
    vid[2, 1:3] = tt[2, :2]
    vid[2, 3:] = (tt[2, 2:T - 1] + 1) % V
    kv_len = torch.tensor([100, 50, 7], dtype=torch.int32)
    am = torch.zeros(B * T, dtype=torch.int32, device=cuda)
    pend = torch.zeros(B, dtype=torch.int32, device=cuda)
    plan = torch.zeros(B, T + 2, dtype=torch.int32, device=cuda)
    kl = kv_len.to(cuda)
    ops.accept_greedy(logits.to(cuda), B, T, vid.to(cuda), am, kl, True, pend, plan,
                      ops.Scratch(cuda))
    torch.cuda.synchronize()
    from oracle.dspark import accept_greedy as ref_accept
    assert torch.equal(am.cpu().view(B, T), tt)
    for b in range(B):
        n, committed = ref_accept(vid[b, 1:].tolist(), tt[b].tolist())
        p = plan[b].tolist()
        assert p[0] == n and p[1] == n + 1 and p[2:3 + n] == committed
        assert int(pend[b]) == committed[-1]
        assert int(kl[b]) == int(kv_len[b]) + n + 1
    assert [int(plan[b, 0]) for b in range(B)] == [T - 1, 0, 2]


def test_accept_argmax_first_index_on_ties(cuda):
    V = 151936
    logits = torch.zeros(2, V, dtype=torch.bfloat16)
    logits[0, 1000] = 3.0
    logits[0, 100000] = 3.0
    logits[0, 500] = 3.0
    logits[1, V - 1] = 1.0
    vid = torch.zeros(1, 2, dtype=torch.int32)
    am = torch.zeros(2, dtype=torch.int32, device=cuda)
    pend = torch.zeros(1, dtype=torch.int32, device=cuda)
    plan = torch.zeros(1, 4, dtype=torch.int32, device=cuda)
    ops.accept_greedy(logits.to(cuda), 1, 2, vid.to(cuda), am, None, False, pend, plan,
                      ops.Scratch(cuda))
    torch.cuda.synchronize()
    assert am.tolist() == [500, V - 1]


def test_markov_sample_block(cuda):
    from oracle.dspark import DSparkRef
    V, R, cap = 4096, 256, 6
    w1, w2 = _qrand(V, R, 21), _qrand(V, R, 22)
    base = (torch.randn(cap, V, generator=torch.Generator().manual_seed(23)) * 0.01).to(torch.bfloat16)

    class W:  # the oracle only reads markov_w1/markov_w2 here
        markov_w1, markov_w2 = w1, w2
    ref = DSparkRef.__new__(DSparkRef)
    ref.w, ref.rnd, ref._deq = W, True, {}
    exp = ref.sample_block(base.float(), 17)
    draft = torch.zeros(1, cap, dtype=torch.int32, device=cuda)
    vids = torch.zeros(1, cap + 1, dtype=torch.int32, device=cuda)
    ops.markov_sample_block(base.to(cuda), cap, 1, cap, pack(w1, device=cuda), pack(w2, device=cuda),
                            torch.tensor([17], dtype=torch.int32, device=cuda), draft, vids,
                            ops.Scratch(cuda))
    torch.cuda.synchronize()
    assert draft[0].tolist() == exp
    assert vids[0].tolist() == [17] + exp


def test_shared_workspace_across_shapes(cuda):
    """Calls of different N, M and families share one Scratch: counters must stay valid
    (a regression test for counter regions overlapping another call's partials)."""
    sc = ops.Scratch(cuda)
    shapes = [(9, 32768, 512), (9, 768, 512), (9, 512, 1536), (9, 32768, 512), (1, 4096, 256),
              (9, 32768, 512)]
    ws = {}
    for i, (M, N, K) in enumerate(shapes):
        if (N, K) not in ws:
            qt = _qrand(N, K, N + K)
            ws[(N, K)] = (qt, pack(qt, device=cuda))
        qt, w = ws[(N, K)]
        x = _x16(M, K, seed=i)
        y = torch.zeros(M, N, dtype=torch.float32, device=cuda)
        ops.gemm(x.to(torch.float16).to(cuda), w, y, epilogue=EPI_STORE_F32, scratch=sc)
        torch.cuda.synchronize()
        ref = x @ qt.dequant().t()
        bound = (x.abs() @ qt.dequant().abs().t()) * 2.0 ** -10 + 1e-5
        assert ((y.cpu() - ref).abs() <= bound).all(), (i, M, N, K)
    assert int(sc.bufs["gemm"][:65536].view(torch.int32).abs().sum()) == 0


def test_kv8_quantizer_follows_mlx_rule_exactly(cuda):
    """The quantize-on-write of 8-bit pages against the oracle's restatement of MLX's affine
    quantizer, bit for bit on the V rows (written without norm or RoPE): groups whose larger-
    magnitude edge is the minimum or the maximum, an all-zero group, constant groups of either
    sign, and random groups."""
    B, T, Hq, Hkv, hd, eps = 1, 8, 0, 1, 128, 1e-6
    pool, st = _pool_and_state(cuda, Hkv, hd, True, B, 256)
    st.seq_len.fill_(0)
    g = torch.Generator().manual_seed(17)
    v = torch.randn(T, hd, generator=g)
    v[0, :64] = 0.0                                  # all zero: bias 0, q 0
    v[1, :64] = -0.75                                # constant negative
    v[1, 64:] = 0.5                                  # constant positive
    v[2, :64] = torch.linspace(-3.0, 1.0, 64)        # |min| > |max|
    v[2, 64:] = torch.linspace(-1.0, 3.0, 64)        # |max| >= |min|
    v[3] *= 1e-4                                     # tiny range
    v[4, :64] = torch.linspace(-1.0, 1.0, 64)        # symmetric edges
    v = v.to(torch.bfloat16)
    qkv = torch.cat([torch.randn(T, hd, generator=g).to(torch.bfloat16), v], dim=1)  # k | v
    kn = torch.ones(hd, dtype=torch.bfloat16)
    freqs = oq.inv_freq(hd, 1e6)
    ops.qkv_rope_kv_write(qkv.to(cuda), B, T, Hq, Hkv, hd, None, kn.to(cuda), eps,
                          freqs.to(cuda), st.seq_len, None, st.layout(0))
    torch.cuda.synchronize()
    _, V = _read_kv(pool, st, 0, T, Hkv, hd)
    ref = oq.quantize_kv(v.float()[None])
    assert torch.equal(V, ref), (V - ref).abs().max()
    assert torch.equal(V[0, 0, :64], torch.zeros(64))
