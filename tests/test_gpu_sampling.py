"""GPU parity of the lossless sampling kernels (K9) against the bit-exact CPU restatement.

Integer outputs (tokens, accepted lengths, plans) must be identical; the truncated
distributions written by dspark_sample_rows must equal the oracle's float32 values bit for
bit. The losslessness test mirrors the reference's test_topp_speculative_sampling_is_lossless
(tests/test_generate_helpers.py:145-170) with the draws made on the GPU.
"""
import numpy as np
import pytest
import torch

from mlx_dspark_b200 import ops
from mlx_dspark_b200.weights import pack, quantize_w8g64
from oracle import sampling as S

pytestmark = pytest.mark.gpu

CASES = [  # (T, top_p, top_k, temp_mode)
    (1.0, 1.0, 0, 0),      # identity: long path, full-vocabulary draw
    (1.0, 0.95, 50, 0),    # the C3 setting: short list
    (0.7, 1.0, 3, 0),
    (1.0, 0.9, 0, 0),      # nucleus only: long path with weight histograms
    (1.3, 0.8, 1000, 0),   # top-k beyond the short list: long path with both cuts
    (0.6, 0.5, 20, 1),     # multiply-by-1/T form of sample_block_probs
]


def _rows(n, V, seed, scale=2.5):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, V, generator=g) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("V", [32768, 151936])
@pytest.mark.parametrize("T,top_p,top_k,tm", CASES)
def test_sample_rows_matches_oracle(cuda, V, T, top_p, top_k, tm):
    G, R = 2, 3
    rows = _rows(G * R, V, seed=V + top_k)
    seeds = [11, 987654321987]
    rng = ops.rng_state(seeds, cuda)
    rng[:, 1] = 5
    tok = torch.full((G * R,), -1, dtype=torch.int32, device=cuda)
    tok2 = torch.full((G * R, 2), -1, dtype=torch.int32, device=cuda)
    probs = torch.zeros(G * R, V, dtype=torch.float32, device=cuda)
    ops.sample_rows(rows.to(cuda), G, R, T, top_p, top_k, rng, tok, stream_id=1, row_base=3,
                    probs=probs, tokens2=tok2, tok2_stride=2, temp_mode=tm)
    torch.cuda.synchronize()
    for r in range(G * R):
        g, y = divmod(r, R)
        t, q = S.sample_row_exact(rows[r], T, tm, top_p, top_k, seeds[g], 5, 3 + y, 1)
        assert int(tok[r]) == t, (r, int(tok[r]), t)
        assert int(tok2[r, 0]) == t
        assert np.array_equal(probs[r].cpu().numpy().view(np.uint32), q.view(np.uint32)), r


def test_sample_rows_ties_and_tiny_vocab(cuda):
    # constant rows: every key ties, so top-k keeps all and the list overflows to the long path
    V = 4096
    rows = torch.zeros(2, V, dtype=torch.bfloat16)
    rows[1, 100:300] = 1.0
    rng = ops.rng_state([3, 4], cuda)
    tok = torch.zeros(2, dtype=torch.int32, device=cuda)
    probs = torch.zeros(2, V, dtype=torch.float32, device=cuda)
    ops.sample_rows(rows.to(cuda), 2, 1, 1.0, 1.0, 50, rng, tok, probs=probs)
    torch.cuda.synchronize()
    for r in range(2):
        t, q = S.sample_row_exact(rows[r], 1.0, 0, 1.0, 50, [3, 4][r], 0, 0, 2)
        assert int(tok[r]) == t
        assert np.array_equal(probs[r].cpu().numpy(), q)
    assert int((probs[1] > 0).sum()) == 200
    # a vocabulary smaller than one CTA's share leaves some CTAs of the cluster empty
    small = _rows(1, 6, 9)
    tok1 = torch.zeros(1, dtype=torch.int32, device=cuda)
    for i in range(20):
        rng = ops.rng_state([i], cuda)
        ops.sample_rows(small.to(cuda), 1, 1, 1.0, 0.8, 0, rng, tok1)
        torch.cuda.synchronize()
        assert int(tok1[0]) == S.sample_row_exact(small[0], 1.0, 0, 0.8, 0, i, 0, 0, 2)[0]


@pytest.mark.parametrize("top_p,top_k", [(0.95, 50), (1.0, 0), (0.9, 0)])
@pytest.mark.parametrize("onehot", [False, True])
def test_accept_sample_matches_oracle(cuda, top_p, top_k, onehot):
    B, T, V = 3, 9, 151936
    L = T - 1
    v_logits = _rows(B * T, V, seed=77, scale=3.0)
    draft_logits = _rows(B * L, V, seed=78, scale=3.0)
    seeds = [1, 2, 3]
    # drafts: sampled from the drafter rows (q), with row b planting target argmaxes so that
    # acceptance runs deep in some blocks and stops early in others
    rng_d = ops.rng_state(seeds, cuda)
    draft = torch.zeros(B * L, dtype=torch.int32, device=cuda)
    q = torch.zeros(B * L, V, dtype=torch.float32, device=cuda)
    ops.sample_rows(draft_logits.to(cuda), B, L, 1.0, top_p, top_k, rng_d, draft, stream_id=1,
                    probs=q)
    torch.cuda.synchronize()
    vid = torch.zeros(B, T, dtype=torch.int32)
    vid[:, 0] = 5
    vid[:, 1:] = draft.view(B, L).cpu()
    am = v_logits.float().argmax(-1).view(B, T)
    vid[0, 1:] = am[0, :L].int()
    vid[1, 1:4] = am[1, :3].int()
    rng = ops.rng_state(seeds, cuda)
    rng[:, 1] = 41
    kv = torch.tensor([100, 200, 300], dtype=torch.int32, device=cuda)
    pend = torch.full((B,), -1, dtype=torch.int32, device=cuda)
    plan = torch.full((B, T + 2), -7, dtype=torch.int32, device=cuda)
    sc = ops.Scratch(cuda)
    kv_exp = [100, 200, 300]
    for call in range(2):  # the second call reuses the workspace counters the first reset
        ops.accept_sample(v_logits.to(cuda), B, T, vid.to(cuda), None if onehot else q, 1.0, top_p,
                          top_k, rng, kv, True, pend, plan, sc, q_onehot=onehot)
        torch.cuda.synchronize()
        for b in range(B):
            qb = None if onehot else q.view(B, L, V)[b].cpu().numpy()
            n, repl, _, _ = S.accept_sample_exact(v_logits[b * T:(b + 1) * T], vid[b].tolist(), qb,
                                                  1.0, 0, top_p, top_k, seeds[b], 41 + call,
                                                  q_onehot=onehot)
            pl = plan[b].tolist()
            assert pl[0] == n and pl[1] == n + 1, (call, b, pl, n)
            assert pl[2:2 + n] == vid[b, 1:1 + n].tolist()
            assert pl[2 + n] == repl and int(pend[b]) == repl
            assert all(v == -1 for v in pl[3 + n:])
            kv_exp[b] += n + 1
        assert kv.tolist() == kv_exp
        assert rng[:, 1].tolist() == [42 + call] * B
    assert int(sc.bufs["accept_sample"][:256].view(torch.int32).abs().sum()) == 0


def test_accept_sample_many_blocks_tiny_vocab_matches_oracle(cuda):
    """2048 independent T=2 blocks over a 6-token vocabulary, block by block."""
    V, N = 6, 2048
    target = torch.tensor([2.0, 1.0, 0.5, 0.0, -1.0, -2.0]).to(torch.bfloat16)
    qlog = torch.tensor([-2.0, -1.0, 0.0, 0.5, 1.0, 2.0]).to(torch.bfloat16)
    seeds = list(range(1000, 1000 + N))
    rng = ops.rng_state(seeds, cuda)
    x = torch.zeros(N, dtype=torch.int32, device=cuda)
    q = torch.zeros(N, V, dtype=torch.float32, device=cuda)
    ops.sample_rows(qlog[None].expand(N, V).contiguous().to(cuda), N, 1, 1.0, 1.0, 0, rng, x,
                    stream_id=1, probs=q)
    vid = torch.stack([torch.zeros(N, dtype=torch.int32, device=cuda), x], 1).contiguous()
    v = target[None].expand(2 * N, V).contiguous().to(cuda)
    pend = torch.zeros(N, dtype=torch.int32, device=cuda)
    plan = torch.zeros(N, 4, dtype=torch.int32, device=cuda)
    ops.accept_sample(v, N, 2, vid, q, 1.0, 1.0, 0, rng, None, False, pend, plan, ops.Scratch(cuda))
    torch.cuda.synchronize()
    xs, qs, pl = x.cpu().tolist(), q.cpu().numpy(), plan.cpu().tolist()
    bad = []
    for g in range(N):
        ex, eq = S.sample_row_exact(qlog, 1.0, 0, 1.0, 0, seeds[g], 0, 0, 1)
        n, repl, fl, cd = S.accept_sample_exact(torch.stack([target, target]), [0, ex], eq[None],
                                                1.0, 0, 1.0, 0, seeds[g], 0)
        got = (xs[g], pl[g][0], pl[g][2 + pl[g][0]])
        if got != (ex, n, repl) or not np.array_equal(qs[g], eq):
            bad.append((g, got, (ex, n, repl, fl, cd)))
    assert not bad, (len(bad), bad[:8])


def test_accept_sample_is_lossless(cuda):
    """Mirror of the reference's losslessness test: committed-token frequencies over 20000
    independent blocks match truncate(softmax(target / T)) within 0.02."""
    V, N = 6, 20000
    target = torch.tensor([2.0, 1.0, 0.5, 0.0, -1.0, -2.0]).to(torch.bfloat16)
    qlog = torch.tensor([-2.0, -1.0, 0.0, 0.5, 1.0, 2.0]).to(torch.bfloat16)
    for (T, tp, tk) in [(1.0, 1.0, 0), (1.0, 0.8, 0), (0.7, 1.0, 3)]:
        rng = ops.rng_state(list(range(1000, 1000 + N)), cuda)
        x = torch.zeros(N, dtype=torch.int32, device=cuda)
        q = torch.zeros(N, V, dtype=torch.float32, device=cuda)
        ops.sample_rows(qlog[None].expand(N, V).contiguous().to(cuda), N, 1, 1.0, 1.0, 0, rng, x,
                        stream_id=1, probs=q)
        vid = torch.stack([torch.zeros(N, dtype=torch.int32, device=cuda), x], 1).contiguous()
        v = target[None].expand(2 * N, V).contiguous().to(cuda)
        pend = torch.zeros(N, dtype=torch.int32, device=cuda)
        plan = torch.zeros(N, 4, dtype=torch.int32, device=cuda)
        ops.accept_sample(v, N, 2, vid, q, T, tp, tk, rng, None, False, pend, plan, ops.Scratch(cuda))
        torch.cuda.synchronize()
        # the first committed token: the draft when accepted, else the residual draw
        first = plan[:, 2]
        emp = np.bincount(first.cpu().numpy(), minlength=V) / N
        kept, _ = S.truncated_weights(S._row_bits(target), T, 0, tp, tk)
        exp = S.probs_of(kept)
        assert np.abs(emp - exp).max() < 0.02, (T, tp, tk, emp, exp)
        n = plan[:, 0]
        assert torch.equal(first[n == 1], x[n == 1])
        assert torch.equal(pend[n == 0], first[n == 0])


def test_markov_sample_block_probs_matches_oracle(cuda):
    from oracle.dspark import DSparkRef
    from oracle.qwen3 import bf
    V, R, cap, B = 4096, 256, 5, 2
    g = torch.Generator().manual_seed(5)
    w1 = quantize_w8g64(torch.randn(V, R, generator=g) * 0.02)
    w2 = quantize_w8g64(torch.randn(V, R, generator=g) * 0.02)
    base = (torch.randn(B * cap, V, generator=g) * 2.0).to(torch.bfloat16)

    class W:
        markov_w1, markov_w2 = w1, w2
    ref = DSparkRef.__new__(DSparkRef)
    ref.w, ref.rnd, ref._deq = W, True, {}
    seeds, first = [21, 22], [17, 4000]
    rng = ops.rng_state(seeds, cuda)
    draft = torch.zeros(B, cap, dtype=torch.int32, device=cuda)
    vids = torch.zeros(B, cap + 1, dtype=torch.int32, device=cuda)
    q = torch.zeros(B, cap, V, dtype=torch.float32, device=cuda)
    ops.markov_sample_block_probs(base.to(cuda), cap, B, cap, pack(w1, device=cuda),
                                  pack(w2, device=cuda), torch.tensor(first, dtype=torch.int32,
                                                                      device=cuda),
                                  draft, vids, 0.8, 0.9, 40, rng, q.view(B * cap, V),
                                  ops.Scratch(cuda))
    torch.cuda.synchronize()
    for b in range(B):
        prev = first[b]
        for i in range(cap):
            logits = bf(base[b * cap + i].float() + ref.step_bias(prev), True).to(torch.bfloat16)
            t, qi = S.sample_row_exact(logits, 0.8, 1, 0.9, 40, seeds[b], 0, i, 1)
            assert int(draft[b, i]) == t, (b, i)
            assert np.array_equal(q[b, i].cpu().numpy(), qi), (b, i)
            prev = t
        assert vids[b].tolist() == [first[b]] + draft[b].tolist()


def test_apply_penalties_matches_oracle(cuda):
    from oracle.penalties import Penalizer
    B, T, V = 2, 9, 32768
    g = torch.Generator().manual_seed(3)
    logits = (torch.randn(B * T, V, generator=g) * 4).to(torch.bfloat16)
    hist = [[5, 5, 9, 100, 31000] + [7] * 300, [1, 2, 3, 3]]
    drafts = [[5, 5, 11, 11, 9, 8, 7, 6], [3, 4, 4, 4, 2, 30000, 1, 1]]
    counts = torch.zeros(B, V, dtype=torch.int32)
    vid = torch.zeros(B, T, dtype=torch.int32)
    for b in range(B):
        for t in hist[b]:
            counts[b, t] += 1
        vid[b, 1:] = torch.tensor(drafts[b])
    out = logits.clone().to(cuda)
    ops.apply_penalties(out, B, T, counts.to(cuda), vid.to(cuda), 0.4, 0.3)
    torch.cuda.synchronize()
    for b in range(B):
        p = Penalizer(0.4, 0.3)
        p.add(hist[b])
        exp = p.apply(logits[b * T:(b + 1) * T], drafts[b])
        assert torch.equal(out[b * T:(b + 1) * T].cpu(), exp), b
    # counts advance by a plan's committed tokens
    plan = torch.tensor([[2, 3, 5, 5, 17, -1, -1, -1, -1, -1, -1],
                         [0, 1, 4, -1, -1, -1, -1, -1, -1, -1, -1]], dtype=torch.int32)
    c = counts.to(cuda)
    ops.penalty_counts_add(c, plan.to(cuda), B)
    torch.cuda.synchronize()
    exp = counts.clone()
    exp[0, 5] += 2
    exp[0, 17] += 1
    exp[1, 4] += 1
    assert torch.equal(c.cpu(), exp)
