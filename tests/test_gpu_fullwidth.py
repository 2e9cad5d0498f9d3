"""Parity at the BASELINE widths (depth-reduced), and the sampled output's distribution.

- Qwen3-8B width (H 4096, 32q/8kv, hd 128, I 12288, V 151936, seed 1, W8) at 1, 2, 4 and 8
  layers, and Qwen3-32B width (H 5120, 64q/8kv, I 25600) at 2 layers: a 91-token prefill (the
  large-M GEMM path) then a 9-token verify block (the small-M path) through Target.run, against
  the CPU oracle on the same quantized weights. Tolerance: every logit within
  2e-2 * sqrt(layers) of its row's largest magnitude, i.e. bf16 rtol 2e-2 at the row scale per
  layer, with independent per-layer errors adding in quadrature (measured: 1.1e-2, 1.4e-2,
  1.8e-2, 2.5e-2 and 6.0e-2 at 1, 2, 4, 8 and 36 layers, about 1e-2 * sqrt(layers)); a
  per-element relative bound is meaningless for logits near zero and is logged, not asserted;
  and the greedy token the oracle's argmax unless the oracle's top-2 gap is within two bf16
  ulps of the top logit.
- Qwen3-4B width (H 2560, tied embeddings) with the DFlash drafter (2 layers, block 16): the
  drafter's head logits for a block, and greedy dflash_generate teacher-forced, against the
  oracle.
- Qwen3-8B at its full 36 layers against the oracle (about 33 GB of host memory for its fp32
  weights), with the same depth bound (0.12 of the row scale), and the greedy token the
  oracle's wherever the oracle's top-2 gap exceeds twice that row's measured error.
- Chi-square goodness of fit of the first committed token of a speculative round at C3's
  sampling parameters (T 1.0, top-p 0.95, top-k 50) on the real 151936-token vocabulary:
  10240 independent seeds, each drafting from a q row and accepting against a p row of the
  4B-width target's own logits; the token counts must fit truncate(softmax(p / T)).

Error figures are appended as JSON lines to $DSPARK_PARITY_LOG when that is set."""
import json
import os

import numpy as np
import pytest
import torch

from mlx_dspark_b200 import ops
from mlx_dspark_b200.config import QWEN3_4B, QWEN3_8B, QWEN3_32B, dflash_for, with_layers
from mlx_dspark_b200.load import dflash_drafter_for, load_target
from mlx_dspark_b200.weights import generate_dflash, generate_target
from oracle import sampling as S
from oracle.dflash import DFlashRef
from oracle.qwen3 import Qwen3Ref

pytestmark = pytest.mark.gpu


def _log(rec: dict) -> None:
    path = os.environ.get("DSPARK_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(rec) + "\n")


def _ulp2(v: float) -> float:
    return 2.0 ** (int(np.floor(np.log2(abs(v) + 1e-30))) - 7) * 2


def _errors(got: torch.Tensor, ref: torch.Tensor) -> dict:
    scale = ref.abs().amax(-1, keepdim=True)
    row_rel = float(((got - ref).abs() / scale).max())
    big = ref.abs() >= 0.1 * scale
    elem_rel = float(((got - ref).abs() / ref.abs().clamp_min(1e-30))[big].max())
    return {"row_max_rel": row_rel, "elem_rel_big": elem_rel}


def _greedy_ok(got: torch.Tensor, ref: torch.Tensor) -> int:
    """Rows whose GPU argmax differs from the oracle's; each must be a near-tie there."""
    flips = 0
    for r in range(ref.shape[0]):
        a, b = int(got[r].argmax()), int(ref[r].argmax())
        if a != b:
            gap = float(ref[r, b] - ref[r, a])
            assert gap <= max(1e-3, _ulp2(float(ref[r, b]))), (r, a, b, gap)
            flips += 1
    return flips


@pytest.mark.parametrize("name,cfg,layers", [("qwen3-8b", QWEN3_8B, 1), ("qwen3-8b", QWEN3_8B, 2),
                                             ("qwen3-8b", QWEN3_8B, 4), ("qwen3-8b", QWEN3_8B, 8),
                                             ("qwen3-32b", QWEN3_32B, 2)])
def test_full_width_forward_matches_oracle(cuda, name, cfg, layers):
    c = with_layers(cfg, layers)
    tw = generate_target(c, 1, "cuda").to("cpu")
    target, _ = load_target(c, weights=tw, device=cuda)
    g = torch.Generator().manual_seed(21)
    prompt = torch.randint(0, c.vocab_size, (100,), generator=g).tolist()
    cache = target.make_cache(256)
    tap = [0]
    lg1, f1 = target.run([prompt[:91]], cache, tap)     # large-M prefill path
    lg2, f2 = target.run([prompt[91:]], cache, tap)     # 9-row verify block (small-M GEMMs)
    target.scratch.check_status()
    got = torch.cat([lg1[0][-4:], lg2[0]]).float().cpu()
    got_tap = torch.cat([f1[0][-4:], f2[0]]).float().cpu()
    del target
    torch.cuda.empty_cache()
    ref = Qwen3Ref(tw)
    rl, rf = ref.run(prompt, ref.make_cache(), tap)
    rl, rf = rl[87:], rf[87:]
    e = _errors(got, rl)
    et = _errors(got_tap, rf)
    flips = _greedy_ok(got, rl)
    _log({"test": "full_width", "model": name, "layers": layers, "logits": e, "tap": et,
          "argmax_flips": flips, "rows": got.shape[0]})
    assert e["row_max_rel"] <= 2e-2 * layers ** 0.5, e
    assert et["row_max_rel"] <= 2e-2, et


def test_qwen3_4b_width_dflash_matches_oracle(cuda):
    from mlx_dspark_b200.generate import SpecSession, dflash_generate, prefill_rows
    from test_gpu_e2e import teacher_forced_check
    c = with_layers(QWEN3_4B, 2)
    fcfg = dflash_for(QWEN3_4B)
    fcfg.target_layer_ids, fcfg.num_target_layers = (0, 1), 2
    tw = generate_target(c, 0, "cuda").to("cpu")
    fw = generate_dflash(fcfg, 0, "cpu")
    target, _ = load_target(c, weights=tw, device=cuda)
    drafter, _ = dflash_drafter_for(target, fcfg, weights=fw, device=cuda)
    g = torch.Generator().manual_seed(23)
    prompt = torch.randint(0, c.vocab_size, (80,), generator=g).tolist()
    cap = drafter.block_size - 1
    sess = SpecSession(target, drafter, 1, cap, len(prompt) + 64)
    last = prefill_rows(target, prompt, sess.tstate, sess.tap, drafter, sess.cstate)
    pending = int(last.float().argmax())
    sess.pending.fill_(pending)
    drafter.draft_dev(sess.pending, 1, cap, sess.cstate, sess.dbuf, sess.draft, sess.vbuf.ids,
                      sess.splits_c)
    torch.cuda.synchronize()
    head_gpu = sess.dbuf.base[:cap].float().cpu()
    sess.release()
    res = dflash_generate(target, None, drafter, prompt_ids=prompt, max_new_tokens=24)
    target.scratch.check_status()
    ref_t, ref_f = Qwen3Ref(tw), DFlashRef(fw, tw)
    _, fused = ref_t.run(prompt, ref_t.make_cache(), list(fcfg.target_layer_ids))
    head = ref_f.draft_logits(pending, fused, ref_f.make_cache(), cap)
    e = _errors(head_gpu, head)
    excused, worst = teacher_forced_check(ref_t, prompt, res.token_ids[:24])
    _log({"test": "qwen3_4b_dflash", "head": e, "greedy_excused": excused,
          "mean_accept": res.mean_accept_len})
    assert e["row_max_rel"] <= 2e-2, e
    assert excused <= 3


def test_qwen3_8b_36_layers_matches_oracle(cuda):
    tw = generate_target(QWEN3_8B, 1, "cuda").to("cpu")
    target, _ = load_target(QWEN3_8B, weights=tw, device=cuda)
    g = torch.Generator().manual_seed(29)
    prompt = torch.randint(0, QWEN3_8B.vocab_size, (73,), generator=g).tolist()
    cache = target.make_cache(256)
    target.run([prompt[:64]], cache, ())
    got = target.run([prompt[64:]], cache, ())[0][0].float().cpu()
    target.scratch.check_status()
    del target, cache
    torch.cuda.empty_cache()
    ref = Qwen3Ref(tw)
    rl, _ = ref.run(prompt, ref.make_cache(), [])
    rl = rl[64:]
    e = _errors(got, rl)
    # greedy: a flip only where the oracle's top-2 gap is within twice the row's error
    flips, unexplained = 0, 0
    for r in range(rl.shape[0]):
        a, b = int(got[r].argmax()), int(rl[r].argmax())
        if a != b:
            flips += 1
            gap = float(rl[r, b] - rl[r, a])
            if gap > 2 * float((got[r] - rl[r]).abs().max()):
                unexplained += 1
    _log({"test": "full_width", "model": "qwen3-8b", "layers": 36, "logits": e,
          "argmax_flips": flips, "unexplained_flips": unexplained, "rows": got.shape[0]})
    assert e["row_max_rel"] <= 2e-2 * 36 ** 0.5, e
    assert unexplained == 0


def test_chi_square_first_token_at_c3_sampling_params(cuda):
    from scipy.stats import chi2
    c = with_layers(QWEN3_4B, 1)
    tw = generate_target(c, 0, "cuda")
    target, _ = load_target(c, weights=tw, device=cuda)
    del tw
    g = torch.Generator().manual_seed(31)
    prompt = torch.randint(0, c.vocab_size, (40,), generator=g).tolist()
    lg, _ = target.run([prompt], target.make_cache(128), ())
    V = c.vocab_size
    # sharpen the random-init rows (the smallest scale, in steps of 2^(1/8), at which the 50
    # largest probabilities hold 95.5% of the mass) so that top-k 50 and top-p 0.95 both cut and
    # tens of tokens stay in the support; the same bf16 rows feed the GPU and the expected
    # distribution
    base_p, base_q = lg[0][-1].float(), lg[0][-2].float()
    mult = 1.0
    for m in [2.0 ** (k / 8) for k in range(0, 96)]:
        pr = torch.softmax(base_p.double().cpu() * m, -1)
        if float(pr.topk(50).values.sum()) >= 0.955:
            mult = m
            break
    p_row = (base_p * mult).to(torch.bfloat16)
    q_row = (base_q * mult).to(torch.bfloat16)
    temp, top_p, top_k = 1.0, 0.95, 50
    kept, _ = S.truncated_weights(S._row_bits(p_row.cpu()), temp, 0, top_p, top_k)
    expected = S.probs_of(kept)
    N, B = 10240, 2048
    counts = np.zeros(V, dtype=np.int64)
    sc = ops.Scratch(cuda)
    for start in range(0, N, B):
        rng = ops.rng_state(list(range(50_000 + start, 50_000 + start + B)), cuda)
        x = torch.zeros(B, dtype=torch.int32, device=cuda)
        q = torch.zeros(B, V, dtype=torch.float32, device=cuda)
        ops.sample_rows(q_row[None].expand(B, V).contiguous(), B, 1, temp, top_p, top_k, rng, x,
                        stream_id=1, probs=q)
        vid = torch.stack([torch.zeros(B, dtype=torch.int32, device=cuda), x], 1).contiguous()
        v = p_row[None].expand(2 * B, V).contiguous()
        pend = torch.zeros(B, dtype=torch.int32, device=cuda)
        plan = torch.zeros(B, 4, dtype=torch.int32, device=cuda)
        ops.accept_sample(v, B, 2, vid, q, temp, top_p, top_k, rng, None, False, pend, plan, sc)
        torch.cuda.synchronize()
        counts += np.bincount(plan[:, 2].cpu().numpy(), minlength=V)
    assert counts.sum() == N
    exp = expected * N
    assert counts[exp == 0].sum() == 0, "a token outside the truncated support was emitted"
    # bins with expected count >= 5, the rest pooled into one tail bin
    order = np.argsort(-exp)
    e_sorted, c_sorted = exp[order], counts[order]
    big = e_sorted >= 5
    e_bins = np.append(e_sorted[big], e_sorted[~big].sum())
    c_bins = np.append(c_sorted[big], c_sorted[~big].sum())
    if e_bins[-1] < 5:              # fold a small tail into the last full bin
        e_bins[-2] += e_bins[-1]
        c_bins[-2] += c_bins[-1]
        e_bins, c_bins = e_bins[:-1], c_bins[:-1]
    stat = float(((c_bins - e_bins) ** 2 / e_bins).sum())
    dof = len(e_bins) - 1
    pval = float(chi2.sf(stat, dof))
    support = int((expected > 0).sum())
    _log({"test": "chi_square_c3", "N": N, "support": support, "bins": len(e_bins),
          "chi2": stat, "dof": dof, "p_value": pval, "logit_scale": mult})
    assert 2 <= support <= top_k and dof >= 5, (support, dof)
    assert pval > 1e-3, (stat, dof, pval)
