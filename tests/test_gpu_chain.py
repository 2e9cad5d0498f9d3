"""The fused layer chain (dspark_run_chain) against the separate-kernel forward and the CPU
oracle (tiny config, bf16 and 8-bit KV, with hidden-state taps): the same rounding points,
so logits and taps agree to within a few bf16 ulps of the row scale (2^-6 relative here: only
reduction orders differ), and both stay within the oracle's bf16 rtol 2e-2."""
import pytest
import torch

from mlx_dspark_b200.config import TINY, dspark_for
from mlx_dspark_b200.load import load_target
from mlx_dspark_b200.weights import generate_target
from oracle.qwen3 import Qwen3Ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("layers,kv", [(1, None), (4, None), (4, 8)])
def test_chain_forward_matches_separate_kernels_and_oracle(cuda, layers, kv):
    from mlx_dspark_b200.config import with_layers
    cfg = with_layers(TINY, layers)
    tw = generate_target(cfg, 0, "cpu")
    target, _ = load_target(cfg, weights=tw, kv_bits=kv, device=cuda)
    tap = [t for t in dspark_for(TINY).target_layer_ids if t < layers]
    g = torch.Generator().manual_seed(11)
    prompt = torch.randint(0, TINY.vocab_size, (150,), generator=g).tolist()
    out = {}
    for chain in (True, False):
        target.use_chain = chain
        cache = target.make_cache(512)
        lg, fu = target.run([prompt[:100]], cache, tap)
        lg2, fu2 = target.run([prompt[100:]], cache, tap)      # continue through the KV cache
        out[chain] = (torch.cat([lg[0], lg2[0]]).float().cpu(),
                      torch.cat([fu[0], fu2[0]]).float().cpu() if tap else None)
    target.use_chain = False
    ref = Qwen3Ref(tw)
    rl, rf = ref.run(prompt, ref.make_cache(kv == 8), tap)
    pairs = [("logits chain/separate", out[True][0], out[False][0], 2.0 ** -6),
             ("logits chain/oracle", out[True][0], rl, 2e-2)]
    if tap:
        pairs += [("taps chain/separate", out[True][1], out[False][1], 2.0 ** -6),
                  ("taps chain/oracle", out[True][1], rf, 2e-2)]
    for name, a, b, tol in pairs:
        sc = b.abs().amax(-1, keepdim=True)
        err = float(((a - b).abs() / sc).max())
        assert err <= tol, (name, err)
