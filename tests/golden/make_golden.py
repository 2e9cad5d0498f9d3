"""Generate tests/golden/qwen3_tiny_hf.pt: outputs of HF transformers' Qwen3ForCausalLM
(transformers 5.5, fp32, eager attention) on the dequantized weights of the seeded tiny
target (BASELINE C1 shapes, seed 0). mlx-lm's qwen3 model is a port of this architecture;
these vectors pin the oracle's forward (tests/test_oracle_pins.py) independently of the
oracle's own code.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from mlx_dspark_b200.config import TINY  # noqa: E402
from mlx_dspark_b200.weights import generate_target  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "qwen3_tiny_hf.pt")
TAPS = (1, 2, 3)


def hf_model(w):
    from transformers import Qwen3Config, Qwen3ForCausalLM

    c = w.cfg
    cfg = Qwen3Config(hidden_size=c.hidden_size, intermediate_size=c.intermediate_size,
                      num_hidden_layers=c.num_hidden_layers,
                      num_attention_heads=c.num_attention_heads,
                      num_key_value_heads=c.num_key_value_heads, head_dim=c.head_dim,
                      vocab_size=c.vocab_size, rms_norm_eps=c.rms_norm_eps,
                      rope_parameters={"rope_type": "default", "rope_theta": c.rope_theta},
                      tie_word_embeddings=c.tie_word_embeddings, max_position_embeddings=4096,
                      attn_implementation="eager")
    m = Qwen3ForCausalLM(cfg).to(torch.float32).eval()
    sd = {"model.embed_tokens.weight": w.embed.dequant(), "model.norm.weight": w.norm.float()}
    for i, L in enumerate(w.layers):
        p = f"model.layers.{i}."
        sd[p + "self_attn.q_proj.weight"] = L.wq.dequant()
        sd[p + "self_attn.k_proj.weight"] = L.wk.dequant()
        sd[p + "self_attn.v_proj.weight"] = L.wv.dequant()
        sd[p + "self_attn.o_proj.weight"] = L.wo.dequant()
        sd[p + "self_attn.q_norm.weight"] = L.q_norm.float()
        sd[p + "self_attn.k_norm.weight"] = L.k_norm.float()
        sd[p + "mlp.gate_proj.weight"] = L.gate.dequant()
        sd[p + "mlp.up_proj.weight"] = L.up.dequant()
        sd[p + "mlp.down_proj.weight"] = L.down.dequant()
        sd[p + "input_layernorm.weight"] = L.input_ln.float()
        sd[p + "post_attention_layernorm.weight"] = L.post_ln.float()
    if not c.tie_word_embeddings:
        sd["lm_head.weight"] = w.lm_head.dequant()
    missing, unexpected = m.load_state_dict(sd, strict=False)
    missing = [k for k in missing if k != "lm_head.weight"]
    assert not missing and not unexpected, (missing, unexpected)
    if c.tie_word_embeddings:
        m.tie_weights()
    return m


def main():
    torch.manual_seed(0)
    w = generate_target(TINY, 0, "cpu")
    m = hf_model(w)
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, TINY.vocab_size, (1, 48), generator=g)
    with torch.no_grad():
        out = m(ids, output_hidden_states=True)
    logits = out.logits[0]
    hs = out.hidden_states  # [0] = embeddings, [i+1] = after layer i
    top = torch.topk(logits, 8, dim=-1)
    blob = {
        "source": "transformers %s Qwen3ForCausalLM fp32 eager" % __import__("transformers").__version__,
        "ids": ids[0].clone(),
        "logits_head": logits[:, :256].clone(),
        "logits_sel": logits[:, 1000:1016].clone(),
        "top_idx": top.indices.clone(),
        "top_val": top.values.clone(),
        "lse": torch.logsumexp(logits, dim=-1).clone(),
        # hidden_states[i + 1] is the output of layer i, except the last entry, which HF
        # stores after the final norm
        "taps": {i: hs[i + 1][0, :, :64].clone() for i in TAPS if i + 1 < len(hs) - 1},
        "final_hidden_norm": hs[-1][0, :, :64].clone(),
    }
    torch.save(blob, OUT)
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
