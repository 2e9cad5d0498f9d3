"""Checkpoint I/O: the mlx-community 8-bit target layout and the DeepSpec / z-lab drafter
layouts load exactly (targets bit for bit; bf16 drafters re-quantize to W8 within 1.5 steps), and
the loaders refuse what they cannot load with an error that names the problem (the
reference's tests/test_formats.py contract, restated for these formats)."""
import dataclasses
import json

import pytest
import torch

from mlx_dspark_b200 import checkpoint as ck
from mlx_dspark_b200.config import TARGETS, DFlashConfig, dflash_for, dspark_for
from mlx_dspark_b200.weights import generate_dflash, generate_dspark, generate_target


def test_safetensors_round_trip(tmp_path):
    g = torch.Generator().manual_seed(0)
    ts = {"a.bf16": torch.randn(3, 5, generator=g).to(torch.bfloat16),
          "b.f16": torch.randn(7, generator=g).to(torch.float16),
          "c.f32": torch.randn(2, 2, 2, generator=g),
          "d.u8": torch.randint(0, 256, (4, 6), dtype=torch.uint8, generator=g),
          "e.i32": torch.randint(-2 ** 31, 2 ** 31 - 1, (9,), dtype=torch.int64, generator=g).to(torch.int32),
          "f.words": torch.tensor([[0, -1, 2 ** 31 - 1, -2 ** 31]], dtype=torch.int32),
          "g.empty": torch.zeros(0, 4)}
    p = str(tmp_path / "x.safetensors")
    ck.write_safetensors(p, ts, u32=("f.words",), metadata={"format": "mlx"})
    back = ck.read_safetensors(p)
    assert set(back) == set(ts)
    for k, v in ts.items():
        assert back[k].dtype == v.dtype and torch.equal(back[k], v), k
    raw = open(p, "rb").read()
    n = int.from_bytes(raw[:8], "little")
    hdr = json.loads(raw[8:8 + n])
    assert hdr["f.words"]["dtype"] == "U32" and hdr["__metadata__"] == {"format": "mlx"}


def test_u8x4_packing_order_and_round_trip():
    q = torch.tensor([[1, 2, 3, 4, 250, 0, 255, 128]], dtype=torch.uint8)
    w = ck.pack_u8x4(q)
    # the first value of each group of four in the lowest byte
    assert int(w[0, 0]) & 0xFFFFFFFF == 0x04030201
    assert int(w[0, 1]) & 0xFFFFFFFF == 0x80FF00FA
    assert torch.equal(ck.unpack_u8x4(w), q)
    g = torch.Generator().manual_seed(3)
    q = torch.randint(0, 256, (33, 64), dtype=torch.uint8, generator=g)
    assert torch.equal(ck.unpack_u8x4(ck.pack_u8x4(q)), q)


def _same_qt(a, b):
    return torch.equal(a.q, b.q) and torch.equal(a.scales, b.scales) and torch.equal(a.biases, b.biases)


@pytest.fixture(scope="module")
def tiny_target():
    return generate_target(TARGETS["tiny"], 0, "cpu")


def test_target_checkpoint_round_trip_is_exact(tmp_path, tiny_target):
    tw = tiny_target
    ck.export_target_checkpoint(tw, str(tmp_path), max_shard_bytes=8 << 20)  # several shards
    assert len(list(tmp_path.glob("*.safetensors"))) > 1
    back = ck.load_target_checkpoint(str(tmp_path))
    assert back.cfg == tw.cfg
    assert _same_qt(back.embed, tw.embed)
    assert (back.lm_head is None) == (tw.lm_head is None)
    if tw.lm_head is not None:
        assert _same_qt(back.lm_head, tw.lm_head)
    assert torch.equal(back.norm, tw.norm)
    for a, b in zip(back.layers, tw.layers):
        for f in ("wq", "wk", "wv", "wo", "gate", "up", "down"):
            assert _same_qt(getattr(a, f), getattr(b, f)), f
        for f in ("input_ln", "post_ln", "q_norm", "k_norm"):
            assert torch.equal(getattr(a, f), getattr(b, f)), f


def _edit_config(path, **changes):
    c = json.loads((path / "config.json").read_text())
    c.update(changes)
    (path / "config.json").write_text(json.dumps(c))


@pytest.mark.parametrize("change,match", [
    ({"quantization": {"group_size": 64, "bits": 4}}, "8-bit, group-64"),
    ({"quantization": {"group_size": 32, "bits": 8}}, "8-bit, group-64"),
    ({"quantization": None}, "8-bit, group-64"),
    ({"model_type": "llama"}, "unsupported target family"),
])
def test_target_config_refusals(tmp_path, tiny_target, change, match):
    ck.export_target_checkpoint(tiny_target, str(tmp_path))
    _edit_config(tmp_path, **change)
    with pytest.raises(ValueError, match=match):
        ck.load_target_checkpoint(str(tmp_path))


def test_target_name_mismatch_refused(tmp_path, tiny_target):
    ck.export_target_checkpoint(tiny_target, str(tmp_path))
    p = str(tmp_path / "model.safetensors")
    ts = ck.read_safetensors(p)
    words = tuple(k for k in ts if k.endswith(".weight") and ts[k].dtype == torch.int32)
    extra = dict(ts)
    extra["model.layers.0.self_attn.rotary_emb.bogus"] = torch.zeros(1)
    ck.write_safetensors(p, extra, u32=words)
    with pytest.raises(ValueError, match="unexpected in checkpoint"):
        ck.load_target_checkpoint(str(tmp_path))
    missing = dict(ts)
    del missing["model.layers.1.mlp.down_proj.scales"]
    ck.write_safetensors(p, missing, u32=tuple(k for k in words if k in missing))
    with pytest.raises(ValueError, match="missing in checkpoint"):
        ck.load_target_checkpoint(str(tmp_path))


def _dspark_config_json(cfg) -> dict:
    d = {k: v for k, v in dataclasses.asdict(cfg).items()
         if k not in ("family", "shared_embeddings", "norm_style")}
    d["model_type"] = "qwen3"
    return d


def _close_to_one_step(qa, qb):
    """Dequantized tensors within 1.5 quantization steps of b's groups. The bf16 export moves
    a weight by at most |w| * 2^-9, about half a step when |w| spans the group's range
    (255 steps); re-quantizing adds at most half a new step, and the new scale and bias are
    rounded to bf16 again. The tiny drafter's worst element is at 1.33 steps."""
    a, b = qa.dequant(), qb.dequant()
    step = qb.scales.float().repeat_interleave(64, dim=1)
    return bool(((a - b).abs() <= step * 1.5 + 1e-7).all())


@pytest.fixture(scope="module")
def tiny_dspark():
    cfg = dspark_for(TARGETS["tiny"])
    cfg = dataclasses.replace(cfg, shared_embeddings=False)
    return generate_dspark(cfg, 0, "cpu")


def test_dspark_checkpoint_round_trip(tmp_path, tiny_dspark):
    dw = tiny_dspark
    ck.export_dspark_checkpoint(dw, str(tmp_path), _dspark_config_json(dw.cfg))
    back = ck.load_dspark_checkpoint(str(tmp_path))
    for f in ("hidden_size", "num_hidden_layers", "block_size", "mask_token_id",
              "target_layer_ids", "markov_rank", "vocab_size"):
        assert getattr(back.cfg, f) == getattr(dw.cfg, f), f
    assert _close_to_one_step(back.fc, dw.fc)
    assert _close_to_one_step(back.markov_w1, dw.markov_w1)
    assert _close_to_one_step(back.markov_w2, dw.markov_w2)
    assert _close_to_one_step(back.embed, dw.embed) and _close_to_one_step(back.lm_head, dw.lm_head)
    for a, b in zip(back.layers, dw.layers):
        for f in ("wq", "wk", "wv", "wo", "gate", "up", "down"):
            assert _close_to_one_step(getattr(a, f), getattr(b, f)), f
        assert torch.equal(a.q_norm, b.q_norm) and torch.equal(a.input_ln, b.input_ln)
    assert torch.equal(back.norm, dw.norm) and torch.equal(back.hidden_norm, dw.hidden_norm)


def test_dspark_confidence_head_round_trip_and_size_check(tmp_path):
    base = dataclasses.replace(dspark_for(TARGETS["tiny"]), shared_embeddings=False)
    cfg = dataclasses.replace(base, enable_confidence_head=True)
    dw = generate_dspark(cfg, 0, "cpu")
    assert dw.conf_w.shape == (cfg.hidden_size + cfg.markov_rank,) and dw.conf_b.shape == (1,)
    ck.export_dspark_checkpoint(dw, str(tmp_path), _dspark_config_json(cfg))
    back = ck.load_dspark_checkpoint(str(tmp_path))
    assert torch.equal(back.conf_w, dw.conf_w) and torch.equal(back.conf_b, dw.conf_b)
    # the other tensors do not depend on the head being there
    plain = generate_dspark(base, 0, "cpu")
    assert plain.conf_w is None and torch.equal(plain.fc.q, dw.fc.q)
    p = str(tmp_path / "model.safetensors")
    ts = ck.read_safetensors(p)
    ts["confidence_head.proj.weight"] = ts["confidence_head.proj.weight"][:, :-1].contiguous()
    ck.write_safetensors(p, ts)
    with pytest.raises(ValueError, match="confidence_head.proj"):
        ck.load_dspark_checkpoint(str(tmp_path))


def test_dspark_name_mismatch_strict_and_relaxed(tmp_path, tiny_dspark):
    ck.export_dspark_checkpoint(tiny_dspark, str(tmp_path), _dspark_config_json(tiny_dspark.cfg))
    p = str(tmp_path / "model.safetensors")
    ts = ck.read_safetensors(p)
    extra = dict(ts)
    extra["bogus.weight"] = torch.zeros(2, dtype=torch.bfloat16)
    ck.write_safetensors(p, extra)
    with pytest.raises(ValueError, match="don't match"):
        ck.load_dspark_checkpoint(str(tmp_path))
    with pytest.warns(UserWarning, match="extra tensors ignored"):
        ck.load_dspark_checkpoint(str(tmp_path), strict=False)
    renamed = dict(ts)
    renamed["bogus.weight"] = renamed.pop("lm_head.weight")
    ck.write_safetensors(p, renamed)
    with pytest.raises(ValueError, match="missing in checkpoint"):
        ck.load_dspark_checkpoint(str(tmp_path), strict=False)  # a missing tensor never loads


def test_dspark_config_refusals_still_apply(tmp_path, tiny_dspark):
    ck.export_dspark_checkpoint(tiny_dspark, str(tmp_path), _dspark_config_json(tiny_dspark.cfg))
    _edit_config(tmp_path, speculators_config={"algorithm": "dspark"})
    with pytest.raises(ValueError, match="speculators"):
        ck.load_dspark_checkpoint(str(tmp_path))


def _dflash_config_json(cfg: DFlashConfig) -> dict:
    d = dataclasses.asdict(cfg)
    d["model_type"] = "qwen3"
    d["architectures"] = ["DFlashDraftModel"]
    d["target_layer_ids"] = list(cfg.target_layer_ids)
    d["layer_types"] = list(cfg.layer_types)
    return d


def test_dflash_checkpoint_round_trip_and_refusals(tmp_path):
    cfg = dflash_for(TARGETS["tiny"])
    dw = generate_dflash(cfg, 0, "cpu")
    ck.export_dflash_checkpoint(dw, str(tmp_path), _dflash_config_json(cfg))
    back = ck.load_dflash_checkpoint(str(tmp_path))
    assert back.cfg.block_size == cfg.block_size and back.cfg.target_layer_ids == tuple(cfg.target_layer_ids)
    assert _close_to_one_step(back.fc, dw.fc)
    for a, b in zip(back.layers, dw.layers):
        assert _close_to_one_step(a.down, b.down) and torch.equal(a.k_norm, b.k_norm)
    _edit_config(tmp_path, markov_rank=256)
    with pytest.raises(ValueError, match="Markov head"):
        ck.load_dflash_checkpoint(str(tmp_path))
    _edit_config(tmp_path, markov_rank=0,
                 layer_types=["sliding_attention"] + ["full_attention"] * (cfg.num_hidden_layers - 1))
    with pytest.raises(ValueError, match="sliding-window"):
        ck.load_dflash_checkpoint(str(tmp_path))
