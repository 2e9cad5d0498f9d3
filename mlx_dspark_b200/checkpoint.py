"""Checkpoint I/O: the on-disk formats on either side of the verify path.

- Targets: mlx-community 8-bit Qwen3 checkpoints (what the reference's ``load_target`` hands to
  mlx-lm, src/mlx_dspark/load.py:291-373): ``config.json`` with ``quantization: {group_size: 64,
  bits: 8}``, and safetensors holding, per linear, ``weight`` uint32 [N, K/4] (four 8-bit
  values per word, the first in the lowest byte), ``scales`` and ``biases`` [N, K/64]; norms as
  vectors. Names follow mlx-lm's qwen3 module tree (``model.embed_tokens``,
  ``model.layers.{i}.self_attn.{q,k,v,o}_proj``, ``...q_norm``, ``...mlp.{gate,up,down}_proj``,
  ``...input_layernorm``, ``...post_attention_layernorm``, ``model.norm``, ``lm_head`` unless
  ``tie_word_embeddings``).
- DSpark drafters: DeepSpec-format bf16 checkpoints loaded by exact parameter names with the
  reference's strictness (load.py:155-215): a name mismatch raises unless ``strict=False``.
  Linears are quantized to W8 g64 at load (the reference quantizes its drafter too, by default
  to 4 bits; the kernels here are W8).
- DFlash drafters: z-lab bf16 checkpoints (load.py:224-289): names must match exactly; a
  DFlash backbone carrying a DSpark Markov head is refused with that reason.

Safetensors are read and written here directly (8-byte little-endian header length, a JSON
header of {name: {dtype, shape, data_offsets}}, then the raw little-endian data), so no
package beyond torch is needed.
"""
from __future__ import annotations

import glob
import json
import os
import struct
import warnings

import torch

from .config import DFlashConfig, DSparkConfig, TargetConfig
from .weights import (GROUP, DFlashWeights, DSparkWeights, LayerWeights, QTensor,
                      TargetWeights, confidence_in_dim, quantize_w8g64)

# ------------------------------------------------------------------------------------------
# safetensors
_DTYPES = {"BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32,
           "F64": torch.float64, "U8": torch.uint8, "I8": torch.int8, "I16": torch.int16,
           "I32": torch.int32, "I64": torch.int64, "BOOL": torch.bool,
           "U32": torch.int32}  # 32-bit words: kept as int32 with the same bits
_NAMES = {torch.bfloat16: "BF16", torch.float16: "F16", torch.float32: "F32",
          torch.float64: "F64", torch.uint8: "U8", torch.int8: "I8", torch.int16: "I16",
          torch.int32: "I32", torch.int64: "I64", torch.bool: "BOOL"}


def read_safetensors(path: str) -> dict[str, torch.Tensor]:
    """Every tensor of one safetensors file (CPU tensors owning their memory)."""
    out: dict[str, torch.Tensor] = {}
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        base = 8 + n
        for name, info in header.items():
            if name == "__metadata__":
                continue
            dt = info["dtype"]
            if dt not in _DTYPES:
                raise ValueError(f"{path}: tensor {name!r} has unsupported dtype {dt}")
            b, e = info["data_offsets"]
            f.seek(base + b)
            raw = bytearray(f.read(e - b))
            t = torch.frombuffer(raw, dtype=_DTYPES[dt]) if raw else torch.empty(0, dtype=_DTYPES[dt])
            out[name] = t.reshape(info["shape"])
    return out


def write_safetensors(path: str, tensors: dict[str, torch.Tensor], *, u32: tuple = (),
                      metadata: dict | None = None) -> None:
    """Write tensors (names in ``u32`` are int32 words stored with dtype U32)."""
    header: dict = {}
    blobs = []
    off = 0
    for name in sorted(tensors):
        t = tensors[name].detach().contiguous().cpu()
        dt = "U32" if name in u32 else _NAMES.get(t.dtype)
        if dt is None:
            raise ValueError(f"cannot store dtype {t.dtype} ({name})")
        raw = t.reshape(-1).view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": dt, "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for raw in blobs:
            f.write(raw)


def _read_dir(path: str) -> dict[str, torch.Tensor]:
    files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"{path}: no *.safetensors files")
    out: dict[str, torch.Tensor] = {}
    for p in files:
        out.update(read_safetensors(p))
    return out


def _check_names(path: str, what: str, expected: set, got: set, *, strict: bool,
                 ignorable: set = frozenset()) -> None:
    missing = sorted(expected - got)
    unexpected = sorted(got - expected - ignorable)
    if not missing and not unexpected:
        return
    detail = ""
    if missing:
        detail += f"\n  missing in checkpoint ({len(missing)}): {missing[:8]}"
    if unexpected:
        detail += f"\n  unexpected in checkpoint ({len(unexpected)}): {unexpected[:8]}"
    if strict or missing:
        raise ValueError(f"{path}: tensor names don't match {what}.{detail}"
                         + ("\n  (strict=False loads a checkpoint whose only mismatch is extra "
                            "tensors)" if not missing else ""))
    warnings.warn(f"{path}: key mismatch, extra tensors ignored:{detail}")


# ------------------------------------------------------------------------------------------
# mlx 8-bit packing (four values per 32-bit word, the first in the lowest byte)
def unpack_u8x4(w: torch.Tensor) -> torch.Tensor:
    """int32 [N, K/4] words -> uint8 [N, K]."""
    w = w.to(torch.int64) & 0xFFFFFFFF
    parts = [((w >> (8 * j)) & 0xFF) for j in range(4)]
    return torch.stack(parts, dim=-1).reshape(w.shape[0], -1).to(torch.uint8)


def pack_u8x4(q: torch.Tensor) -> torch.Tensor:
    """uint8 [N, K] -> int32 [N, K/4] words (the inverse of unpack_u8x4)."""
    N, K = q.shape
    if K % 4:
        raise ValueError("K must be a multiple of 4")
    v = q.to(torch.int64).reshape(N, K // 4, 4)
    w = v[..., 0] | (v[..., 1] << 8) | (v[..., 2] << 16) | (v[..., 3] << 24)
    return torch.where(w >= 2 ** 31, w - 2 ** 32, w).to(torch.int32)


def _as_bf16(t: torch.Tensor, name: str) -> torch.Tensor:
    """Norm weights as the kernels read them, bf16. An fp16 checkpoint's values are rounded to
    bf16 (a relative change of at most 2^-9 on a norm weight); fp32 values must be exact in
    bf16."""
    if t.dtype == torch.bfloat16:
        return t
    b = t.to(torch.bfloat16)
    if t.dtype != torch.float16 and not torch.equal(b.to(t.dtype), t):
        raise ValueError(f"{name}: {t.dtype} values are not exactly representable in bf16")
    return b


def _scale_dtype(t: torch.Tensor, name: str) -> torch.Tensor:
    """Quantization scales / biases as stored: bf16 or fp16 (an fp16 source model's 8-bit
    checkpoint) kept as they are; fp32 narrowed to bf16 or fp16 when one holds it exactly."""
    if t.dtype in (torch.bfloat16, torch.float16):
        return t
    for dt in (torch.bfloat16, torch.float16):
        n = t.to(dt)
        if torch.equal(n.to(t.dtype), t):
            return n
    raise ValueError(f"{name}: {t.dtype} values are exact in neither bf16 nor fp16")


def _qtensor(ts: dict, prefix: str, N: int, K: int) -> QTensor:
    w, s, b = ts[prefix + ".weight"], ts[prefix + ".scales"], ts[prefix + ".biases"]
    if tuple(w.shape) != (N, K // 4) or tuple(s.shape) != (N, K // GROUP) or tuple(b.shape) != (N, K // GROUP):
        raise ValueError(f"{prefix}: shapes {tuple(w.shape)}, {tuple(s.shape)}, {tuple(b.shape)} do "
                         f"not fit an 8-bit group-64 [{N}, {K}] linear")
    return QTensor(unpack_u8x4(w), _scale_dtype(s, prefix + ".scales"),
                   _scale_dtype(b, prefix + ".biases"))


# ------------------------------------------------------------------------------------------
# targets (mlx-community 8-bit Qwen3)
def _linears(cfg: TargetConfig) -> dict[str, tuple[int, int]]:
    """Relative linear names of one decoder layer -> (N, K)."""
    H, I, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    return {"self_attn.q_proj": (cfg.num_attention_heads * hd, H),
            "self_attn.k_proj": (cfg.num_key_value_heads * hd, H),
            "self_attn.v_proj": (cfg.num_key_value_heads * hd, H),
            "self_attn.o_proj": (H, cfg.num_attention_heads * hd),
            "mlp.gate_proj": (I, H), "mlp.up_proj": (I, H), "mlp.down_proj": (H, I)}


def _norms() -> tuple:
    return ("self_attn.q_norm", "self_attn.k_norm", "input_layernorm", "post_attention_layernorm")


def target_config_from_json(path: str) -> TargetConfig:
    """TargetConfig of an mlx-community Qwen3 8-bit checkpoint directory (its config.json)."""
    with open(os.path.join(path, "config.json")) as f:
        c = json.load(f)
    mt = c.get("model_type", "")
    if mt != "qwen3":
        raise ValueError(f"{path}: unsupported target family (model_type={mt!r}); this build "
                         f"runs dense qwen3 targets")
    qz = c.get("quantization") or c.get("quantization_config")
    if not qz or qz.get("bits") != 8 or qz.get("group_size") != GROUP or \
            qz.get("mode", "affine") != "affine":
        raise ValueError(f"{path}: the W8 kernels need an 8-bit, group-64 affine checkpoint "
                         f"(config quantization: {qz!r})")
    rp = c.get("rope_parameters") or {}
    return TargetConfig(
        hidden_size=c["hidden_size"], num_hidden_layers=c["num_hidden_layers"],
        num_attention_heads=c["num_attention_heads"],
        num_key_value_heads=c.get("num_key_value_heads", c["num_attention_heads"]),
        head_dim=c.get("head_dim", c["hidden_size"] // c["num_attention_heads"]),
        intermediate_size=c["intermediate_size"], vocab_size=c["vocab_size"],
        rms_norm_eps=c.get("rms_norm_eps", 1e-6),
        rope_theta=c.get("rope_theta", rp.get("rope_theta", 1_000_000.0)),
        tie_word_embeddings=bool(c.get("tie_word_embeddings", False)))


def _target_names(cfg: TargetConfig) -> set:
    names = {f"model.embed_tokens.{p}" for p in ("weight", "scales", "biases")}
    names.add("model.norm.weight")
    if not cfg.tie_word_embeddings:
        names |= {f"lm_head.{p}" for p in ("weight", "scales", "biases")}
    for i in range(cfg.num_hidden_layers):
        for lin in _linears(cfg):
            names |= {f"model.layers.{i}.{lin}.{p}" for p in ("weight", "scales", "biases")}
        names |= {f"model.layers.{i}.{n}.weight" for n in _norms()}
    return names


def load_target_checkpoint(path: str) -> TargetWeights:
    """Canonical W8 weights of an mlx-community 8-bit Qwen3 checkpoint directory. Every
    expected tensor must be present and nothing else (a partially loaded target computes
    garbage; the reference's mlx-lm load is strict the same way)."""
    cfg = target_config_from_json(path)
    ts = _read_dir(path)
    _check_names(path, "an 8-bit mlx-community qwen3 target", _target_names(cfg), set(ts), strict=True)
    H, V = cfg.hidden_size, cfg.vocab_size
    embed = _qtensor(ts, "model.embed_tokens", V, H)
    layers = []
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        lin = {n: _qtensor(ts, p + n, *nk) for n, nk in _linears(cfg).items()}
        nrm = {n: _as_bf16(ts[p + n + ".weight"], p + n) for n in _norms()}
        layers.append(LayerWeights(
            nrm["input_layernorm"], nrm["post_attention_layernorm"], nrm["self_attn.q_norm"],
            nrm["self_attn.k_norm"], lin["self_attn.q_proj"], lin["self_attn.k_proj"],
            lin["self_attn.v_proj"], lin["self_attn.o_proj"], lin["mlp.gate_proj"],
            lin["mlp.up_proj"], lin["mlp.down_proj"]))
    norm = _as_bf16(ts["model.norm.weight"], "model.norm")
    head = None if cfg.tie_word_embeddings else _qtensor(ts, "lm_head", V, H)
    return TargetWeights(cfg, embed, layers, norm, head)


def export_target_checkpoint(tw: TargetWeights, path: str, *, max_shard_bytes: int = 2 << 30) -> None:
    """Write canonical target weights as an mlx-community 8-bit checkpoint directory."""
    os.makedirs(path, exist_ok=True)
    c = tw.cfg
    cfg = {"model_type": "qwen3", "hidden_size": c.hidden_size,
           "num_hidden_layers": c.num_hidden_layers, "num_attention_heads": c.num_attention_heads,
           "num_key_value_heads": c.num_key_value_heads, "head_dim": c.head_dim,
           "intermediate_size": c.intermediate_size, "vocab_size": c.vocab_size,
           "rms_norm_eps": c.rms_norm_eps, "rope_theta": c.rope_theta,
           "tie_word_embeddings": c.tie_word_embeddings,
           "quantization": {"group_size": GROUP, "bits": 8}}
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    items: dict[str, torch.Tensor] = {}
    u32: list[str] = []

    def put_q(prefix: str, qt: QTensor):
        items[prefix + ".weight"] = pack_u8x4(qt.q.cpu())
        u32.append(prefix + ".weight")
        items[prefix + ".scales"] = qt.scales.cpu()
        items[prefix + ".biases"] = qt.biases.cpu()

    put_q("model.embed_tokens", tw.embed)
    for i, L in enumerate(tw.layers):
        p = f"model.layers.{i}."
        for n, qt in (("self_attn.q_proj", L.wq), ("self_attn.k_proj", L.wk),
                      ("self_attn.v_proj", L.wv), ("self_attn.o_proj", L.wo),
                      ("mlp.gate_proj", L.gate), ("mlp.up_proj", L.up), ("mlp.down_proj", L.down)):
            put_q(p + n, qt)
        for n, t in (("input_layernorm", L.input_ln), ("post_attention_layernorm", L.post_ln),
                     ("self_attn.q_norm", L.q_norm), ("self_attn.k_norm", L.k_norm)):
            items[p + n + ".weight"] = t.cpu()
    items["model.norm.weight"] = tw.norm.cpu()
    if tw.lm_head is not None:
        put_q("lm_head", tw.lm_head)
    _write_shards(path, items, set(u32), max_shard_bytes)


def _write_shards(path: str, items: dict, u32: set, max_shard_bytes: int) -> None:
    shards: list[dict] = [{}]
    size = 0
    for name in sorted(items):
        nb = items[name].numel() * items[name].element_size()
        if shards[-1] and size + nb > max_shard_bytes:
            shards.append({})
            size = 0
        shards[-1][name] = items[name]
        size += nb
    n = len(shards)
    for k, sh in enumerate(shards):
        fn = "model.safetensors" if n == 1 else f"model-{k + 1:05d}-of-{n:05d}.safetensors"
        write_safetensors(os.path.join(path, fn), sh, u32=tuple(u32 & set(sh)),
                          metadata={"format": "mlx"})


# ------------------------------------------------------------------------------------------
# drafters (bf16 checkpoints, quantized to W8 g64 here)
def _drafter_layer_names(i: int, attention_bias: bool) -> set:
    p = f"layers.{i}."
    names = {p + f"self_attn.{n}.weight" for n in ("q_proj", "k_proj", "v_proj", "o_proj",
                                                   "q_norm", "k_norm")}
    if attention_bias:
        names |= {p + f"self_attn.{n}.bias" for n in ("q_proj", "k_proj", "v_proj", "o_proj")}
    names |= {p + f"mlp.{n}.weight" for n in ("gate_proj", "up_proj", "down_proj")}
    names |= {p + "input_layernorm.weight", p + "post_attention_layernorm.weight"}
    return names


def _bf16_layer(ts: dict, i: int) -> LayerWeights:
    p = f"layers.{i}."
    q = lambda n: quantize_w8g64(ts[p + n + ".weight"].float())  # noqa: E731
    v = lambda n: _as_bf16(ts[p + n + ".weight"], p + n)  # noqa: E731
    return LayerWeights(v("input_layernorm"), v("post_attention_layernorm"),
                        v("self_attn.q_norm"), v("self_attn.k_norm"), q("self_attn.q_proj"),
                        q("self_attn.k_proj"), q("self_attn.v_proj"), q("self_attn.o_proj"),
                        q("mlp.gate_proj"), q("mlp.up_proj"), q("mlp.down_proj"))


def dspark_names(cfg: DSparkConfig) -> set:
    """Parameter names of a DeepSpec-format qwen3 DSpark drafter (model.py:220-241)."""
    names = {"embed_tokens.weight", "fc.weight", "hidden_norm.weight", "norm.weight",
             "lm_head.weight"}
    for i in range(cfg.num_hidden_layers):
        names |= _drafter_layer_names(i, cfg.attention_bias)
    if cfg.markov_rank > 0:
        names |= {"markov_head.markov_w1.weight", "markov_head.markov_w2.weight"}
    if cfg.enable_confidence_head:
        names |= {"confidence_head.proj.weight", "confidence_head.proj.bias"}
    return names


def load_dspark_checkpoint(path: str, *, strict: bool = True) -> DSparkWeights:
    """W8 weights of a DeepSpec-format DSpark drafter directory (bf16 safetensors). A name
    mismatch raises (strict=True, the reference's default: a partly loaded drafter drafts
    near-zero acceptance); strict=False tolerates extra tensors with a warning. The confidence
    head's proj weight and bias are kept in bf16 (speculative_generate's confidence_threshold)."""
    cfg = DSparkConfig.from_json(os.path.join(path, "config.json"))
    if cfg.attention_bias:
        raise ValueError(f"{path}: attention biases are not supported by this build's drafter")
    ts = _read_dir(path)
    _check_names(path, "a DeepSpec-format DSpark drafter", dspark_names(cfg), set(ts),
                 strict=strict)
    layers = [_bf16_layer(ts, i) for i in range(cfg.num_hidden_layers)]
    w1 = w2 = None
    if cfg.markov_rank > 0:
        w1 = quantize_w8g64(ts["markov_head.markov_w1.weight"].float())
        w2 = quantize_w8g64(ts["markov_head.markov_w2.weight"].float())
    conf_w = conf_b = None
    if cfg.enable_confidence_head:
        conf_w = _as_bf16(ts["confidence_head.proj.weight"], "confidence_head.proj").reshape(-1)
        conf_b = _as_bf16(ts["confidence_head.proj.bias"], "confidence_head.proj.bias").reshape(-1)
        if conf_w.numel() != confidence_in_dim(cfg) or conf_b.numel() != 1:
            raise ValueError(f"{path}: confidence_head.proj has {conf_w.numel()} inputs and "
                             f"{conf_b.numel()} biases, expected {confidence_in_dim(cfg)} and 1")
    return DSparkWeights(cfg, quantize_w8g64(ts["fc.weight"].float()),
                         _as_bf16(ts["hidden_norm.weight"], "hidden_norm"), layers,
                         _as_bf16(ts["norm.weight"], "norm"), w1, w2,
                         quantize_w8g64(ts["embed_tokens.weight"].float()),
                         quantize_w8g64(ts["lm_head.weight"].float()), conf_w, conf_b)


def _layer_bf16(L: LayerWeights) -> dict:
    d = {"self_attn.q_proj": L.wq, "self_attn.k_proj": L.wk, "self_attn.v_proj": L.wv,
         "self_attn.o_proj": L.wo, "mlp.gate_proj": L.gate, "mlp.up_proj": L.up,
         "mlp.down_proj": L.down}
    out = {k + ".weight": v.dequant().to(torch.bfloat16) for k, v in d.items()}
    for k, t in (("input_layernorm", L.input_ln), ("post_attention_layernorm", L.post_ln),
                 ("self_attn.q_norm", L.q_norm), ("self_attn.k_norm", L.k_norm)):
        out[k + ".weight"] = t.cpu()
    return out


def export_dspark_checkpoint(dw: DSparkWeights, path: str, config: dict) -> None:
    """Write a drafter as a DeepSpec-format bf16 checkpoint (the W8 values dequantized);
    ``config`` is the config.json content."""
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(config, f, indent=1)
    items = {"fc.weight": dw.fc.dequant().to(torch.bfloat16),
             "hidden_norm.weight": dw.hidden_norm.cpu(), "norm.weight": dw.norm.cpu()}
    for i, L in enumerate(dw.layers):
        items.update({f"layers.{i}.{k}": v for k, v in _layer_bf16(L).items()})
    if dw.markov_w1 is not None:
        items["markov_head.markov_w1.weight"] = dw.markov_w1.dequant().to(torch.bfloat16)
        items["markov_head.markov_w2.weight"] = dw.markov_w2.dequant().to(torch.bfloat16)
    if dw.embed is not None:
        items["embed_tokens.weight"] = dw.embed.dequant().to(torch.bfloat16)
    if dw.lm_head is not None:
        items["lm_head.weight"] = dw.lm_head.dequant().to(torch.bfloat16)
    if dw.cfg.enable_confidence_head:
        din = confidence_in_dim(dw.cfg)
        w = dw.conf_w if dw.conf_w is not None else torch.zeros(din, dtype=torch.bfloat16)
        b = dw.conf_b if dw.conf_b is not None else torch.zeros(1, dtype=torch.bfloat16)
        items["confidence_head.proj.weight"] = w.cpu().reshape(1, din)
        items["confidence_head.proj.bias"] = b.cpu().reshape(1)
    write_safetensors(os.path.join(path, "model.safetensors"), items)


def dflash_config_from_json(path: str) -> DFlashConfig:
    """DFlashConfig of a z-lab checkpoint directory, with the reference's refusal of a DFlash
    backbone carrying a DSpark Markov head (load.py:236-245) and tolerance of a nested
    rope_parameters block."""
    with open(os.path.join(path, "config.json")) as f:
        c = json.load(f)
    if c.get("markov_rank"):
        raise ValueError(f"{path}: this DFlash checkpoint carries a Markov head "
                         f"(markov_rank={c['markov_rank']}), a DFlash+DSpark hybrid this build "
                         f"cannot load")
    rope = c.get("rope_parameters") or {}
    layer_types = tuple(c.get("layer_types") or ["full_attention"] * c["num_hidden_layers"])
    if any(t != "full_attention" for t in layer_types):
        raise ValueError(f"{path}: sliding-window DFlash layers are not supported by this build")
    dfc = c.get("dflash_config", {})
    return DFlashConfig(
        hidden_size=c["hidden_size"], num_hidden_layers=c["num_hidden_layers"],
        num_attention_heads=c["num_attention_heads"], num_key_value_heads=c["num_key_value_heads"],
        head_dim=c["head_dim"], intermediate_size=c["intermediate_size"],
        vocab_size=c["vocab_size"], rms_norm_eps=c["rms_norm_eps"],
        rope_theta=c.get("rope_theta", rope.get("rope_theta", 1_000_000.0)),
        max_position_embeddings=c.get("max_position_embeddings", 40960),
        block_size=c["block_size"],
        target_layer_ids=tuple(dfc.get("target_layer_ids") or c["target_layer_ids"]),
        num_target_layers=c["num_target_layers"],
        mask_token_id=dfc.get("mask_token_id", c.get("mask_token_id", 0)),
        layer_types=layer_types, sliding_window=c.get("sliding_window"),
        final_logit_softcapping=c.get("final_logit_softcapping"))


def dflash_names(cfg: DFlashConfig) -> set:
    """Parameter names of a z-lab DFlash drafter (dflash_model.py:150-166; no embed/head)."""
    names = {"fc.weight", "hidden_norm.weight", "norm.weight"}
    for i in range(cfg.num_hidden_layers):
        names |= _drafter_layer_names(i, False)
    return names


def load_dflash_checkpoint(path: str) -> DFlashWeights:
    """W8 weights of a z-lab DFlash drafter directory; names must match exactly."""
    cfg = dflash_config_from_json(path)
    ts = _read_dir(path)
    _check_names(path, "a z-lab DFlash drafter", dflash_names(cfg), set(ts), strict=True)
    layers = [_bf16_layer(ts, i) for i in range(cfg.num_hidden_layers)]
    return DFlashWeights(cfg, quantize_w8g64(ts["fc.weight"].float()),
                         _as_bf16(ts["hidden_norm.weight"], "hidden_norm"), layers,
                         _as_bf16(ts["norm.weight"], "norm"))


def export_dflash_checkpoint(dw: DFlashWeights, path: str, config: dict) -> None:
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(config, f, indent=1)
    items = {"fc.weight": dw.fc.dequant().to(torch.bfloat16),
             "hidden_norm.weight": dw.hidden_norm.cpu(), "norm.weight": dw.norm.cpu()}
    for i, L in enumerate(dw.layers):
        items.update({f"layers.{i}.{k}": v for k, v in _layer_bf16(L).items()})
    write_safetensors(os.path.join(path, "model.safetensors"), items)


__all__ = ["read_safetensors", "write_safetensors", "pack_u8x4", "unpack_u8x4",
           "target_config_from_json", "load_target_checkpoint", "export_target_checkpoint",
           "dspark_names", "load_dspark_checkpoint", "export_dspark_checkpoint",
           "dflash_config_from_json", "dflash_names", "load_dflash_checkpoint",
           "export_dflash_checkpoint"]
