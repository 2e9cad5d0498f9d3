"""Seeded synthetic W8 checkpoints and their packing into the kernel layout.

Canonical form (what a checkpoint holds and what the CPU oracle reads): for every linear
``W[N, K]`` an affine 8-bit group-64 quantization ``q`` uint8 ``[N, K]`` with ``scales`` and
``biases`` bf16 ``[N, K/64]``, ``W ~= scales * q + biases`` per 64-wide group along K — the
tensor set of an mlx-community 8-bit checkpoint (``quantization: {group_size: 64, bits: 8}``)
with the 4-per-uint32 packing undone. Norm weights are bf16 vectors.

Kernel form (``PackedLinear``): the same ``q`` plus ``sb`` int32 ``[K/64, N]`` whose low half
is the fp16 scale and whose high half is the fp16 bias of group (n, g) — the layout the TMA
producer of the W8A16 GEMM streams. Fused projections are packed once at load time:
q|k|v rows concatenated, gate/up interleaved in 64-row halves of each 128-row tile.

Weights are drawn N(0, 0.02) from one ``torch.Generator`` seeded with ``seed`` on the
generating device, tensor by tensor in a fixed order, then quantized with this module's
quantizer (scale = (max - min) / 255, bias = min, both rounded to bf16, q = round((w - bias)
/ scale) clamped to [0, 255]). The oracle and the GPU receive the *same* quantized tensors,
so parity never depends on a quantizer's rounding.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from .config import DFlashConfig, DSparkConfig, TargetConfig

GROUP = 64
STD = 0.02


@dataclass
class QTensor:
    """Canonical W8 affine group-64 tensor."""

    q: torch.Tensor       # uint8 [N, K]
    scales: torch.Tensor  # bf16 (or an fp16 checkpoint's fp16) [N, K/64]
    biases: torch.Tensor  # bf16 [N, K/64]

    @property
    def shape(self):
        return tuple(self.q.shape)

    def dequant(self, dtype=torch.float32) -> torch.Tensor:
        N, K = self.q.shape
        s = self.scales.to(torch.float32).repeat_interleave(GROUP, dim=1)
        b = self.biases.to(torch.float32).repeat_interleave(GROUP, dim=1)
        return (s * self.q.to(torch.float32) + b).to(dtype)

    def to(self, device) -> "QTensor":
        return QTensor(self.q.to(device), self.scales.to(device), self.biases.to(device))

    def nbytes(self) -> int:
        return self.q.numel() + 2 * self.scales.numel() * 2


def quantize_w8g64(w: torch.Tensor) -> QTensor:
    """Affine 8-bit, group 64 along the last axis (this build's own quantizer)."""
    N, K = w.shape
    assert K % GROUP == 0, K
    g = w.to(torch.float32).reshape(N, K // GROUP, GROUP)
    mn = g.amin(dim=-1)
    mx = g.amax(dim=-1)
    scale = ((mx - mn) / 255.0).to(torch.bfloat16)
    bias = mn.to(torch.bfloat16)
    sf = scale.to(torch.float32).unsqueeze(-1)
    bf = bias.to(torch.float32).unsqueeze(-1)
    q = torch.where(sf > 0, torch.round((g - bf) / torch.where(sf > 0, sf, torch.ones_like(sf))),
                    torch.zeros_like(g))
    q = q.clamp_(0, 255).to(torch.uint8).reshape(N, K)
    return QTensor(q, scale, bias)


def _randn(gen: torch.Generator, shape, device) -> torch.Tensor:
    return torch.randn(*shape, generator=gen, device=device, dtype=torch.float32)


def _qlinear(gen, N, K, device) -> QTensor:
    w = _randn(gen, (N, K), device) * STD
    t = quantize_w8g64(w)
    del w
    return t


def _norm(gen, n, device) -> torch.Tensor:
    return (1.0 + 0.1 * _randn(gen, (n,), device)).to(torch.bfloat16)


# ----------------------------------------------------------------------------------------
# canonical checkpoints
@dataclass
class LayerWeights:
    input_ln: torch.Tensor
    post_ln: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    wq: QTensor
    wk: QTensor
    wv: QTensor
    wo: QTensor
    gate: QTensor
    up: QTensor
    down: QTensor


@dataclass
class TargetWeights:
    cfg: TargetConfig
    embed: QTensor
    layers: list[LayerWeights]
    norm: torch.Tensor
    lm_head: QTensor | None  # None when tied (the embedding is the head)

    @property
    def head(self) -> QTensor:
        return self.embed if self.lm_head is None else self.lm_head

    def to(self, device) -> "TargetWeights":
        return TargetWeights(
            self.cfg, self.embed.to(device),
            [LayerWeights(*(getattr(l, f).to(device) for f in LayerWeights.__dataclass_fields__))
             for l in self.layers],
            self.norm.to(device), None if self.lm_head is None else self.lm_head.to(device))


def _layer(gen, cfg, device) -> LayerWeights:
    H, I, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    wq = _qlinear(gen, cfg.num_attention_heads * hd, H, device)
    wk = _qlinear(gen, cfg.num_key_value_heads * hd, H, device)
    wv = _qlinear(gen, cfg.num_key_value_heads * hd, H, device)
    wo = _qlinear(gen, H, cfg.num_attention_heads * hd, device)
    gate = _qlinear(gen, I, H, device)
    up = _qlinear(gen, I, H, device)
    down = _qlinear(gen, H, I, device)
    input_ln = _norm(gen, H, device)
    post_ln = _norm(gen, H, device)
    q_norm = _norm(gen, hd, device)
    k_norm = _norm(gen, hd, device)
    return LayerWeights(input_ln, post_ln, q_norm, k_norm, wq, wk, wv, wo, gate, up, down)


def generate_target(cfg: TargetConfig, seed: int, device="cpu") -> TargetWeights:
    """Seeded random-init Qwen3 target, quantized W8 g64 (see module docstring)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    embed = _qlinear(gen, cfg.vocab_size, cfg.hidden_size, device)
    layers = [_layer(gen, cfg, device) for _ in range(cfg.num_hidden_layers)]
    norm = _norm(gen, cfg.hidden_size, device)
    lm_head = None if cfg.tie_word_embeddings else _qlinear(gen, cfg.vocab_size, cfg.hidden_size, device)
    return TargetWeights(cfg, embed, layers, norm, lm_head)


@dataclass
class DSparkWeights:
    cfg: DSparkConfig
    fc: QTensor                 # [H, n_tap*H]
    hidden_norm: torch.Tensor
    layers: list[LayerWeights]
    norm: torch.Tensor
    markov_w1: QTensor | None   # [V, R] embedding
    markov_w2: QTensor | None   # [V, R] linear R -> V
    embed: QTensor | None = None    # None: the target's embedding is shared
    lm_head: QTensor | None = None  # None: the target's head is shared
    # confidence head proj (model.py:211-217): bf16 [H (+ R)] weight row and bf16 [1] bias
    conf_w: torch.Tensor | None = None
    conf_b: torch.Tensor | None = None

    def to(self, device) -> "DSparkWeights":
        f = lambda t: None if t is None else t.to(device)  # noqa: E731
        return DSparkWeights(
            self.cfg, self.fc.to(device), self.hidden_norm.to(device),
            [LayerWeights(*(getattr(l, k).to(device) for k in LayerWeights.__dataclass_fields__))
             for l in self.layers],
            self.norm.to(device), f(self.markov_w1), f(self.markov_w2), f(self.embed),
            f(self.lm_head), f(self.conf_w), f(self.conf_b))


def generate_dspark(cfg: DSparkConfig, seed: int, device="cpu") -> DSparkWeights:
    gen = torch.Generator(device=device)
    gen.manual_seed(seed + 1_000_003)
    H = cfg.hidden_size
    tcfg = TargetConfig(hidden_size=H, num_hidden_layers=cfg.num_hidden_layers,
                        num_attention_heads=cfg.num_attention_heads,
                        num_key_value_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim,
                        intermediate_size=cfg.intermediate_size, vocab_size=cfg.vocab_size)
    fc = _qlinear(gen, H, len(cfg.target_layer_ids) * H, device)
    hidden_norm = _norm(gen, H, device)
    layers = [_layer(gen, tcfg, device) for _ in range(cfg.num_hidden_layers)]
    norm = _norm(gen, H, device)
    w1 = w2 = None
    if cfg.markov_rank > 0:
        w1 = _qlinear(gen, cfg.vocab_size, cfg.markov_rank, device)
        w2 = _qlinear(gen, cfg.vocab_size, cfg.markov_rank, device)
    embed = lm_head = None
    if not cfg.shared_embeddings:
        embed = _qlinear(gen, cfg.vocab_size, H, device)
        lm_head = _qlinear(gen, cfg.vocab_size, H, device)
    conf_w = conf_b = None
    if cfg.enable_confidence_head:
        # drawn last so the other tensors do not depend on the flag; a logit ~ N(2, 1) keeps
        # the per-position survival probabilities in the range where truncation varies
        din = confidence_in_dim(cfg)
        conf_w = (_randn(gen, (din,), device) * din ** -0.5).to(torch.bfloat16)
        conf_b = torch.full((1,), 2.0, dtype=torch.bfloat16, device=device)
    return DSparkWeights(cfg, fc, hidden_norm, layers, norm, w1, w2, embed, lm_head, conf_w,
                         conf_b)


def confidence_in_dim(cfg: DSparkConfig) -> int:
    """Input width of the confidence head: H, plus the Markov rank when the head also reads the
    previous token's Markov embedding (model.py:240-242)."""
    with_markov = cfg.confidence_head_with_markov and cfg.markov_rank > 0
    return cfg.hidden_size + (cfg.markov_rank if with_markov else 0)


@dataclass
class DFlashWeights:
    cfg: DFlashConfig
    fc: QTensor
    hidden_norm: torch.Tensor
    layers: list[LayerWeights]
    norm: torch.Tensor

    def to(self, device) -> "DFlashWeights":
        return DFlashWeights(
            self.cfg, self.fc.to(device), self.hidden_norm.to(device),
            [LayerWeights(*(getattr(l, k).to(device) for k in LayerWeights.__dataclass_fields__))
             for l in self.layers],
            self.norm.to(device))


def generate_dflash(cfg: DFlashConfig, seed: int, device="cpu") -> DFlashWeights:
    gen = torch.Generator(device=device)
    gen.manual_seed(seed + 2_000_003)
    H = cfg.hidden_size
    tcfg = TargetConfig(hidden_size=H, num_hidden_layers=cfg.num_hidden_layers,
                        num_attention_heads=cfg.num_attention_heads,
                        num_key_value_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim,
                        intermediate_size=cfg.intermediate_size, vocab_size=cfg.vocab_size)
    fc = _qlinear(gen, H, len(cfg.target_layer_ids) * H, device)
    hidden_norm = _norm(gen, H, device)
    layers = [_layer(gen, tcfg, device) for _ in range(cfg.num_hidden_layers)]
    norm = _norm(gen, H, device)
    return DFlashWeights(cfg, fc, hidden_norm, layers, norm)


# ----------------------------------------------------------------------------------------
# kernel packing
@dataclass
class PackedLinear:
    """Kernel layout of a W8 g64 linear: ``q`` uint8 [N, K], ``sb`` int32 [K/64, N]."""

    q: torch.Tensor
    sb: torch.Tensor
    N: int
    K: int

    def nbytes(self) -> int:
        return self.q.numel() + self.sb.numel() * 4


def _sb(scales: torch.Tensor, biases: torch.Tensor) -> torch.Tensor:
    """(scale, bias) [N, G] -> int32 [G, N] of fp16 pairs, the GEMM's dequantization operands.
    fp16 holds every bf16 value of magnitude 2^-17 .. 65504 exactly (11 significand bits
    against 8) and every fp16 checkpoint value. Smaller magnitudes (the groups of a nearly
    constant weight row; MLX's quantizer floors a scale at 1e-7) round to fp16 subnormals, an
    absolute error of at most 2^-25 per scale or bias, so at most 255 * 2^-25 ~ 7.6e-6 on a
    weight of such a group. Values past the fp16 range are refused."""
    s16 = scales.to(torch.float16)
    b16 = biases.to(torch.float16)
    for a, name in ((s16, "scale"), (b16, "bias")):
        if not torch.isfinite(a).all():
            bad = (~torch.isfinite(a)).sum().item()
            raise ValueError(f"{bad} W8 {name} values are outside the fp16 range")
    lo = s16.view(torch.int16).to(torch.int32) & 0xFFFF
    hi = b16.view(torch.int16).to(torch.int32) << 16
    return (lo | hi).t().contiguous()


def pack(*parts: QTensor, interleave64: bool = False, device="cuda") -> PackedLinear:
    """Pack one or more canonical linears (row-concatenated) for the GEMM kernel.
    ``interleave64``: two parts (gate, up) interleaved in 64-row halves per 128-row tile."""
    if interleave64:
        assert len(parts) == 2
        g, u = parts
        N, K = g.q.shape
        assert N % 64 == 0
        def il(a, b):
            a = a.reshape(N // 64, 64, -1)
            b = b.reshape(N // 64, 64, -1)
            return torch.stack([a, b], dim=1).reshape(2 * N, -1)
        q = il(g.q.to(device), u.q.to(device))
        sc = il(g.scales.to(device), u.scales.to(device))
        bi = il(g.biases.to(device), u.biases.to(device))
    else:
        q = torch.cat([p.q.to(device) for p in parts], dim=0) if len(parts) > 1 else parts[0].q.to(device)
        sc = torch.cat([p.scales.to(device) for p in parts], dim=0)
        bi = torch.cat([p.biases.to(device) for p in parts], dim=0)
    q = q.contiguous()
    N, K = q.shape
    return PackedLinear(q, _sb(sc, bi), N, K)

