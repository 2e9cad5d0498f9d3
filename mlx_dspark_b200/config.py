"""Model configurations: the Qwen3 target shape, the DSpark and DFlash drafter configs, and
the named workload presets of the benchmark (C1..C5).

``DSparkConfig`` keeps the field names of the reference (src/mlx_dspark/config.py:67-133)
for the qwen3 family; ``DFlashConfig`` mirrors src/mlx_dspark/dflash_model.py:52-71.
``from_json`` applies the same format refusals as the reference (config.py:87-185).
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field, replace
from pathlib import Path


@dataclass(frozen=True)
class TargetConfig:
    """Dense Qwen3 decoder: pre-RMSNorm, per-head q/k RMSNorm, rotate-half RoPE, GQA, SwiGLU."""

    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    intermediate_size: int
    vocab_size: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    tie_word_embeddings: bool = False
    model_type: str = "qwen3"

    @property
    def q_dim(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_key_value_heads * self.head_dim

    @property
    def qkv_dim(self) -> int:
        return self.q_dim + 2 * self.kv_dim

    def param_count(self) -> int:
        H, I, V = self.hidden_size, self.intermediate_size, self.vocab_size
        per_layer = H * self.qkv_dim + self.q_dim * H + 3 * H * I
        head = 0 if self.tie_word_embeddings else V * H
        return self.num_hidden_layers * per_layer + V * H + head

    def w8_bytes_per_forward(self) -> int:
        """Weight bytes one verify forward reads (W8: 1 B/weight + 4 B scale/bias per 64)."""
        H, I, V = self.hidden_size, self.intermediate_size, self.vocab_size
        per_layer = H * self.qkv_dim + self.q_dim * H + 3 * H * I
        n = self.num_hidden_layers * per_layer + V * H  # + lm_head (tied: embedding as linear)
        return n + n * 4 // 64


@dataclass
class DSparkConfig:
    """DSpark drafter config, qwen3 family (reference src/mlx_dspark/config.py:67-133)."""

    family: str = "qwen3"
    hidden_size: int = 4096
    vocab_size: int = 151936
    num_hidden_layers: int = 1
    intermediate_size: int = 12288
    rms_norm_eps: float = 1e-6
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int = 128
    attention_bias: bool = False
    rope_theta: float = 1_000_000.0
    block_size: int = 8
    mask_token_id: int = 4
    target_layer_ids: list[int] = field(default_factory=lambda: [1, 17, 33])
    num_target_layers: int = 36
    markov_rank: int = 256
    markov_head_type: str = "vanilla"
    enable_confidence_head: bool = False
    confidence_head_with_markov: bool = True
    final_logit_softcapping: float | None = None
    pad_token_id: int = 0
    mlp_activation: str = "silu"
    norm_style: str = "qwen"
    use_v_norm: bool = False
    attention_scaling: float | None = None
    shared_embeddings: bool = True  # embed_tokens / lm_head are the target's tensors

    @property
    def attn_head_dim(self) -> int:
        return self.head_dim

    @property
    def n_kv_heads(self) -> int:
        return self.num_key_value_heads

    @property
    def scaling(self) -> float:
        if self.attention_scaling is not None:
            return self.attention_scaling
        return self.attn_head_dim ** -0.5

    @classmethod
    def from_json(cls, path: str | Path) -> "DSparkConfig":
        """Parse a DeepSpec-format drafter config.json with the reference's refusals
        (src/mlx_dspark/config.py:87-185). Only the qwen3 family is built here."""
        with open(path) as f:
            c = json.load(f)
        mt = c.get("model_type", "")
        if "speculators_config" in c or "speculators_model_type" in c:
            raise ValueError(f"{path}: this checkpoint is in the vLLM 'speculators' format "
                             f"(speculators_config present), which cannot be loaded")
        if "block_size" not in c and any(k.startswith("dspark_") for k in c):
            raise ValueError(f"{path}: this looks like a full target model with an embedded "
                             f"DSpark drafter, not a standalone drafter checkpoint")
        if "qwen3" not in mt:
            raise ValueError(f"{path}: unsupported drafter family (model_type={mt!r}); "
                             f"this build supports qwen3 drafters")
        required = ("hidden_size", "vocab_size", "num_hidden_layers", "intermediate_size",
                    "num_attention_heads", "block_size", "mask_token_id", "target_layer_ids")
        missing = [k for k in required if k not in c]
        if missing:
            raise ValueError(f"{path}: config is missing required DeepSpec drafter fields {missing}")
        rp = c.get("rope_parameters") or {}
        return cls(
            family="qwen3",
            hidden_size=c["hidden_size"], vocab_size=c["vocab_size"],
            num_hidden_layers=c["num_hidden_layers"], intermediate_size=c["intermediate_size"],
            rms_norm_eps=c.get("rms_norm_eps", 1e-6),
            num_attention_heads=c["num_attention_heads"],
            num_key_value_heads=c.get("num_key_value_heads", 8),
            head_dim=c.get("head_dim", c["hidden_size"] // c["num_attention_heads"]),
            attention_bias=c.get("attention_bias", False),
            rope_theta=rp.get("rope_theta", c.get("rope_theta", 1_000_000.0)),
            block_size=c["block_size"], mask_token_id=c["mask_token_id"],
            target_layer_ids=list(c["target_layer_ids"]),
            num_target_layers=c.get("num_target_layers", 36),
            markov_rank=c.get("markov_rank", 256),
            markov_head_type=c.get("markov_head_type", "vanilla"),
            enable_confidence_head=c.get("enable_confidence_head", True),
            confidence_head_with_markov=c.get("confidence_head_with_markov", True),
            final_logit_softcapping=c.get("final_logit_softcapping", None),
            pad_token_id=c.get("pad_token_id") or 0,
            shared_embeddings=False,
        )


@dataclass
class DFlashConfig:
    """DFlash block-diffusion drafter (reference src/mlx_dspark/dflash_model.py:52-71)."""

    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    intermediate_size: int
    vocab_size: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    max_position_embeddings: int = 40960
    block_size: int = 16
    target_layer_ids: tuple = (1, 17, 33)
    num_target_layers: int = 36
    mask_token_id: int = 0
    layer_types: tuple = ()
    sliding_window: int | None = None
    final_logit_softcapping: float | None = None

    def __post_init__(self):
        if not self.layer_types:
            self.layer_types = ("full_attention",) * self.num_hidden_layers

    @property
    def scaling(self) -> float:
        """SDPA scale head_dim^-0.5 (dflash_model.py:89)."""
        return self.head_dim ** -0.5


# ----------------------------------------------------------------------------------------
# the BASELINE workloads
TINY = TargetConfig(hidden_size=512, num_hidden_layers=4, num_attention_heads=8,
                    num_key_value_heads=2, head_dim=64, intermediate_size=1536,
                    vocab_size=32768, tie_word_embeddings=True)
QWEN3_4B = TargetConfig(hidden_size=2560, num_hidden_layers=36, num_attention_heads=32,
                        num_key_value_heads=8, head_dim=128, intermediate_size=9728,
                        vocab_size=151936, tie_word_embeddings=True)
QWEN3_8B = TargetConfig(hidden_size=4096, num_hidden_layers=36, num_attention_heads=32,
                        num_key_value_heads=8, head_dim=128, intermediate_size=12288,
                        vocab_size=151936, tie_word_embeddings=False)
QWEN3_32B = TargetConfig(hidden_size=5120, num_hidden_layers=64, num_attention_heads=64,
                         num_key_value_heads=8, head_dim=128, intermediate_size=25600,
                         vocab_size=151936, tie_word_embeddings=False)

TARGETS = {"tiny": TINY, "qwen3-4b": QWEN3_4B, "qwen3-8b": QWEN3_8B, "qwen3-32b": QWEN3_32B}


def dspark_for(target: TargetConfig, *, block_size: int = 8, taps=None,
               num_hidden_layers: int = 1) -> DSparkConfig:
    """A 1-layer DSpark drafter sized to `target`, fusing three evenly spread taps."""
    L = target.num_hidden_layers
    if taps is None:
        taps = [1, L // 2 - 1, L - 3] if L >= 8 else [1, 2, 3][: max(1, L - 1)]
    return DSparkConfig(
        hidden_size=target.hidden_size, vocab_size=target.vocab_size,
        num_hidden_layers=num_hidden_layers, intermediate_size=target.intermediate_size,
        rms_norm_eps=target.rms_norm_eps, num_attention_heads=target.num_attention_heads,
        num_key_value_heads=target.num_key_value_heads, head_dim=target.head_dim,
        rope_theta=target.rope_theta, block_size=block_size, mask_token_id=4,
        target_layer_ids=list(taps), num_target_layers=L,
    )


def dflash_for(target: TargetConfig, *, block_size: int = 16, num_hidden_layers: int = 2,
               taps=None) -> DFlashConfig:
    L = target.num_hidden_layers
    if taps is None:
        taps = (1, L // 2 - 1, L - 3) if L >= 8 else (1, 2, 3)
    return DFlashConfig(
        hidden_size=target.hidden_size, num_hidden_layers=num_hidden_layers,
        num_attention_heads=target.num_attention_heads,
        num_key_value_heads=target.num_key_value_heads, head_dim=target.head_dim,
        intermediate_size=target.intermediate_size, vocab_size=target.vocab_size,
        rms_norm_eps=target.rms_norm_eps, rope_theta=target.rope_theta,
        block_size=block_size, target_layer_ids=tuple(taps), num_target_layers=L,
        mask_token_id=4,
    )


@dataclass(frozen=True)
class Workload:
    name: str
    target: str
    seed: int
    prompt_len: int
    new_tokens: int
    drafter: str = "dspark"  # "dspark" | "dflash"
    block_size: int = 8
    batch: int = 1
    kv_bits: int | None = None
    accept_p: float | None = None  # Bernoulli agree mask for the draft override
    temperature: float = 0.0
    top_p: float = 1.0
    top_k: int = 0
    tp: int = 1


WORKLOADS = {
    "C1": Workload("C1-tiny", "tiny", seed=0, prompt_len=128, new_tokens=256),
    "C2": Workload("C2-qwen3-8b", "qwen3-8b", seed=1, prompt_len=1024, new_tokens=512,
                   accept_p=0.7),
    "C3": Workload("C3-qwen3-4b-dflash", "qwen3-4b", seed=0, prompt_len=512, new_tokens=256,
                   drafter="dflash", block_size=16, temperature=1.0, top_p=0.95, top_k=50),
    "C4": Workload("C4-qwen3-8b-batch-kv8", "qwen3-8b", seed=1, prompt_len=2048,
                   new_tokens=512, batch=4, kv_bits=8),
    "C5": Workload("C5-qwen3-32b-tp", "qwen3-32b", seed=1, prompt_len=16384, new_tokens=512,
                   accept_p=0.7, tp=8),
}


def with_layers(cfg: TargetConfig, n: int) -> TargetConfig:
    """Same widths, fewer layers (depth-reduced parity cases)."""
    return replace(cfg, num_hidden_layers=n)
