"""Loaders with the reference's names (src/mlx_dspark/load.py:155-373).

There is no network here, so the named models are seeded synthetic checkpoints of the
BASELINE shapes (config.TARGETS); ``seed`` selects the random-init weights. The return
shapes follow the reference: ``load_target -> (target, tokenizer)``,
``load_drafter -> (drafter, config)``, ``load_pair -> (target, tokenizer, drafter, config)``.
"""
from __future__ import annotations

import torch

from .config import TARGETS, DFlashConfig, DSparkConfig, TargetConfig, dflash_for, dspark_for
from .model import DFlashDrafter, DSparkDrafter
from .target import Target
from .weights import generate_dflash, generate_dspark, generate_target


class IdTokenizer:
    """Stand-in tokenizer for synthetic checkpoints: ids map to code points for display."""

    eos_token_id = None
    chat_template = None

    def __init__(self, vocab_size: int):
        self.vocab_size = vocab_size

    def encode(self, text: str) -> list[int]:
        return [min(ord(c), self.vocab_size - 1) for c in text]

    def decode(self, ids) -> str:
        return "".join(chr(0x20 + (int(i) % 0x5f)) for i in ids)


def _gen_device(device) -> str:
    return "cuda" if torch.device(device).type == "cuda" else "cpu"


def load_target(repo_or_path: str | TargetConfig = "tiny", *, require_tap: bool = False,
                kv_bits: int | None = None, seed: int = 0, device="cuda",
                gen_device: str | None = None, weights=None):
    """(Target, tokenizer) for a synthetic preset name or a TargetConfig."""
    cfg = TARGETS[repo_or_path] if isinstance(repo_or_path, str) else repo_or_path
    if weights is None:
        weights = generate_target(cfg, seed, gen_device or _gen_device(device))
    t = Target(weights, IdTokenizer(cfg.vocab_size), kv_bits=kv_bits, device=device)
    return t, t.tokenizer


def load_drafter(target: Target, config: DSparkConfig | None = None, *, seed: int = 0,
                 device="cuda", gen_device: str | None = None, weights=None):
    """(DSparkDrafter, config) sized to `target` (1 layer, block 8, three taps by default)."""
    cfg = config or dspark_for(target.cfg)
    if weights is None:
        weights = generate_dspark(cfg, seed, gen_device or _gen_device(device))
    return DSparkDrafter(weights, target, device=device), cfg


def load_dflash_drafter(target: Target, config: DFlashConfig | None = None, *, seed: int = 0,
                        device="cuda", gen_device: str | None = None, weights=None):
    """(DFlashDrafter, config) bound to `target` (2 layers, block 16 by default;
    load.py:224-289 loads z-lab DFlash checkpoints the same way, bound to the target)."""
    cfg = config or dflash_for(target.cfg)
    if weights is None:
        weights = generate_dflash(cfg, seed, gen_device or _gen_device(device))
    return DFlashDrafter(weights, target, device=device), cfg


def load_pair(model: str = "tiny", *, drafter: DSparkConfig | DFlashConfig | str | None = None,
              seed: int = 0, kv_bits: int | None = None, device="cuda"):
    """(target, tokenizer, drafter, config); drafter "dflash" (or a DFlashConfig) selects the
    block-diffusion drafter, anything else the DSpark drafter."""
    target, tok = load_target(model, require_tap=True, kv_bits=kv_bits, seed=seed, device=device)
    if drafter == "dflash" or isinstance(drafter, DFlashConfig):
        d, cfg = load_dflash_drafter(target, None if drafter == "dflash" else drafter, seed=seed,
                                     device=device)
    else:
        d, cfg = load_drafter(target, None if drafter == "dspark" else drafter, seed=seed,
                              device=device)
    return target, tok, d, cfg
