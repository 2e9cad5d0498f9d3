"""Loaders with the reference's names (src/mlx_dspark/load.py:155-373).

A directory path loads a checkpoint from disk (``checkpoint.py``): an mlx-community 8-bit
Qwen3 target, a DeepSpec-format DSpark drafter, or a z-lab DFlash drafter. A preset name
(config.TARGETS) builds a seeded synthetic checkpoint of the BASELINE shapes (there is no
network here); ``seed`` selects its random-init weights. The return shapes follow the
reference: ``load_target -> (target, tokenizer)``, ``load_drafter -> (drafter, config)``,
``load_pair -> (target, tokenizer, drafter, config)``.
"""
from __future__ import annotations

import os

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


def _checkpoint_tokenizer(path: str, vocab_size: int):
    """The checkpoint's own tokenizer when its files are present (transformers, offline),
    else the id stand-in."""
    if any(os.path.exists(os.path.join(path, f)) for f in ("tokenizer.json", "tokenizer_config.json")):
        try:
            from transformers import AutoTokenizer
            return AutoTokenizer.from_pretrained(path, local_files_only=True)
        except Exception:  # noqa: BLE001 - a tokenizer is a convenience, never a failure
            pass
    return IdTokenizer(vocab_size)


def load_target(repo_or_path: str | TargetConfig = "tiny", *, require_tap: bool = False,
                kv_bits: int | None = None, seed: int = 0, device="cuda",
                gen_device: str | None = None, weights=None):
    """(Target, tokenizer) for a checkpoint directory, a synthetic preset name or a
    TargetConfig."""
    if isinstance(repo_or_path, str) and os.path.isdir(repo_or_path):
        from .checkpoint import load_target_checkpoint
        weights = load_target_checkpoint(repo_or_path) if weights is None else weights
        tok = _checkpoint_tokenizer(repo_or_path, weights.cfg.vocab_size)
        t = Target(weights, tok, kv_bits=kv_bits, device=device)
        return t, tok
    cfg = TARGETS[repo_or_path] if isinstance(repo_or_path, str) else repo_or_path
    if weights is None:
        weights = generate_target(cfg, seed, gen_device or _gen_device(device))
    t = Target(weights, IdTokenizer(cfg.vocab_size), kv_bits=kv_bits, device=device)
    return t, t.tokenizer


def load_drafter(target: Target, config: DSparkConfig | str | None = None, *, seed: int = 0,
                 device="cuda", gen_device: str | None = None, weights=None,
                 strict: bool = True):
    """(DSparkDrafter, config): from a DeepSpec-format checkpoint directory (strict name
    matching, load.py:155-215), or synthetic and sized to `target` (1 layer, block 8, three
    taps by default)."""
    if isinstance(config, str) and os.path.isdir(config):
        from .checkpoint import load_dspark_checkpoint
        weights = load_dspark_checkpoint(config, strict=strict) if weights is None else weights
        return DSparkDrafter(weights, target, device=device), weights.cfg
    cfg = config or dspark_for(target.cfg)
    if weights is None:
        weights = generate_dspark(cfg, seed, gen_device or _gen_device(device))
    return DSparkDrafter(weights, target, device=device), cfg


def load_dflash_drafter(target: Target, config: DFlashConfig | str | None = None, *,
                        seed: int = 0, device="cuda", gen_device: str | None = None,
                        weights=None):
    """(DFlashDrafter, config) bound to `target`: from a z-lab checkpoint directory
    (load.py:224-289), or synthetic (2 layers, block 16 by default)."""
    if isinstance(config, str) and os.path.isdir(config):
        from .checkpoint import load_dflash_checkpoint
        weights = load_dflash_checkpoint(config) if weights is None else weights
        return DFlashDrafter(weights, target, device=device), weights.cfg
    cfg = config or dflash_for(target.cfg)
    if weights is None:
        weights = generate_dflash(cfg, seed, gen_device or _gen_device(device))
    return DFlashDrafter(weights, target, device=device), cfg


def load_pair(model: str = "tiny", *, drafter: DSparkConfig | DFlashConfig | str | None = None,
              seed: int = 0, kv_bits: int | None = None, device="cuda"):
    """(target, tokenizer, drafter, config); drafter "dflash" (or a DFlashConfig) selects the
    block-diffusion drafter, a checkpoint directory its own kind (a config.json with
    ``dflash_config`` or DFlash architectures is DFlash), anything else the DSpark drafter."""
    target, tok = load_target(model, require_tap=True, kv_bits=kv_bits, seed=seed, device=device)
    if isinstance(drafter, str) and os.path.isdir(drafter):
        import json
        with open(os.path.join(drafter, "config.json")) as f:
            c = json.load(f)
        if "dflash_config" in c or any("DFlash" in a for a in c.get("architectures", [])):
            d, cfg = load_dflash_drafter(target, drafter, device=device)
        else:
            d, cfg = load_drafter(target, drafter, device=device)
        return target, tok, d, cfg
    if drafter == "dflash" or isinstance(drafter, DFlashConfig):
        d, cfg = load_dflash_drafter(target, None if drafter == "dflash" else drafter, seed=seed,
                                     device=device)
    else:
        d, cfg = load_drafter(target, None if drafter == "dspark" else drafter, seed=seed,
                              device=device)
    return target, tok, d, cfg
