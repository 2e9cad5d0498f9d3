"""Loaders with the reference's names and call shapes (src/mlx_dspark/load.py:1-373).

``load_target(repo_or_path)`` -> (target, tokenizer); ``load_drafter(repo_or_path, *, quantize,
bits, group_size, strict)`` -> (drafter, config); ``load_dflash(repo_or_path, ...)`` ->
(drafter, config); ``load_pair`` / ``load_dflash_pair`` -> (target, tokenizer, drafter, config).
The registry (``PRESETS``, ``DFLASH_PRESETS``, ``REGISTRY``) and ``resolve`` / ``resolve_mode``
keep the reference's tables and rules.

What a name resolves to:
  * a directory: a checkpoint on disk (``checkpoint.py``): an mlx-community 8-bit Qwen3 target,
    a DeepSpec-format DSpark drafter, or a z-lab DFlash drafter;
  * a synthetic preset (``config.TARGETS``: "tiny", "qwen3-4b", "qwen3-8b", "qwen3-32b"): seeded
    random-init weights of that architecture (``seed`` selects them);
  * any other name (a Hugging Face repo id): the local Hugging Face cache only. There is no
    network here, so a repo that is not cached raises ValueError with the reason.

A drafter comes back unbound, like the reference's (whose DSpark drafter owns its embedding and
whose DFlash drafter is bound by ``bind(target.model)``): the generate loops bind it to their
target on first use (``drafter.bind(target)``), which attaches the target's embedding and head
where the drafter shares them. On the device every drafter linear runs as W8 group-64, the one
format the GEMM kernels take; ``bits`` 4 (the reference's default) and 8 both load as W8, which
changes acceptance only, never output (the target verifies every token).
"""
from __future__ import annotations

import os

import torch

from .config import TARGETS, DFlashConfig, DSparkConfig, TargetConfig, dflash_for, dspark_for
from .model import DFlashDrafter, DSparkDrafter
from .target import Target
from .weights import generate_dflash, generate_dspark, generate_target

# The reference's tables (load.py:17-60), kept as data. The default is the reference's qwen3
# preset: its gemma4 default needs the Gemma-4 family, which this build refuses.
PRESETS = {
    "gemma4": {"target": "mlx-community/gemma-4-12B-it-8bit",
               "drafter": "deepseek-ai/dspark_gemma4_12b_block7"},
    "qwen3": {"target": "mlx-community/Qwen3-4B-8bit",
              "drafter": "deepseek-ai/dspark_qwen3_4b_block7"},
}
DEFAULT_TARGET = PRESETS["qwen3"]["target"]
DEFAULT_DRAFTER = PRESETS["qwen3"]["drafter"]
DFLASH_PRESETS = {
    "gemma4": {"target": "mlx-community/gemma-4-12B-it-8bit",
               "drafter": "z-lab/gemma4-12B-it-DFlash"},
    "qwen3": {"target": "mlx-community/Qwen3-4B-8bit", "drafter": "z-lab/Qwen3-4B-DFlash-b16"},
}
REGISTRY = [
    {"id": "qwen3-4b", "target": "mlx-community/Qwen3-4B-8bit",
     "dspark": "deepseek-ai/dspark_qwen3_4b_block7", "dflash": "z-lab/Qwen3-4B-DFlash-b16",
     "ram": "~8 GB"},
    {"id": "qwen3-8b", "target": "mlx-community/Qwen3-8B-8bit",
     "dspark": "deepseek-ai/dspark_qwen3_8b_block7", "dflash": "z-lab/Qwen3-8B-DFlash-b16",
     "ram": "~11 GB"},
    {"id": "gemma-4-12b", "target": "mlx-community/gemma-4-12B-it-8bit",
     "dspark": "deepseek-ai/dspark_gemma4_12b_block7", "dflash": "z-lab/gemma4-12B-it-DFlash",
     "ram": "~15 GB"},
]
_FAMILY_ALIASES = {"qwen3": "mlx-community/Qwen3-4B-8bit",
                   "gemma4": "mlx-community/gemma-4-12B-it-8bit"}


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


# ---------------------------------------------------------------------------------- registry
def _registry_entry(target: str) -> dict | None:
    """The REGISTRY entry whose id occurs in the target's repo or directory name, matched
    without regard to quantization or dashes, longest id first (load.py:66-76)."""
    name = os.path.basename(str(target).rstrip("/")).lower()
    flat = name.replace("-", "")
    for entry in sorted(REGISTRY, key=lambda e: len(e["id"]), reverse=True):
        if entry["id"] in name or entry["id"].replace("-", "") in flat:
            return entry
    return None


def resolve(model: str | None = None, *, mode: str = "dspark", drafter: str | None = None,
            family: str | None = None, target: str | None = None) -> tuple[str, str | None]:
    """(target_repo, drafter_repo) for a target and a mode (load.py:79-110): baseline and
    lookup need no drafter; an explicit drafter wins; else the registry's drafter for a known
    target; else ValueError. ``family`` / ``target`` are the deprecated aliases of ``model``."""
    tgt = model or target or family
    tgt = _FAMILY_ALIASES.get(tgt, tgt) if tgt else DEFAULT_TARGET
    if mode in ("baseline", "lookup"):
        return tgt, None
    if drafter:
        return tgt, drafter
    entry = _registry_entry(tgt)
    if entry is not None and entry.get(mode):
        return tgt, entry[mode]
    raise ValueError(f"no built-in {mode} drafter is registered for target {tgt!r}: pass "
                     f"drafter=<repo or path>, use a registered target, or use mode 'auto' or "
                     f"'lookup' (no drafter needed)")


def resolve_mode(model: str | None = None, *, mode: str = "auto", drafter: str | None = None,
                 family: str | None = None, target: str | None = None
                 ) -> tuple[str, str, str | None]:
    """``resolve`` plus mode "auto" (load.py:113-135): the registry's DSpark drafter, else its
    DFlash drafter, else drafter-free lookup. Returns (mode, target_repo, drafter_repo)."""
    if mode != "auto":
        tgt, drf = resolve(model, mode=mode, drafter=drafter, family=family, target=target)
        return mode, tgt, drf
    if drafter:
        tgt, drf = resolve(model, mode="dspark", drafter=drafter, family=family, target=target)
        return "dspark", tgt, drf
    tgt, _ = resolve(model, mode="baseline", family=family, target=target)
    entry = _registry_entry(tgt)
    if entry is not None:
        for m in ("dspark", "dflash"):
            if entry.get(m):
                return m, tgt, entry[m]
    return "lookup", tgt, None


def apply_wired_limit() -> None:
    """The reference wires MLX's working set so weights stay resident (load.py:138-145).
    Device memory here is never paged out, so there is nothing to do."""
    return None


def _resolve_path(repo_or_path: str) -> str:
    """A checkpoint directory for a local path or a cached Hugging Face repo id."""
    if os.path.isdir(repo_or_path):
        return repo_or_path
    try:
        from huggingface_hub import snapshot_download
        return snapshot_download(repo_or_path, local_files_only=True)
    except Exception as e:  # noqa: BLE001 - turned into the loader's own error
        raise ValueError(f"{repo_or_path}: not a directory, a synthetic preset "
                         f"({', '.join(TARGETS)}), or a Hugging Face repo in the local cache "
                         f"(there is no network to download it): {e.__class__.__name__}") from e


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


def _check_quant(quantize: bool, bits: int, group_size: int) -> None:
    if bits not in (4, 8):
        raise ValueError(f"bits must be 4 or 8 (got {bits}); drafters run as W8 group-64")
    if group_size != 64:
        raise ValueError(f"group_size must be 64 (got {group_size}): the W8 kernels take "
                         f"group-64 scales only")


# ---------------------------------------------------------------------------------- loaders
def load_target(repo_or_path: str | TargetConfig = DEFAULT_TARGET, *, require_tap: bool = False,
                kv_bits: int | None = None, kv_group_size: int = 64, seed: int = 0,
                device="cuda", gen_device: str | None = None, weights=None):
    """(Target, tokenizer) for a checkpoint directory, a cached repo id, a synthetic preset
    name or a TargetConfig (load.py:292-335). ``kv_bits`` 8 selects the 8-bit KV cache with
    group ``kv_group_size`` (64, the only size built)."""
    if kv_group_size != 64:
        raise ValueError("kv_group_size must be 64")
    if isinstance(repo_or_path, TargetConfig) or repo_or_path in TARGETS:
        cfg = TARGETS[repo_or_path] if isinstance(repo_or_path, str) else repo_or_path
        if weights is None:
            weights = generate_target(cfg, seed, gen_device or _gen_device(device))
        t = Target(weights, IdTokenizer(cfg.vocab_size), kv_bits=kv_bits, device=device)
        return t, t.tokenizer
    path = repo_or_path if weights is not None else _resolve_path(repo_or_path)
    from .checkpoint import load_target_checkpoint
    weights = load_target_checkpoint(path) if weights is None else weights
    tok = _checkpoint_tokenizer(path, weights.cfg.vocab_size)
    t = Target(weights, tok, kv_bits=kv_bits, device=device)
    if require_tap:
        t.verify_tap()
    return t, tok


def load_drafter(repo_or_path: str | DSparkConfig = DEFAULT_DRAFTER, *, quantize: bool = True,
                 bits: int = 4, group_size: int = 64, strict: bool = True, seed: int = 0,
                 device="cuda", gen_device: str | None = None, weights=None):
    """(DSparkDrafter, config), unbound (load.py:155-215): a DeepSpec-format checkpoint with
    strict tensor-name matching (``strict=False`` loads the intersection with a warning), or a
    synthetic drafter for a preset target name / a DSparkConfig. The generate loops bind it to
    their target."""
    _check_quant(quantize, bits, group_size)
    if isinstance(repo_or_path, DSparkConfig) or repo_or_path in TARGETS:
        cfg = repo_or_path if isinstance(repo_or_path, DSparkConfig) else dspark_for(TARGETS[repo_or_path])
        if weights is None:
            weights = generate_dspark(cfg, seed, gen_device or _gen_device(device))
        return DSparkDrafter(weights, None, device=device), cfg
    from .checkpoint import load_dspark_checkpoint
    weights = load_dspark_checkpoint(_resolve_path(repo_or_path), strict=strict) \
        if weights is None else weights
    return DSparkDrafter(weights, None, device=device), weights.cfg


def load_dflash(repo_or_path: str | DFlashConfig, *, quantize: bool = True, bits: int = 4,
                group_size: int = 64, seed: int = 0, device="cuda",
                gen_device: str | None = None, weights=None):
    """(DFlashDrafter, config), unbound (load.py:224-289): a z-lab checkpoint (exact tensor
    names; the reference's refusals of Markov-head hybrids and unsupported layers), or a
    synthetic drafter for a preset target name / a DFlashConfig. ``drafter.bind(target)``
    attaches the target's embedding and head (dflash_generate does it)."""
    _check_quant(quantize, bits, group_size)
    if isinstance(repo_or_path, DFlashConfig) or repo_or_path in TARGETS:
        cfg = repo_or_path if isinstance(repo_or_path, DFlashConfig) else dflash_for(TARGETS[repo_or_path])
        if weights is None:
            weights = generate_dflash(cfg, seed, gen_device or _gen_device(device))
        return DFlashDrafter(weights, None, device=device), cfg
    from .checkpoint import load_dflash_checkpoint
    weights = load_dflash_checkpoint(_resolve_path(repo_or_path)) if weights is None else weights
    return DFlashDrafter(weights, None, device=device), weights.cfg


def drafter_for(target: Target, config: DSparkConfig | None = None, *, seed: int = 0,
                device="cuda", gen_device: str | None = None, weights=None):
    """(DSparkDrafter, config) sized to `target` and bound to it: synthetic weights from
    `config` (default: 1 layer, block 8, three taps) or the given DSparkWeights."""
    cfg = weights.cfg if weights is not None else (config or dspark_for(target.cfg))
    if weights is None:
        weights = generate_dspark(cfg, seed, gen_device or _gen_device(device))
    return DSparkDrafter(weights, target, device=device), cfg


def dflash_drafter_for(target: Target, config: DFlashConfig | None = None, *, seed: int = 0,
                       device="cuda", gen_device: str | None = None, weights=None):
    """(DFlashDrafter, config) sized to `target` and bound to it (2 layers, block 16 by
    default)."""
    cfg = weights.cfg if weights is not None else (config or dflash_for(target.cfg))
    if weights is None:
        weights = generate_dflash(cfg, seed, gen_device or _gen_device(device))
    return DFlashDrafter(weights, target, device=device), cfg


def _is_dflash_dir(path: str) -> bool:
    import json
    with open(os.path.join(path, "config.json")) as f:
        c = json.load(f)
    return "dflash_config" in c or any("DFlash" in a for a in c.get("architectures", []))


def load_pair(model: str = DEFAULT_TARGET, *, drafter: str | DSparkConfig | DFlashConfig | None = None,
              seed: int = 0, kv_bits: int | None = None, device="cuda"):
    """(target, tokenizer, DSpark drafter, config) (load.py:338-347). ``model`` is a target
    directory, repo id or synthetic preset; the drafter resolves from the registry unless
    given. For a synthetic preset the drafter is synthetic too ("dflash" or a DFlashConfig
    selects the block-diffusion drafter); a drafter directory loads as its own kind."""
    if model in TARGETS:
        target, tok = load_target(model, require_tap=True, kv_bits=kv_bits, seed=seed, device=device)
        if isinstance(drafter, str) and os.path.isdir(drafter):
            d, cfg = (load_dflash if _is_dflash_dir(drafter) else load_drafter)(drafter, device=device)
        elif drafter == "dflash" or isinstance(drafter, DFlashConfig):
            d, cfg = dflash_drafter_for(target, None if drafter == "dflash" else drafter,
                                        seed=seed, device=device)
        else:
            d, cfg = drafter_for(target, None if drafter in (None, "dspark") else drafter,
                                 seed=seed, device=device)
        return target, tok, d.bind(target), cfg
    target_repo, drafter_repo = resolve(model, mode="dspark", drafter=drafter)
    target, tok = load_target(target_repo, require_tap=True, kv_bits=kv_bits, device=device)
    d, cfg = load_drafter(drafter_repo, device=device)
    return target, tok, d.bind(target), cfg


def load_dflash_pair(model: str = DEFAULT_TARGET, *, drafter: str | DFlashConfig | None = None,
                     seed: int = 0, kv_bits: int | None = None, device="cuda"):
    """(target, tokenizer, DFlash drafter bound to the target, config) (load.py:366-373)."""
    if model in TARGETS:
        return load_pair(model, drafter=drafter if drafter is not None else "dflash", seed=seed,
                         kv_bits=kv_bits, device=device)
    target_repo, drafter_repo = resolve(model, mode="dflash", drafter=drafter)
    target, tok = load_target(target_repo, require_tap=True, kv_bits=kv_bits, device=device)
    d, cfg = load_dflash(drafter_repo, device=device)
    return target, tok, d.bind(target), cfg


__all__ = ["PRESETS", "DFLASH_PRESETS", "REGISTRY", "DEFAULT_TARGET", "DEFAULT_DRAFTER",
           "resolve", "resolve_mode", "apply_wired_limit", "load_target", "load_drafter",
           "load_dflash", "load_pair", "load_dflash_pair", "drafter_for", "dflash_drafter_for",
           "IdTokenizer"]
