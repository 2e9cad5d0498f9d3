"""mlx_dspark_b200 — the speculative verify step of mlx-dspark on B200 (sm_100a).

PyTorch on the host drives hand-written sm_100a kernels through the C ABI of
libdspark_b200.so (include/dspark_b200.h): W8A16 tcgen05 GEMMs, paged GQA attention,
fused greedy and rejection-sampling acceptance with in-place KV commit, and the DSpark and
DFlash drafters. The public names
follow the reference package (src/mlx_dspark/__init__.py:54-116).
"""
__version__ = "0.1.0"

from .config import DFlashConfig, DSparkConfig, TargetConfig, WORKLOADS, TARGETS
from .generate import (GenResult, StopStreaming, dflash_generate, encode_messages, encode_prompt,
                       greedy_generate, speculative_generate)
from .load import (DEFAULT_DRAFTER, DEFAULT_TARGET, DFLASH_PRESETS, PRESETS, REGISTRY,
                   apply_wired_limit, dflash_drafter_for, drafter_for, load_dflash,
                   load_dflash_pair, load_drafter, load_pair, load_target, resolve, resolve_mode)
from .lookup import NGramIndex, lookup_generate
from .batch_engine import SpecSlots, batch_generate_baseline, batch_spec_generate, serve_requests
from .calibrate import CapController, calibrate
from .engine import BatchEngine, Engine
from .prefix_cache import PrefixBlocks, PrefixCache
from .model import DFlashDrafter, DSparkDrafter, Sampling
from .target import Target

# the reference's class name for the DFlash drafter (dflash_model.py:150)
DFlashDraftModel = DFlashDrafter

# Reference exports not provided (src/mlx_dspark/__init__.py:54-116): run_server, the
# OpenAI-compatible HTTP layer, is out of scope (its scheduling layer is Engine / BatchEngine).
NOT_PROVIDED = {"run_server": "the HTTP server is out of scope; Engine/BatchEngine are its "
                              "scheduling layer"}

__all__ = [
    "DSparkConfig", "DFlashConfig", "DFlashDraftModel", "TargetConfig", "Target",
    "DSparkDrafter", "DFlashDrafter", "Sampling",
    "load_drafter", "load_dflash", "load_target", "load_pair", "load_dflash_pair",
    "drafter_for", "dflash_drafter_for",
    "speculative_generate", "dflash_generate", "lookup_generate", "greedy_generate",
    "calibrate", "CapController", "NGramIndex", "StopStreaming", "encode_messages",
    "encode_prompt", "GenResult", "Engine", "BatchEngine",
    "PRESETS", "DFLASH_PRESETS", "REGISTRY", "resolve", "resolve_mode", "apply_wired_limit",
    "DEFAULT_TARGET", "DEFAULT_DRAFTER",
    "SpecSlots", "batch_spec_generate", "batch_generate_baseline", "serve_requests",
    "PrefixCache", "PrefixBlocks", "WORKLOADS", "TARGETS",
]
