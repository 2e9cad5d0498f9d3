"""mlx_dspark_b200 — the speculative verify step of mlx-dspark on B200 (sm_100a).

PyTorch on the host drives hand-written sm_100a kernels through the C ABI of
libdspark_b200.so (include/dspark_b200.h): W8A16 tcgen05 GEMMs, paged GQA attention,
fused greedy and rejection-sampling acceptance with in-place KV commit, and the DSpark and
DFlash drafters. The public names
follow the reference package (src/mlx_dspark/__init__.py:54-116).
"""
__version__ = "0.1.0"

from .config import DFlashConfig, DSparkConfig, TargetConfig, WORKLOADS, TARGETS
from .generate import GenResult, dflash_generate, greedy_generate, speculative_generate
from .load import load_dflash_drafter, load_drafter, load_pair, load_target
from .lookup import NGramIndex, lookup_generate
from .batch_engine import SpecSlots, batch_generate_baseline, batch_spec_generate, serve_requests
from .prefix_cache import PrefixBlocks, PrefixCache
from .model import DFlashDrafter, DSparkDrafter, Sampling
from .target import Target

__all__ = [
    "DSparkConfig", "DFlashConfig", "TargetConfig", "Target", "DSparkDrafter", "DFlashDrafter",
    "Sampling", "load_drafter", "load_dflash_drafter", "load_target", "load_pair",
    "speculative_generate", "dflash_generate", "greedy_generate", "lookup_generate",
    "NGramIndex", "SpecSlots", "batch_spec_generate", "batch_generate_baseline",
    "serve_requests", "PrefixCache", "PrefixBlocks", "GenResult", "WORKLOADS", "TARGETS",
]
