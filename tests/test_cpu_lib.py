"""Host-side checks that need no GPU: the C-ABI library loads, exports and binds every
entry point of include/dspark_b200.h, rejects bad arguments with a message, and the host
packing / layout helpers are right."""
import os
import re

import pytest
import torch

from mlx_dspark_b200 import _lib
from mlx_dspark_b200.weights import pack, quantize_w8g64

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "dspark_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(dspark_[a-z0-9_]+)\s*\(", src)))


def test_library_loads_and_exports_every_declared_symbol():
    L = _lib.lib()
    names = declared_functions()
    assert len(names) >= 15
    for n in names:
        assert hasattr(L, n), n
    assert sorted(names) == sorted(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)
    assert L.dspark_version() >= 10000


def test_bad_arguments_return_codes_and_messages():
    L = _lib.lib()
    rc = L.dspark_w8a16_gemm(None, 0, None, None, 0, 128, 128, None, 0, None, 0, 0, None, 0,
                             None, None)
    assert rc == 1
    assert b"null pointer" in L.dspark_last_error()
    with pytest.raises(_lib.DsparkError) as e:
        _lib.call("dspark_rmsnorm", None, 0, None, 0, 0, 1e-6, None, 0, None, 0, None)
    assert "rmsnorm" in str(e.value)


def test_kv_page_bytes():
    L = _lib.lib()
    assert L.dspark_kv_page_bytes(64, 8, 128, 0) == 2 * 8 * 64 * 128 * 2
    assert L.dspark_kv_page_bytes(64, 8, 128, 1) == 2 * 8 * 64 * 128 + 2 * 8 * 64 * 2 * 4


def test_pack_layout_and_interleave():
    g = quantize_w8g64(torch.randn(128, 256) * 0.02)
    u = quantize_w8g64(torch.randn(128, 256) * 0.02)
    p = pack(g, u, interleave64=True, device="cpu")
    assert p.N == 256 and p.K == 256 and p.sb.shape == (4, 256)
    # packed tile t = [gate rows 64t..64t+63; up rows 64t..64t+63]
    assert torch.equal(p.q[0:64], g.q[0:64]) and torch.equal(p.q[64:128], u.q[0:64])
    assert torch.equal(p.q[128:192], g.q[64:128]) and torch.equal(p.q[192:256], u.q[64:128])
    # sb[g, n] = fp16 scale (low) | fp16 bias (high)
    s = (p.sb[1, 65] & 0xFFFF).to(torch.int16).view(torch.float16).float()
    b = (p.sb[1, 65] >> 16).to(torch.int16).view(torch.float16).float()
    assert s == u.scales[1, 1].float() and b == u.biases[1, 1].float()


def test_pack_rounds_tiny_scales_and_refuses_fp16_overflow():
    """Scales and biases below fp16's normal range (groups of nearly constant weights; MLX floors
    a scale at 1e-7) pack as fp16 subnormals within 2^-25; values past 65504 are refused."""
    g = torch.Generator().manual_seed(5)
    w = torch.randn(256, 256, generator=g) * 0.02
    w[0, :64] = 0.0                                      # constant group: scale floor 1e-7
    w[1, :64] = 0.01 + torch.arange(64) * 1e-7           # range 6.3e-6: scale ~2.5e-8
    qt = quantize_w8g64(w)
    # a synthetic scale distribution down to 2^-30, and biases of either sign below 2^-17
    qt.scales[2:, 0] = (2.0 ** -torch.linspace(4, 30, 254)).to(torch.bfloat16)
    qt.biases[2:, 1] = (-(2.0 ** -torch.linspace(17, 28, 254))).to(torch.bfloat16)
    assert float(qt.scales.float().abs().min()) < 2.0 ** -17
    pl = pack(qt, device="cpu")
    sb = pl.sb.t().contiguous()                          # [N, G] int32 of fp16 pairs
    s16 = (sb & 0xFFFF).to(torch.int16).view(torch.float16).float()
    b16 = (sb >> 16).to(torch.int16).view(torch.float16).float()
    assert (s16 - qt.scales.float()).abs().max() <= 2.0 ** -25
    assert (b16 - qt.biases.float()).abs().max() <= 2.0 ** -25
    # and exactly where fp16 holds the value
    big = qt.scales.float().abs() >= 2.0 ** -17
    assert torch.equal(s16[big], qt.scales.float()[big])
    qt.scales[0, 0] = torch.tensor(1e5).to(torch.bfloat16)
    with pytest.raises(ValueError):
        pack(qt, device="cpu")


def test_checkpoint_keeps_fp16_scales():
    """An fp16 source model's 8-bit checkpoint: scales and biases stay fp16 (packed exactly),
    norm weights are rounded to bf16."""
    from mlx_dspark_b200.checkpoint import _as_bf16, _scale_dtype
    s = (torch.rand(4, 4) * 1e-3).to(torch.float16)
    assert _scale_dtype(s, "s").dtype == torch.float16
    assert _scale_dtype(s.float(), "s").dtype in (torch.bfloat16, torch.float16)
    with pytest.raises(ValueError):
        _scale_dtype(torch.tensor([1.0 + 2.0 ** -20]), "s")
    assert _as_bf16(torch.ones(4, dtype=torch.float16) * 1.001, "n").dtype == torch.bfloat16


def test_gemm_opts_struct_matches_the_c_layout():
    import ctypes
    from mlx_dspark_b200 import _lib
    assert ctypes.sizeof(_lib.GemmOpts) == _lib.lib().dspark_gemm_opts_size()


# The public names of the reference package (src/mlx_dspark/__init__.py:89-116): each one is
# exported here or listed, with the reason, in mlx_dspark_b200.NOT_PROVIDED.
REFERENCE_ALL = [
    "DSparkConfig", "DFlashConfig", "DFlashDraftModel", "Target", "load_drafter", "load_dflash",
    "load_target", "load_pair", "load_dflash_pair", "speculative_generate", "dflash_generate",
    "lookup_generate", "greedy_generate", "calibrate", "CapController", "NGramIndex",
    "StopStreaming", "encode_messages", "encode_prompt", "GenResult", "Engine", "run_server",
    "PRESETS", "DFLASH_PRESETS", "REGISTRY", "resolve", "resolve_mode", "apply_wired_limit",
    "DEFAULT_TARGET", "DEFAULT_DRAFTER",
]


def test_reference_public_names_exported_or_excused():
    import mlx_dspark_b200 as pkg
    missing = [n for n in REFERENCE_ALL
               if n not in pkg.NOT_PROVIDED and not (n in pkg.__all__ and hasattr(pkg, n))]
    assert not missing, missing
    for n, why in pkg.NOT_PROVIDED.items():
        assert n in REFERENCE_ALL and why


def test_loader_signatures_follow_the_reference():
    import inspect

    from mlx_dspark_b200 import load
    sig = inspect.signature(load.load_drafter)
    first = list(sig.parameters)[0]
    assert first == "repo_or_path"
    for kw, default in (("quantize", True), ("bits", 4), ("group_size", 64), ("strict", True)):
        p = sig.parameters[kw]
        assert p.kind is p.KEYWORD_ONLY and p.default == default, kw
    assert list(inspect.signature(load.load_dflash).parameters)[0] == "repo_or_path"
    for fn in (load.load_pair, load.load_dflash_pair):
        assert "drafter" in inspect.signature(fn).parameters
    from mlx_dspark_b200.generate import speculative_generate
    assert inspect.signature(speculative_generate).parameters["lookup_drafts"].default is True
    with pytest.raises(ValueError):
        load.load_drafter("tiny", group_size=32, device="cpu")


def test_resolve_rules():
    from mlx_dspark_b200 import load
    assert load.resolve("mlx-community/Qwen3-8B-4bit") == (
        "mlx-community/Qwen3-8B-4bit", "deepseek-ai/dspark_qwen3_8b_block7")
    assert load.resolve("some/unknown-model", mode="lookup") == ("some/unknown-model", None)
    assert load.resolve("qwen3", mode="dflash")[1] == "z-lab/Qwen3-4B-DFlash-b16"
    assert load.resolve("x/y", drafter="my/drafter") == ("x/y", "my/drafter")
    with pytest.raises(ValueError):
        load.resolve("some/unknown-model")
    assert load.resolve_mode("mlx-community/Qwen3-4B-8bit")[0] == "dspark"
    assert load.resolve_mode("some/unknown-model") == ("lookup", "some/unknown-model", None)
    with pytest.raises(ValueError):
        load.load_target("not/a-cached-repo", device="cpu")
