"""ctypes binding of libdspark_b200.so (the C ABI declared in include/dspark_b200.h).

The library is required: there is no CPU or PyTorch fallback. Importing this module
without the built library raises with the build command to run.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_double, c_float, c_int, c_longlong, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libdspark_b200.so")

DSPARK_OK = 0
DSPARK_ERR_TIMEOUT = 4
ERR_NAMES = {1: "invalid argument", 2: "alignment", 3: "launch failed", 4: "device wait timed out",
             5: "unsupported", 6: "CUDA error", 7: "workspace",
             8: "fp16 operand out of range"}

EPI_STORE_BF16, EPI_RESIDUAL_BF16, EPI_SILU_MUL_F16, EPI_STORE_F32, EPI_PEER_F32 = 0, 1, 2, 3, 4


class DsparkError(RuntimeError):
    def __init__(self, what: str, code: int, msg: str):
        super().__init__(f"{what}: {ERR_NAMES.get(code, code)}: {msg}")
        self.code = code


class KvLayout(ctypes.Structure):
    """dspark_kv_layout"""
    _fields_ = [("pool", c_void_p), ("block_table", c_void_p), ("max_pages", c_int),
                ("page_size", c_int), ("num_kv_heads", c_int), ("head_dim", c_int),
                ("kv8", c_int), ("reserved", c_int), ("page_bytes", c_longlong)]


P = c_void_p
I = c_int
class GemmOpts(ctypes.Structure):
    """dspark_gemm_opts (include/dspark_b200.h)."""
    _fields_ = [("prefetch", c_void_p * 2), ("prefetch_bytes", c_size_t * 2),
                ("row_sumsq", c_void_p), ("norm_sumsq", c_void_p), ("norm_w", c_void_p),
                ("norm_tiles", c_int), ("norm_eps", c_float), ("norm_ld", c_int),
                ("reserved", c_int), ("copy_f16", c_void_p), ("copy_f16_ld", c_int),
                ("reserved2", c_int)]


class PeerAR(ctypes.Structure):
    """dspark_peer_ar (include/dspark_b200.h): the ranks' mapped buffers of one fused
    all-reduce."""
    _fields_ = [("recv", c_void_p * 8), ("flags", c_void_p * 8), ("world", c_int),
                ("rank", c_int), ("m_cap", c_int), ("n", c_int), ("epoch", c_int),
                ("reserved", c_int), ("epoch_dev", c_void_p)]


# name -> (restype, argtypes); mirrors include/dspark_b200.h
SIGNATURES = {
    "dspark_version": (I, []),
    "dspark_last_error": (c_char_p, []),
    "dspark_launch_count": (c_longlong, []),
    "dspark_w8a16_gemm_workspace_bytes": (c_size_t, [I, I, I]),
    "dspark_w8a16_gemm": (I, [P, I, P, P, I, I, I, P, I, P, I, I, P, c_size_t, P, P]),
    "dspark_w8a16_gemm_pf": (I, [P, I, P, P, I, I, I, P, I, P, I, I, P, c_size_t, P, c_size_t, P,
                                 c_size_t, P, P]),
    "dspark_peer_alloc": (I, [c_size_t, POINTER(c_void_p)]),
    "dspark_peer_free": (I, [P]),
    "dspark_ipc_handle": (I, [P, P]),
    "dspark_ipc_open": (I, [P, POINTER(c_void_p)]),
    "dspark_ipc_close": (I, [P]),
    "dspark_w8a16_gemm_peer": (I, [P, I, P, P, I, I, I, POINTER(PeerAR), P, c_size_t, P, P]),
    "dspark_peer_reduce_residual": (I, [P, I, I, POINTER(PeerAR), c_longlong, P, P]),
    "dspark_w8a16_gemm_wide": (I, [P, I, P, P, I, I, I, I, P, I, P, I, P, I, P, P]),
    "dspark_w8a16_gemm_wide_plan": (I, [I, I, I, P, P]),
    "dspark_w8a16_gemm_wide_bn": (I, [I]),
    "dspark_embed_w8": (I, [P, I, P, P, I, I, P, I, P]),
    "dspark_embed_w8_sumsq": (I, [P, I, P, P, I, I, P, I, P, P]),
    "dspark_embed_block_w8": (I, [P, I, I, I, P, P, I, I, P, I, P, P]),
    "dspark_rmsnorm": (I, [P, I, P, I, I, c_float, P, I, P, I, P]),
    "dspark_kv_page_bytes": (c_longlong, [I, I, I, I]),
    "dspark_qkv_rope_kv_write": (I, [P, I, I, I, I, I, I, P, P, c_float, P, P, P,
                                     POINTER(KvLayout), P]),
    "dspark_w8a16_gemm_qkv_rope": (I, [P, I, P, P, I, I, I, I, I, I, P, P, c_float, P, P, P,
                                       POINTER(KvLayout), POINTER(GemmOpts), P, c_size_t, P, P]),
    "dspark_w8a16_gemm_ex": (I, [P, I, P, P, I, I, I, P, I, P, I, I, POINTER(GemmOpts), P,
                                 c_size_t, P, P]),
    "dspark_gemm_opts_size": (c_size_t, []),
    "dspark_attention_workspace_bytes": (c_size_t, [I, I, I, I, I, I]),
    "dspark_attention": (I, [P, I, I, I, POINTER(KvLayout), P, I, c_float, P, I, I, P,
                             c_size_t, P, P]),
    "dspark_accept_workspace_bytes": (c_size_t, [I, I]),
    "dspark_accept_greedy": (I, [P, I, I, I, I, P, P, P, I, P, P, P, c_size_t, P]),
    "dspark_accept_greedy_noalloc": (I, [P, I, I, I, I, P, P, P, I, P, P, P]),
    "dspark_commit_lengths": (I, [P, I, I, P, P, P]),
    "dspark_draft_override": (I, [I, I, I, P, I, P, I, P, P, P, P, P]),
    "dspark_markov_workspace_bytes": (c_size_t, [I, I]),
    "dspark_markov_sample_block": (I, [P, I, I, I, I, I, I, P, P, P, P, P, P, P, P, c_size_t, P, P]),
    "dspark_bf16_to_f16": (I, [P, I, P, I, I, I, P, P]),
    "dspark_apply_penalties": (I, [P, c_longlong, I, I, I, P, P, c_double, c_double, P]),
    "dspark_penalty_counts_add": (I, [P, I, I, P, I, P]),
    "dspark_argmax_rows": (I, [P, c_longlong, I, I, P, I, P, I, P, I, P]),
    "dspark_logprobs": (I, [P, c_longlong, I, I, P, I, I, I, P, P, P, P]),
    "dspark_confidence": (I, [P, c_longlong, I, I, P, c_float, P, P, I, I, P, P, P, P, P, P, P]),
    "dspark_residual_add_f32": (I, [P, I, P, I, I, I, P]),
    "dspark_accept_greedy_sharded": (I, [P, P, I, I, I, P, P, I, P, P, P]),
    "dspark_sample_rows": (I, [P, c_longlong, I, I, I, c_float, I, c_double, I, P, I, I, P,
                               c_longlong, P, I, P, I, P]),
    "dspark_accept_sample_workspace_bytes": (c_size_t, [I, I]),
    "dspark_accept_sample": (I, [P, c_longlong, I, I, I, P, P, c_longlong, I, c_float, I,
                                 c_double, I, P, P, I, P, P, P, c_size_t, P]),
    "dspark_markov_probs_workspace_bytes": (c_size_t, [I, I]),
    "dspark_markov_sample_block_probs": (I, [P, I, I, I, I, I, I, P, P, P, P, P, P, P, c_float,
                                             c_double, I, P, P, c_longlong, P, c_size_t, P]),
}

_lib = None


def lib():
    """Load the library once and attach the signatures."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH.name} is not built; run `python -m mlx_dspark_b200.build` "
                           f"(there is no fallback path)")
    L = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(rc: int, what: str) -> None:
    if rc != DSPARK_OK:
        msg = lib().dspark_last_error()
        raise DsparkError(what, rc, msg.decode() if msg else "")


# kernel launches issued through call() (graph replays re-run them without Python), as
# counted by the library itself
LAUNCHES = {"n": 0}


def call(name: str, *args) -> None:
    L = lib()
    n0 = L.dspark_launch_count()
    check(getattr(L, name)(*args), name)
    LAUNCHES["n"] += L.dspark_launch_count() - n0


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
