"""Cost curves and the live speculative-cap controller (``--max-draft auto``), on the B200 path.

Drop-in for src/mlx_dspark/calibrate.py: the same measurements (verify ms by width, drafter ms
by cap, the batched verify grid), the same controller contract (``cap``, ``update``,
``cap_for``, ``info``) and the same disk cache (JSON, keyed by device, library versions, mode,
model basenames, context length and KV bits). Timings are CUDA-event device times of the
sm_100a forwards (``Target.forward``, ``draft_dev``) over a context of CTX_LEN zero-filled KV
positions; content does not change them.

What differs on B200 is the measured curve, not the method. The reference's verify cost is
convex with a knee where MLX's quantized matmul leaves its few-row path (calibrate.py:1-11).
Here every verify width up to 64 rows streams the same W8 weights once through the small-M
GEMM, so the curve is flat up to the bandwidth knee, and the rate-maximising cap is the full
block whenever the acceptance estimate is not tiny.

The cap only decides how many drafted tokens are verified per round: the target verifies every
emitted token, so output is the same for any cap sequence (lossless).
"""
from __future__ import annotations

import json
import os

import torch

from . import ops
from .kvcache import CacheState

CACHE_DIR = os.path.expanduser("~/.cache/mlx_dspark_b200")
CACHE_FILE = "calibration.json"
SCHEMA = 1
CTX_LEN = 512   # the curve's shape barely depends on the context (split-KV attention)
TOKEN_ID = 7    # any id: timings do not depend on content


def _device_ms(fn, iters: int = 8, warmup: int = 3) -> float:
    """Mean device time of fn() in ms (CUDA events on the current stream, after warm-up)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def _context_state(pool_owner, ctx_len: int, rows: int = 1) -> CacheState:
    """A state of `rows` rows holding ctx_len positions (pages zero-filled) plus room for a
    block: verify and draft forwards over it write past ctx_len and never advance it."""
    tokens = ctx_len + 128
    st = CacheState(pool_owner.new_pool(tokens, rows), rows, tokens, pool_owner.device)
    for b in range(rows):
        st.ensure(b, tokens)
        st.set_len(b, ctx_len)
    return st


# ------------------------------------------------------------------------------ measurement
def measure_verify_curve(target, tap: list[int], widths: list[int],
                         ctx_len: int = CTX_LEN) -> dict[int, float]:
    """ms per verify forward (logits + hidden-state tap) at each width (calibrate.py:58-75)."""
    st = _context_state(target, ctx_len)
    try:
        curve = {}
        for T in sorted(int(w) for w in widths):
            buf = target.buffers(1, T, len(tap))
            buf.ids.fill_(TOKEN_ID)
            splits = target.attn_splits(1, st.max_pages)
            curve[T] = _device_ms(lambda: target.forward(buf, st, tap, splits=splits))
        target.scratch.check_status()
        return curve
    finally:
        st.release()


def measure_batch_verify_grid(target, tap: list[int], batch_widths: list[int],
                              widths: list[int], ctx_len: int = CTX_LEN
                              ) -> dict[int, dict[int, float]]:
    """verify ms [B][width] of the batched forward, every row at ctx_len (calibrate.py:103-139).
    The small-M GEMM's cost follows B x width rows, so the best cap can shrink as B grows."""
    grid = {}
    for B in sorted({int(b) for b in batch_widths if int(b) > 1}):
        st = _context_state(target, ctx_len, rows=B)
        try:
            row = {}
            for T in sorted(int(w) for w in widths):
                if B * T > 64:  # past the verify GEMM's rows
                    continue
                buf = target.buffers(B, T, len(tap))
                buf.ids.fill_(TOKEN_ID)
                splits = target.attn_splits(B, st.max_pages)
                row[T] = _device_ms(lambda: target.forward(buf, st, tap, splits=splits))
            grid[B] = row
        finally:
            st.release()
    target.scratch.check_status()
    return grid


def measure_drafter_curve(drafter, caps: list[int], ctx_len: int = CTX_LEN) -> dict[int, float]:
    """ms per draft round at each cap (calibrate.py:78-100 for DSpark; a DFlash round costs
    about the same at every cap, calibrate.py:142-154): the backbone over the whole block, the
    head over the first `cap` rows, then the Markov head or the argmax."""
    st = _context_state(drafter, ctx_len)
    dev = drafter.device
    try:
        k = drafter.block_size
        pending = torch.full((1,), TOKEN_ID, dtype=torch.int32, device=dev)
        curve = {}
        for cap in sorted(int(c) for c in caps):
            buf = drafter.buffers(1, k, cap + 1)
            draft = torch.zeros(1, cap, dtype=torch.int32, device=dev)
            vids = torch.zeros(cap + 1, dtype=torch.int32, device=dev)
            splits = drafter.target.attn_splits(1, st.max_pages)
            curve[cap] = _device_ms(
                lambda: drafter.draft_dev(pending, 1, cap, st, buf, draft, vids, splits))
        drafter.scratch.check_status()
        return curve
    finally:
        st.release()


# ------------------------------------------------------------------------------ curve reading
def knee_width(verify_ms: dict[int, float]) -> int:
    """The smallest width whose marginal verify cost is clearly (1.8x) above the cheapest
    marginal cost seen below it, or the top width when there is none (calibrate.py:157-174)."""
    ws = sorted(verify_ms)
    if len(ws) < 3:
        return ws[-1] if ws else 0
    cheapest = verify_ms[ws[1]] - verify_ms[ws[0]]
    for lo, hi in zip(ws[1:], ws[2:]):
        step = verify_ms[hi] - verify_ms[lo]
        if step > 1.8 * max(cheapest, 1e-6):
            return hi
        cheapest = min(cheapest, step)
    return ws[-1]


def drafter_recommendation(verify_ms: dict[int, float], dflash_block: int = 16) -> dict:
    """DSpark vs DFlash from the verify curve: a knee at or past the DFlash block width keeps
    DFlash's full-block verify cheap (calibrate.py:177-185)."""
    knee = knee_width(verify_ms)
    viable = knee >= dflash_block
    return {"knee_width": knee, "dflash_full_block_viable": viable,
            "recommend": "dflash-on-structured" if viable else "dspark"}


def _interp(curve: dict[int, float], x: int) -> float:
    """Piecewise-linear over the measured points; the last segment's slope past the end."""
    xs = sorted(curve)
    if x in curve:
        return curve[x]
    if x <= xs[0]:
        return curve[xs[0]]
    if x >= xs[-1]:
        if len(xs) == 1:
            return curve[xs[-1]]
        a, b = xs[-2], xs[-1]
        return curve[b] + (curve[b] - curve[a]) / (b - a) * (x - b)
    hi = next(v for v in xs if v > x)
    lo = max(v for v in xs if v < x)
    return curve[lo] + (x - lo) / (hi - lo) * (curve[hi] - curve[lo])


# ------------------------------------------------------------------------------ controller
class CapController:
    """Picks the cap that maximises expected committed tokens per ms of round time
    (calibrate.py:211-297).

    p is an EWMA of the per-position conditional acceptance: a round that accepted n of c
    drafts contributes n successes, plus one failure unless all c were accepted (a fully
    accepted block says nothing about position c + 1). The expected committed tokens at cap C
    are 1 + p + p^2 + ... + p^C; the round time is drafter(C) + verify(C + 1). Every
    `repick_every` rounds the cap moves to the best rate if that beats the current cap's by the
    hysteresis factor. Not thread-safe; one generation loop drives it."""

    def __init__(self, verify_ms: dict[int, float], drafter_ms: dict[int, float] | float,
                 max_cap: int, *, init_cap: int = 2, prior_p: float = 0.65,
                 alpha: float = 0.02, hysteresis: float = 1.03, repick_every: int = 4,
                 verify_grid: dict[int, dict[int, float]] | None = None):
        self.verify_ms = {int(w): float(v) for w, v in verify_ms.items()}
        self.drafter_ms = ({int(c): float(v) for c, v in drafter_ms.items()}
                           if isinstance(drafter_ms, dict) else float(drafter_ms))
        self.max_cap = max(1, int(max_cap))
        self.cap = min(max(1, int(init_cap)), self.max_cap)
        self.p = float(prior_p)
        self.alpha = float(alpha)
        self.hysteresis = float(hysteresis)
        self.repick_every = max(1, int(repick_every))
        self.rounds = 0
        self.verify_grid = ({int(B): {int(w): float(v) for w, v in row.items()}
                             for B, row in verify_grid.items()} if verify_grid else None)

    def _draft_cost(self, cap: int) -> float:
        if isinstance(self.drafter_ms, dict):
            return _interp(self.drafter_ms, cap)
        return self.drafter_ms

    def expected_committed(self, cap: int) -> float:
        """The bonus (or replacement) token plus the expected accepted prefix."""
        total, term = 1.0, 1.0
        for _ in range(cap):
            term *= self.p
            total += term
        return total

    def _rate(self, cap: int, verify: dict[int, float]) -> float:
        t = self._draft_cost(cap) + _interp(verify, cap + 1)
        return self.expected_committed(cap) / max(t, 1e-6)

    def rate(self, cap: int) -> float:
        """Expected committed tokens per ms at this cap (batch 1)."""
        return self._rate(cap, self.verify_ms)

    def update(self, accepted_n: int, cap_used: int) -> None:
        for _ in range(int(accepted_n)):
            self.p += self.alpha * (1.0 - self.p)
        if accepted_n < cap_used:
            self.p -= self.alpha * self.p
        self.rounds += 1
        if self.rounds % self.repick_every == 0:
            self._repick()

    def _repick(self) -> None:
        best = max(range(1, self.max_cap + 1), key=self.rate)
        if best != self.cap and self.rate(best) > self.hysteresis * self.rate(self.cap):
            self.cap = best

    def cap_for(self, batch_width: int) -> int:
        """Best cap when batch_width rows verify together, from the measured grid row of the
        smallest measured B >= batch_width (else the largest); the live cap without a grid."""
        if batch_width <= 1 or not self.verify_grid:
            return self.cap
        bs = sorted(self.verify_grid)
        row = self.verify_grid[next((b for b in bs if b >= batch_width), bs[-1])]
        return max(range(1, self.max_cap + 1), key=lambda c: self._rate(c, row))

    def info(self) -> dict:
        out = {"cap": self.cap, "p": round(self.p, 3), "rounds": self.rounds,
               "knee_width": knee_width(self.verify_ms),
               "predicted_rates": {c: round(self.rate(c) * 1e3, 1)
                                   for c in range(1, self.max_cap + 1)}}
        if self.verify_grid:
            out["batch_caps"] = {b: self.cap_for(b) for b in sorted(self.verify_grid)}
        return out


# ------------------------------------------------------------------------------ disk cache
def _cache_path(cache_dir: str | None = None) -> str:
    return os.path.join(cache_dir or CACHE_DIR, CACHE_FILE)


def cache_key(mode: str, target_repo: str, drafter_repo: str | None, ctx_len: int = CTX_LEN,
              kv_bits: int | None = None, device_name: str | None = None) -> str:
    """Entries are per device, library and torch versions, mode, model basenames, context and
    KV bits (calibrate.py:304-310; the 8-bit KV cache changes the verify curve)."""
    from . import __version__ as lib_version
    dev = device_name or (torch.cuda.get_device_name() if torch.cuda.is_available() else "cpu")
    tgt = os.path.basename(str(target_repo).rstrip("/"))
    drf = os.path.basename(str(drafter_repo).rstrip("/")) if drafter_repo else "-"
    kv = f"|kv{kv_bits}" if kv_bits else ""
    return (f"v{SCHEMA}|{dev}|dspark_b200-{lib_version}|torch{torch.__version__}|{mode}|{tgt}|"
            f"{drf}|ctx{ctx_len}{kv}")


def load_cached(key: str, cache_dir: str | None = None) -> dict | None:
    try:
        with open(_cache_path(cache_dir)) as f:
            return json.load(f).get(key)
    except (OSError, ValueError):
        return None


def save_cached(key: str, entry: dict, cache_dir: str | None = None) -> None:
    path = _cache_path(cache_dir)
    os.makedirs(os.path.dirname(path), exist_ok=True)
    try:
        with open(path) as f:
            data = json.load(f)
    except (OSError, ValueError):
        data = {}
    data[key] = entry
    tmp = path + ".tmp"
    with open(tmp, "w") as f:
        json.dump(data, f, indent=1)
    os.replace(tmp, path)


# ------------------------------------------------------------------------------ entry point
def calibrate(target, drafter, *, mode: str, target_repo: str = "", drafter_repo: str | None = None,
              cache_dir: str | None = None, verbose: bool = True,
              batch_widths: list[int] | None = None, ctx_len: int = CTX_LEN) -> CapController:
    """Measure (or load) this device's cost curves for the pair and return a CapController
    (calibrate.py:338-404). mode "dspark": caps 1..block_size, widths cap + 1; mode "dflash":
    caps up to block_size - 1, a sample of widths, and one drafter cost (the backbone always
    denoises the whole block)."""
    if getattr(drafter, "target", None) is not target:
        drafter.bind(target)
    k = int(drafter.config.block_size)
    if mode == "dspark":
        max_cap = k
        widths = list(range(2, max_cap + 2))
        caps = list(range(1, max_cap + 1))
    elif mode == "dflash":
        max_cap = k - 1
        widths = sorted({2, 3, 4, 5, 7, 9, 12, max_cap + 1})
        caps = [max_cap]
    else:
        raise ValueError(f"auto cap supports dspark/dflash, not {mode!r}")
    tap = list(drafter.config.target_layer_ids)
    key = cache_key(mode, target_repo, drafter_repo, ctx_len, getattr(target, "kv_bits", None))
    entry = load_cached(key, cache_dir)
    if entry is None:
        if verbose:
            print(f"calibrating the {mode} cap on this device (once, cached)", flush=True)
        verify = measure_verify_curve(target, tap, widths, ctx_len)
        dcurve = measure_drafter_curve(drafter, caps, ctx_len)
        entry = {"verify": {str(w): v for w, v in verify.items()},
                 "drafter": ({str(c): v for c, v in dcurve.items()} if mode == "dspark"
                             else dcurve[max_cap])}
        save_cached(key, entry, cache_dir)
        if verbose:
            rec = drafter_recommendation(verify)
            print("  verify ms by width: " +
                  " ".join(f"{w}:{v:.2f}" for w, v in sorted(verify.items())), flush=True)
            print(f"  knee at width {rec['knee_width']} -> {rec['recommend']}", flush=True)
    want = sorted({int(b) for b in (batch_widths or []) if int(b) > 1})
    have = {int(b) for b in (entry.get("verify_grid") or {})}
    if mode == "dspark" and any(b not in have for b in want):
        grid = measure_batch_verify_grid(target, tap, want, widths, ctx_len)
        vg = entry.setdefault("verify_grid", {})
        for B, row in grid.items():
            vg[str(B)] = {str(w): v for w, v in row.items()}
        save_cached(key, entry, cache_dir)
    verify = {int(w): float(v) for w, v in entry["verify"].items()}
    dms = entry["drafter"]
    dms = {int(c): float(v) for c, v in dms.items()} if isinstance(dms, dict) else float(dms)
    ctrl = CapController(verify, dms, max_cap, init_cap=2, verify_grid=entry.get("verify_grid"))
    if verbose:
        rates = ctrl.info()["predicted_rates"]
        print(f"  predicted tok/s by cap at the prior acceptance: {rates}", flush=True)
    return ctrl


__all__ = ["CapController", "calibrate", "measure_verify_curve", "measure_batch_verify_grid",
           "measure_drafter_curve", "knee_width", "drafter_recommendation", "cache_key",
           "load_cached", "save_cached", "CTX_LEN"]
