"""CPU oracle for the speculative verify step — TEST INFRASTRUCTURE ONLY.

A PyTorch-CPU (fp32) restatement of the reference's arithmetic for this path. Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s ``cpu_baseline`` / ``--impl
reference`` legs may import it, and only as the checker or the timed CPU baseline. The
product package (``mlx_dspark_b200``) never imports or calls anything here.

Parity status:
  * pinned: the Qwen3 target forward (taps, KV cache, tied/untied head) against HF
    transformers' Qwen3 implementation (transformers 5.5, the architecture mlx-lm's qwen3
    ports) through the committed fixtures in tests/golden/ (fp32 mode); the host logic
    (masks, trims, prefix reuse, n-gram lookup, penalties, spec-sampling distribution,
    batched Markov, GQA == tiling) through the reference's own unit tests restated in tests/.
  * parity unpinned against MLX itself: mlx / mlx-lm are not installed and cannot be
    (no network), so the bf16 rounding points below follow the documented behaviour of a
    bf16 MLX model (every op's output rounded to bf16; fast kernels compute in fp32) rather
    than outputs of MLX run here.

Rounding model (``rnd=True``, the default): every linear, norm, rope, attention and
elementwise result is rounded to bf16, as an MLX bf16 model stores it; accumulations are
fp32. ``rnd=False`` computes everything in fp32 (used against the HF fixtures).
"""
