"""The timed CPU baseline's own pieces (test infrastructure checking test infrastructure): the
threaded C group-64 GEMV against a float64 restatement, and the streaming one-token decoder
against the oracle's greedy decode on the tiny target."""
import ctypes

import pytest
import torch

from mlx_dspark_b200.config import TINY
from mlx_dspark_b200.weights import generate_target
from oracle.cpu_baseline import StreamingDecoder, _gemv_lib
from oracle.dspark import greedy_generate_ref
from oracle.qwen3 import Qwen3Ref


@pytest.mark.parametrize("threads", [1, 3])
def test_c_gemv_matches_float64(threads):
    lib = _gemv_lib()
    if lib is None:
        pytest.skip("gcc could not build oracle/cpu_gemv.c")
    g = torch.Generator().manual_seed(0)
    N, K = 301, 512
    q = torch.randint(0, 256, (N, K), dtype=torch.uint8, generator=g)
    s = (torch.rand(N, K // 64, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(N, K // 64, generator=g) * 0.5).to(torch.bfloat16)
    x = torch.randn(K, generator=g)
    y = torch.zeros(N)
    xs = torch.zeros(K // 64)
    P = ctypes.c_void_p
    lib.dspark_cpu_w8_gemv(P(q.data_ptr()), P(s.data_ptr()), P(b.data_ptr()), P(x.data_ptr()),
                           P(y.data_ptr()), N, K, P(xs.data_ptr()), threads)
    w = (q.double().view(N, K // 64, 64) * s.double()[..., None] + b.double()[..., None])
    want = w.view(N, K) @ x.double()
    assert torch.allclose(y.double(), want, rtol=1e-5, atol=1e-4 * want.abs().max().item())


def test_streaming_decoder_is_greedy_decode():
    tw = generate_target(TINY, 0, "cpu")
    prompt = torch.randint(0, TINY.vocab_size, (24,), generator=torch.Generator().manual_seed(1)).tolist()
    want, _ = greedy_generate_ref(Qwen3Ref(tw), prompt, 8)
    dec = StreamingDecoder(tw, len(prompt) + 16, threads=2)
    tok = None
    for t in prompt:                 # one position at a time stands in for the prefill
        tok = dec.step(t)
    got = [tok]
    for _ in range(7):
        got.append(dec.step(got[-1]))
    assert got == want
