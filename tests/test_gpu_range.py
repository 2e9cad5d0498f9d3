"""fp16 operands at the edge of their range: the SiLU*up activations, the fp16 hidden-state taps
and the attention output are bf16 values stored as fp16 for the next GEMM, exact while
|x| <= 65504. Values scaled toward 6e4 pass through exactly; one past the range is stored as an
fp16 infinity and reported as DSPARK_ERR_RANGE in the status word (a DsparkError with code 8
on the host), after which the status is clear again."""
import pytest
import torch

from mlx_dspark_b200 import _lib, ops
from mlx_dspark_b200._lib import EPI_RESIDUAL_BF16, EPI_SILU_MUL_F16
from mlx_dspark_b200.weights import QTensor, pack
from oracle import qwen3 as oq

pytestmark = pytest.mark.gpu

RANGE = 8  # DSPARK_ERR_RANGE


def _expect_range_error(sc: ops.Scratch) -> None:
    with pytest.raises(_lib.DsparkError) as e:
        sc.check_status()
    assert e.value.code == RANGE
    sc.check_status()  # cleared


def _const_linear(N: int, K: int) -> QTensor:
    """Every weight 255 * 2^-8 (q = 255, scale 2^-8, bias 0: exact in bf16 and fp16)."""
    q = torch.full((N, K), 255, dtype=torch.uint8)
    s = torch.full((N, K // 64), 2.0 ** -8).to(torch.bfloat16)
    b = torch.zeros(N, K // 64, dtype=torch.bfloat16)
    return QTensor(q, s, b)


def test_silu_output_range(cuda):
    K = 128
    g, u = _const_linear(128, K), _const_linear(128, K)
    w = pack(g, u, interleave64=True, device=cuda)
    sc = ops.Scratch(cuda)
    y = torch.zeros(1, 128, dtype=torch.float16, device=cuda)
    # gate = up = 127.5 * v; v = 1.921875: bf16(245.04) = 245, act = bf16(245^2) = 59904
    x = torch.full((1, K), 1.921875, dtype=torch.float16, device=cuda)
    ops.gemm(x, w, y, epilogue=EPI_SILU_MUL_F16, scratch=sc, M=1)
    torch.cuda.synchronize()
    sc.check_status()
    assert torch.all(y.float() == 59904.0), y.float().unique()
    # v = 2.0625: bf16(262.97) = 262, act = bf16(262^2) = 68608 > 65504
    x.fill_(2.0625)
    ops.gemm(x, w, y, epilogue=EPI_SILU_MUL_F16, scratch=sc, M=1)
    torch.cuda.synchronize()
    _expect_range_error(sc)
    assert torch.isinf(y.float()).all()


def test_hidden_state_tap_range(cuda):
    H, K = 256, 128
    w = pack(_const_linear(H, K), device=cuda)
    sc = ops.Scratch(cuda)
    x = torch.zeros(2, K, dtype=torch.float16, device=cuda)   # the GEMM adds 0
    tap = torch.zeros(2, H, dtype=torch.float16, device=cuda)
    # (65280 is the largest bf16 value inside the fp16 range)
    for value, ok in ((60000.0, True), (65280.0, True), (70000.0, False), (-1e5, False)):
        h = torch.full((2, H), value, dtype=torch.bfloat16, device=cuda)
        want = h.float().clone()
        ops.gemm(x, w, h, epilogue=EPI_RESIDUAL_BF16, residual=h, scratch=sc, M=2, copy16=tap)
        torch.cuda.synchronize()
        assert torch.equal(h.float(), want)
        if ok:
            sc.check_status()
            assert torch.equal(tap.float(), want)
        else:
            _expect_range_error(sc)
            assert torch.isinf(tap.float()).all()


def test_attention_output_range(cuda):
    from test_gpu_kernels import CacheStateRow, _pool_and_state
    Hq, Hkv, hd, T, L = 8, 1, 128, 1, 200
    pool, st = _pool_and_state(cuda, Hkv, hd, False, 1, L + T + 64)
    sc = ops.Scratch(cuda)
    q = torch.randn(T, Hq * hd).to(torch.bfloat16).to(cuda)
    out = torch.zeros(T, Hq * hd, dtype=torch.float16, device=cuda)
    for value, ok in ((6.0e4, True), (7.0e4, False)):
        # K rows random (normalised by the writer), V rows all `value`: the output is `value`
        kv = torch.cat([torch.randn(L + T, hd), torch.full((L + T, hd), value)], 1).to(torch.bfloat16)
        view = CacheStateRow(st, 0)
        for done in range(0, L + T, 64):      # the writer takes up to 64 rows a call
            t = min(64, L + T - done)
            view.seq_len.fill_(done)
            ops.qkv_rope_kv_write(kv[done:done + t].to(cuda), 1, t, 0, Hkv, hd, None,
                                  torch.ones(hd, dtype=torch.bfloat16, device=cuda), 1e-6,
                                  oq.inv_freq(hd, 1e6).to(cuda), view.seq_len, None,
                                  view.layout(0))
        st.seq_len.fill_(L)
        for splits in (1, 4):
            ops.attention(q, 1, T, Hq, st.layout(0), st.seq_len, True, hd ** -0.5, out, splits, sc)
            torch.cuda.synchronize()
            want = torch.tensor(value).to(torch.bfloat16).float().to(cuda)
            if ok:
                sc.check_status()
                # P is rounded to bf16 before P.V, so the mean of equal values may move by an ulp
                assert torch.allclose(out.float(), want.expand_as(out), rtol=2.0 ** -7, atol=0), \
                    (splits, out.float().unique())
            else:
                _expect_range_error(sc)
                assert torch.isinf(out.float()).all()
