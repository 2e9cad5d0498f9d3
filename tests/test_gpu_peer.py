"""The fused one-shot all-reduce on one GPU (dspark_w8a16_gemm_peer +
dspark_peer_reduce_residual), with both "ranks" in this process: two GEMM calls send their
partials and flags into two receive buffers of this GPU, and the reduce sums them in rank order
into the residual stream. The reduce runs only after both senders have finished (stream order),
so no kernel waits for another one running beside it. A flag that nothing raises makes the
bounded wait run out: the status word reports it and the GPU stays usable."""
import ctypes

import pytest
import torch

from mlx_dspark_b200 import _lib, ops
from mlx_dspark_b200.weights import pack, quantize_w8g64
from oracle import qwen3 as oq

pytestmark = pytest.mark.gpu


def _descriptor(recv, flags, rank, m_cap, n, epoch):
    ar = _lib.PeerAR()
    for r in range(2):
        ar.recv[r] = recv[r].data_ptr()
        ar.flags[r] = flags[r].data_ptr()
    ar.world, ar.rank, ar.m_cap, ar.n, ar.epoch = 2, rank, m_cap, n, epoch
    return ar


@pytest.mark.parametrize("M,N,K", [(9, 512, 1024), (1, 256, 256), (33, 1024, 512)])
def test_peer_gemm_and_reduce_loopback(cuda, M, N, K):
    g = torch.Generator().manual_seed(M + N)
    qts = [quantize_w8g64(torch.randn(N, K, generator=g) * 0.02) for _ in range(2)]
    xs = [(torch.randn(M, K, generator=g)).to(torch.bfloat16).float() for _ in range(2)]
    h0 = torch.randn(M, N, generator=g).to(torch.bfloat16)
    m_cap = 64
    recv = [torch.zeros(2 * 2 * m_cap * N, dtype=torch.float32, device=cuda) for _ in range(2)]
    flags = [torch.zeros(2 * 2 * (N // 128), dtype=torch.int32, device=cuda) for _ in range(2)]
    sc = ops.Scratch(cuda)
    h = h0.clone().to(cuda)
    for epoch in (1, 2):   # both slots, and the same residual twice
        for rank in range(2):
            ops.gemm_peer(xs[rank].to(torch.float16).to(cuda), pack(qts[rank], device=cuda),
                          _descriptor(recv, flags, rank, m_cap, N, epoch), scratch=sc, M=M)
        ops.peer_reduce_residual(h, _descriptor(recv, flags, 0, m_cap, N, epoch), M, sc,
                                 timeout_ns=100_000_000)
        torch.cuda.synchronize()
        sc.check_status()
        # the partial of each rank sits in both receive buffers, slot epoch & 1
        slot = epoch & 1
        for r in range(2):
            view = recv[r].view(2, 2, m_cap, N)
            for src in range(2):
                ref_p = xs[src] @ qts[src].dequant().t()
                bound = (xs[src].abs() @ qts[src].dequant().abs().t()) * 2.0 ** -10 + 1e-5
                assert ((view[slot, src, :M].cpu() - ref_p).abs() <= bound).all()
        assert int(flags[1].view(2, 2, -1)[slot].min()) == epoch
    # h = bf16(bf16(h0 + bf16(p0 + p1)) + bf16(p0 + p1)) with the GPU's own partials
    view = recv[0].view(2, 2, m_cap, N).cpu()
    s1 = oq.bf(view[1, 0, :M] + view[1, 1, :M])
    s2 = oq.bf(view[0, 0, :M] + view[0, 1, :M])
    ref_h = oq.bf(oq.bf(h0.float() + s1) + s2)
    assert torch.equal(h.float().cpu(), ref_h)


def test_peer_reduce_times_out_on_a_missing_flag(cuda):
    N, m_cap = 256, 8
    recv = [torch.zeros(2 * 2 * m_cap * N, dtype=torch.float32, device=cuda) for _ in range(2)]
    flags = [torch.zeros(2 * 2 * (N // 128), dtype=torch.int32, device=cuda) for _ in range(2)]
    sc = ops.Scratch(cuda)
    h = torch.zeros(1, N, dtype=torch.bfloat16, device=cuda)
    ops.peer_reduce_residual(h, _descriptor(recv, flags, 0, m_cap, N, 5), 1, sc,
                             timeout_ns=5_000_000)
    torch.cuda.synchronize()
    assert int(sc.status.item()) == _lib.DSPARK_ERR_TIMEOUT
    sc.status.zero_()
    # the context is intact: a normal call afterwards completes
    torch.ones(4, device=cuda).sum().item()
    with pytest.raises(_lib.DsparkError):
        ops.peer_reduce_residual(h, _descriptor(recv, flags, 0, m_cap, N, 0), 1, sc)  # epoch 0
