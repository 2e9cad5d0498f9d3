"""The allocation-free acceptance entry point, called through the C ABI.

Some hosts give this library only their input and output buffers and do not let it allocate
device memory: a serving process whose device memory pool is fixed at start-up, or a binding
from another language that has no handle on the process's allocator.
dspark_accept_greedy_noalloc serves them with scratch that lives inside the library. This test
checks that it returns exactly what the workspace-based dspark_accept_greedy returns (argmax,
accepted length, committed tokens, pending token, committed KV length), on two calls in a row,
since the second call finds the first call's leftovers in the shared scratch.
"""
import pytest
import torch

from mlx_dspark_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _inputs(seed, B, T, V, device):
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(B * T, V, generator=g).to(torch.bfloat16)
    tt = logits.float().argmax(-1).view(B, T).int()
    vid = (tt + 1) % V                       # every draft rejected ...
    vid[:, 0] = 7
    vid[0, 1:] = tt[0, :T - 1]               # ... except row 0 (all accepted)
    if B > 2:
        vid[2, 1:3] = tt[2, :2]              # row 2: two accepted
    kv_len = torch.tensor([100 + 13 * b for b in range(B)], dtype=torch.int32)
    return logits.to(device), vid.to(device), kv_len.to(device)


def _outputs(B, T, device):
    return (torch.full((B * T,), -5, dtype=torch.int32, device=device),
            torch.full((B,), -5, dtype=torch.int32, device=device),
            torch.full((B, T + 2), -5, dtype=torch.int32, device=device))


def test_accept_noalloc_matches_workspace_entry_point(cuda):
    L = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    for call, (B, T, V) in enumerate([(3, 9, 151936), (2, 5, 32768)]):
        logits, vid, kv0 = _inputs(call, B, T, V, cuda)
        # reference: the workspace entry point
        am_a, pend_a, plan_a = _outputs(B, T, cuda)
        kv_a = kv0.clone()
        ops.accept_greedy(logits, B, T, vid, am_a, kv_a, True, pend_a, plan_a, ops.Scratch(cuda))
        # the allocation-free entry point, straight through the C ABI
        am_b, pend_b, plan_b = _outputs(B, T, cuda)
        kv_b = kv0.clone()
        rc = L.dspark_accept_greedy_noalloc(logits.data_ptr(), logits.stride(0), B, T, V,
                                            vid.data_ptr(), am_b.data_ptr(), kv_b.data_ptr(), 1,
                                            pend_b.data_ptr(), plan_b.data_ptr(), stream)
        assert rc == 0, L.dspark_last_error()
        torch.cuda.synchronize()
        # integer outputs: the tolerance is exact equality
        assert torch.equal(am_b, am_a), call
        assert torch.equal(pend_b, pend_a), call
        assert torch.equal(plan_b, plan_a), call
        assert torch.equal(kv_b, kv_a), call
        assert int(plan_b[0, 0]) == T - 1 and int(plan_b[1, 0]) == 0


def test_accept_noalloc_rejects_more_rows_than_its_scratch(cuda):
    L = _lib.lib()
    logits = torch.zeros(65, 1024, dtype=torch.bfloat16, device=cuda)
    ids = torch.zeros(65, dtype=torch.int32, device=cuda)
    out = torch.zeros(65 + 2, dtype=torch.int32, device=cuda)
    rc = L.dspark_accept_greedy_noalloc(logits.data_ptr(), 1024, 65, 1, 1024, ids.data_ptr(),
                                        out.data_ptr(), None, 0, out.data_ptr(), out.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream)
    assert rc == 5  # DSPARK_ERR_UNSUPPORTED
    assert b"fixed scratch" in L.dspark_last_error()
