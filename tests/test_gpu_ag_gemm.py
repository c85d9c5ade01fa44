"""The all-gather GEMM on one GPU with an emulated world: the "peer" shards are local buffers,
so the kernel's own-shard-first tile order, puller, ready counters and the G / shard source
switch all run, without NVLink.  Checked against an fp32 X W^T and the exact gathered weight."""
import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K,ws,rank", [(256, 1024, 512, 4, 1), (512, 2048, 256, 8, 7), (384, 512, 768, 2, 0),
                                           (256, 4096, 1024, 8, 3)])
def test_emulated_all_gather_gemm(M, N, K, ws, rank):
    from my_muon_fsdp2_b200._ext import check_device_error, ext

    torch.manual_seed(M + N + K + ws)
    rows = N // ws
    shards = [torch.randn(rows, K, device="cuda").to(torch.bfloat16) for _ in range(ws)]
    full = torch.cat(shards)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    g = torch.empty(N, K, device="cuda", dtype=torch.bfloat16)
    ready = torch.zeros(N // 128 + 1, dtype=torch.int32, device="cuda")
    for _ in range(2):  # the second call reuses the ready counters (reset inside)
        y = ext().ag_gemm(x, [s.data_ptr() for s in shards], rank, g, ready, 2e-3)
        torch.cuda.synchronize()
    check_device_error(0)
    assert torch.equal(g, full)
    ref = x.float() @ full.float().t()
    assert rel_err(y, ref) < 1e-2
