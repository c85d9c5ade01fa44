"""The all-gather GEMM on one GPU with an emulated world: the "peer" shards are local buffers,
so the kernel's own-shard-first tile order, puller, ready counters and the G / shard source
switch all run, without NVLink.  Checked against an fp32 X W^T and the exact gathered weight."""
import os

import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu

_EXPERIMENTAL = pytest.mark.skipif(os.environ.get("MMF_TEST_EXPERIMENTAL") != "1",
                                   reason="experimental kernel, enabled by MMF_TEST_EXPERIMENTAL=1")


@pytest.mark.parametrize("variant", [0, pytest.param(1, marks=_EXPERIMENTAL)], ids=["cta1", "cta_pair"])
@pytest.mark.parametrize("M,N,K,ws,rank", [(256, 1024, 512, 4, 1), (512, 2048, 256, 8, 7), (384, 512, 768, 2, 0),
                                           (256, 4096, 1024, 8, 3)])
def test_emulated_all_gather_gemm(M, N, K, ws, rank, variant):
    from my_muon_fsdp2_b200._ext import check_device_error, ext

    if variant == 1 and M % 256:
        pytest.skip("the CTA pair takes M % 256 == 0 (the launcher falls back to one CTA otherwise)")
    torch.manual_seed(M + N + K + ws)
    rows = N // ws
    shards = [torch.randn(rows, K, device="cuda").to(torch.bfloat16) for _ in range(ws)]
    full = torch.cat(shards)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    g = torch.empty(N, K, device="cuda", dtype=torch.bfloat16)
    ready = torch.zeros(N // 128 + 1, dtype=torch.int32, device="cuda")
    ext().set_ag_gemm_variant(variant)
    try:
        for _ in range(2):  # the second call reuses the ready counters (reset inside)
            y = ext().ag_gemm(x, [s.data_ptr() for s in shards], rank, g, ready, 2e-3)
            torch.cuda.synchronize()
    finally:
        ext().set_ag_gemm_variant(0)
    check_device_error(0)
    assert torch.equal(g, full)
    ref = x.float() @ full.float().t()
    assert rel_err(y, ref) < 1e-2
