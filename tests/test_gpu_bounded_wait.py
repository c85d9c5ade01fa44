"""Bounded device waits: a barrier whose peer flag is never set gives up after its limit and
reports an error status to the host; the CUDA context stays usable.  Single GPU: both "ranks'"
signal pads are ordinary local buffers and the second rank simply never signals."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_barrier_timeout_reports_error_and_context_survives():
    from my_muon_fsdp2_b200._ext import check_device_error, ext

    pads = [torch.zeros(64, dtype=torch.int32, device="cuda") for _ in range(2)]
    ptrs = torch.tensor([p.data_ptr() for p in pads], dtype=torch.int64, device="cuda")
    t0 = time.time()
    ext().symm_barrier(ptrs, 0, 2, 1, 0, None, None, 0.2)  # rank 1 never signals
    torch.cuda.synchronize()
    assert time.time() - t0 < 5.0
    with pytest.raises(RuntimeError, match="timed out"):
        check_device_error(0)
    # rank 0 did signal rank 1's pad
    assert pads[1][0].item() == 1
    # the context is still healthy and the error word was cleared
    x = torch.randn(1024, device="cuda")
    assert torch.isfinite(x.sum()).item()
    check_device_error(0)


def test_barrier_completes_when_peer_signalled():
    from my_muon_fsdp2_b200._ext import check_device_error, ext

    pads = [torch.zeros(64, dtype=torch.int32, device="cuda") for _ in range(2)]
    pads[0][1] = 5  # "rank 1" already signalled epoch 5 into rank 0's pad
    ptrs = torch.tensor([p.data_ptr() for p in pads], dtype=torch.int64, device="cuda")
    payload = torch.arange(3, dtype=torch.float32, device="cuda")
    rows = [torch.zeros(6, dtype=torch.float32, device="cuda") for _ in range(2)]
    pptrs = torch.tensor([r.data_ptr() for r in rows], dtype=torch.int64, device="cuda")
    ext().symm_barrier(ptrs, 0, 2, 5, 0, payload, pptrs, 2.0)
    torch.cuda.synchronize()
    check_device_error(0)
    for r in rows:
        assert torch.equal(r[:3], payload)
