"""The allocation-free RMSNorm backward C entry point agrees with the regular entry point.

It is meant for callers that cannot allocate device memory when they run the kernel (a
runtime with its own pre-planned memory arena, or code without PyTorch's allocator); it keeps
its scratch in a fixed static device array.  The test calls the exported C symbol through
ctypes, twice in a row (the second call reuses the scratch left by the first), and compares
with ``rmsnorm_bwd`` of the extension within the tolerance used by the other kernel tests.
Both are also checked against a plain fp32 PyTorch restatement of the RMSNorm backward.
The cases include the documented maximum row width (8192, every slot of the per-thread
accumulator and the whole 64 x 8192 scratch in use) and a width that is not a multiple of 256.
This file is collected last on purpose.
"""
import ctypes

import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


def _lib():
    import my_muon_fsdp2_b200._C as C

    lib = ctypes.CDLL(C.__file__)
    fn = lib.mmf_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    lib.mmf_noalloc_last_error.restype = ctypes.c_char_p
    return lib, fn


def _rmsnorm_bwd_fp32(dy, x, w, rstd):
    """dx = rstd * (dy * w) - x * rstd^3 * mean(dy * w * x); dw = sum_rows dy * x * rstd."""
    dy, x, w, r = dy.float(), x.float(), w.float(), rstd.float()[:, None]
    gw = dy * w
    dx = r * gw - x * r.pow(3) * (gw * x).mean(-1, keepdim=True)
    return dx, (dy * x * r).sum(0)


def test_noalloc_rmsnorm_bwd_matches_regular_entry_point_twice():
    from my_muon_fsdp2_b200._ext import ext

    lib, fn = _lib()
    torch.manual_seed(0)
    stream = torch.cuda.current_stream()
    for rows, cols in [(300, 4096), (37, 768), (200, 8192), (64, 8000)]:
        x = torch.randn(rows, cols, device="cuda").to(torch.bfloat16)
        w = torch.randn(cols, device="cuda").to(torch.bfloat16)
        _, rstd = ext().rmsnorm_fwd(x, w, 1e-5)
        for call in range(2):
            dy = torch.randn(rows, cols, device="cuda").to(torch.bfloat16)
            ref_dx, ref_dw = ext().rmsnorm_bwd(dy, x, w, rstd)
            dx = torch.empty_like(x)
            dw = torch.empty_like(w)
            rc = fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(), rows,
                    cols, stream.cuda_stream)
            assert rc == 0, lib.mmf_noalloc_last_error()
            torch.cuda.synchronize()
            assert rel_err(dx, ref_dx) < 1e-2, f"dx mismatch on call {call}"
            assert rel_err(dw, ref_dw) < 1e-2, f"dw mismatch on call {call}"
            f_dx, f_dw = _rmsnorm_bwd_fp32(dy, x, w, rstd)
            assert rel_err(dx, f_dx) < 1e-2, f"dx differs from fp32 on call {call} ({rows}x{cols})"
            assert rel_err(dw, f_dw) < 1e-2, f"dw differs from fp32 on call {call} ({rows}x{cols})"


def test_noalloc_rejects_a_stream_of_another_device():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    lib, fn = _lib()
    t = torch.zeros(8, device="cuda:0")
    with torch.cuda.device(1):
        s1 = torch.cuda.Stream()
    rc = fn(t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), 1, 8, s1.cuda_stream)
    assert rc == 4, lib.mmf_noalloc_last_error()


def test_noalloc_rejects_oversized_rows():
    lib, fn = _lib()
    t = torch.zeros(1, device="cuda")
    rc = fn(t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), 4, 8193,
            torch.cuda.current_stream().cuda_stream)
    assert rc == 1
    assert b"8192" in lib.mmf_noalloc_last_error()
