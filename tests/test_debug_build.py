"""The debug build (MMF_DEVICE_CHECKS=1: device-side index and segment checks that record an
error code and skip the access) must compile for sm_100a next to the release build.  Cross-
compiles the kernels that carry checks to object files; needs nvcc, no GPU."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "my_muon_fsdp2_b200", "csrc")


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="needs nvcc")
@pytest.mark.parametrize("src", ["tc_gemm.cu", "linear_gemm.cu"])
def test_device_checks_build_compiles(src, tmp_path):
    from torch.utils.cpp_extension import include_paths

    cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
           "--expt-relaxed-constexpr", "-DMMF_DEVICE_CHECKS", f"-I{CSRC}"]
    cmd += [f"-I{p}" for p in include_paths()]
    cmd += ["-c", os.path.join(CSRC, src), "-o", str(tmp_path / (src + ".o"))]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]


def test_error_codes_are_decoded():
    from my_muon_fsdp2_b200._ext import _ERROR_TEXT

    assert set(_ERROR_TEXT) == set(range(1, 9))
    assert "timed out" in _ERROR_TEXT[5] and "debug check" in _ERROR_TEXT[8]
