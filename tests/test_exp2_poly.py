"""The FMA-pipe 2^x of csrc/exp2_poly.cuh: refit its coefficients by the documented procedure
(Lawson-weighted least squares for relative error, degree 3 on [0, 1]) and check the compiled
function itself (host build of the same header) against exp2 over the softmax's input range."""
import os
import shutil
import subprocess

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "my_muon_fsdp2_b200", "csrc")
COEFFS = [0.99992467893137, 0.69583643337042, 0.22606565398868, 0.07802255922514]


def test_coefficients_follow_from_the_fit():
    f = np.linspace(0, 1, 20001)
    y = 2.0 ** f
    a = np.vstack([f ** k for k in range(4)]).T
    w = 1 / y
    c = np.linalg.lstsq(a * w[:, None], y * w, rcond=None)[0]
    for _ in range(50):
        err = (a @ c - y) / y
        w = w * (np.abs(err) / np.abs(err).max()) ** 0.5 + 1e-12
        c = np.linalg.lstsq(a * w[:, None], y * w, rcond=None)[0]
    assert np.allclose(c, COEFFS, rtol=0, atol=1e-9)
    assert np.abs((a @ c - y) / y).max() < 7.6e-5


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_compiled_function_matches_exp2(tmp_path):
    src = tmp_path / "probe.cpp"
    src.write_text(
        '#include <cmath>\n#include <cstdio>\n#include "exp2_poly.cuh"\n'
        "int main() {\n"
        "  double worst = 0; int bad = 0;\n"
        "  for (int i = 0; i <= 1340000; ++i) {\n"
        "    float x = -125.0f + i * 1.0e-4f;\n"
        "    double want = std::exp2(static_cast<double>(x));\n"
        "    double got = mmf::exp2_poly(x);\n"
        "    double rel = std::fabs(got - want) / want;\n"
        "    if (rel > worst) worst = rel;\n"
        "  }\n"
        "  if (mmf::exp2_poly(-INFINITY) != 0.0f) bad |= 1;\n"
        "  if (mmf::exp2_poly(-125.5f) != 0.0f) bad |= 2;\n"
        "  if (mmf::exp2_poly(0.0f) != mmf::EXP2_POLY_C0) bad |= 4;\n"
        "  if (!std::isnan(mmf::exp2_poly(NAN))) bad |= 8;\n"
        '  std::printf("%.9g %d\\n", worst, bad);\n'
        "  return 0;\n}\n")
    exe = tmp_path / "probe"
    subprocess.run(["g++", "-O2", "-std=c++17", f"-I{CSRC}", str(src), "-o", str(exe)], check=True)
    worst, bad = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()
    assert int(bad) == 0
    assert float(worst) < 1.0e-4  # 7.6e-5 from the polynomial, plus float32 rounding of x - n
