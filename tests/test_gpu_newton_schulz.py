"""Batched bf16 tcgen05 Newton–Schulz chain vs. the fp64 restatement of the reference loop."""
import pytest
import torch

from my_muon_fsdp2_b200.ops.newton_schulz import newton_schulz_reference, zeropower_via_newtonschulz5
from tests.conftest import MAX_ORTHOGONALITY_ERROR, orthogonality_error, rel_err

pytestmark = pytest.mark.gpu

# bf16 operands through 3*steps GEMMs: a few percent relative Frobenius error vs fp64.
NS_TOL = 0.06


@pytest.mark.parametrize("shape", [(256, 256), (512, 256), (256, 512), (300, 700), (1024, 4096), (4096, 1024)])
@pytest.mark.parametrize("steps", [1, 5])
def test_ns_matches_fp64_oracle(shape, steps):
    torch.manual_seed(0)
    G = torch.randn(*shape)
    ref = newton_schulz_reference(G.double(), steps=steps)
    out = zeropower_via_newtonschulz5(G.cuda(), steps=steps)
    assert out.shape == G.shape and out.dtype == G.dtype
    err = rel_err(out.cpu(), ref)
    assert err < NS_TOL, f"rel err {err:.4f}"


def test_ns_bf16_in_out_and_orthogonality():
    torch.manual_seed(1)
    G = torch.randn(512, 512, dtype=torch.bfloat16, device="cuda")
    W = zeropower_via_newtonschulz5(G)
    assert W.dtype == torch.bfloat16
    assert orthogonality_error(W) < MAX_ORTHOGONALITY_ERROR


def test_ns_steps_zero_is_normalised_input():
    G = torch.randn(128, 300, device="cuda")
    W = zeropower_via_newtonschulz5(G, steps=0)
    ref = G / (G.norm() + 1e-7)
    assert rel_err(W, ref) < 1e-2


def test_ns_batched_mixed_shapes():
    from my_muon_fsdp2_b200.ops.ns_cuda import newton_schulz_batched

    torch.manual_seed(2)
    mats = [torch.randn(256, 512, device="cuda"), torch.randn(256, 512, device="cuda"), torch.randn(384, 128, device="cuda")]
    outs = newton_schulz_batched(mats, steps=5)
    for m, o in zip(mats, outs):
        assert rel_err(o.cpu(), newton_schulz_reference(m.cpu().double())) < NS_TOL
