"""CPU tests of the Newton–Schulz map (restating the reference's tests/test_utils.py coverage)."""
import pytest
import torch

from my_muon_fsdp2_b200 import zeropower_via_newtonschulz5
from my_muon_fsdp2_b200.ops.newton_schulz import newton_schulz_reference
from tests.conftest import MAX_ORTHOGONALITY_ERROR, orthogonality_error, rel_err


class TestZeropower:
    @pytest.mark.parametrize("shape", [(256, 256), (512, 512), (512, 256), (256, 512), (16, 16)])
    def test_orthogonality_and_shape(self, shape):
        torch.manual_seed(0)
        G = torch.randn(*shape)
        W = zeropower_via_newtonschulz5(G)
        assert W.shape == G.shape
        assert orthogonality_error(W) < MAX_ORTHOGONALITY_ERROR

    @pytest.mark.parametrize("shape", [(64, 64), (96, 40), (40, 96), (3, 50)])
    @pytest.mark.parametrize("steps", [0, 1, 3, 5, 10])
    def test_smaller_gram_equals_reference_larger_gram(self, shape, steps):
        """Iterating on the wide orientation equals the reference's tall orientation (fp64)."""
        torch.manual_seed(1)
        G = torch.randn(*shape, dtype=torch.float64)
        assert rel_err(zeropower_via_newtonschulz5(G, steps=steps), newton_schulz_reference(G, steps=steps)) < 1e-9

    def test_fp32_close_to_fp64_oracle(self):
        torch.manual_seed(2)
        G = torch.randn(300, 200)
        assert rel_err(zeropower_via_newtonschulz5(G), newton_schulz_reference(G.double())) < 1e-4

    def test_bfloat16_roundtrip(self, bfloat16_matrix):
        W = zeropower_via_newtonschulz5(bfloat16_matrix)
        assert W.dtype == torch.bfloat16 and W.shape == bfloat16_matrix.shape

    def test_dtype_override(self):
        W = zeropower_via_newtonschulz5(torch.randn(32, 32), dtype=torch.float64)
        assert W.dtype == torch.float64

    def test_empty(self):
        W = zeropower_via_newtonschulz5(torch.tensor([]).reshape(0, 0))
        assert W.numel() == 0

    def test_invalid_dims(self):
        with pytest.raises(ValueError, match="at least 2 dimensions"):
            zeropower_via_newtonschulz5(torch.randn(256))

    def test_invalid_steps(self):
        with pytest.raises(ValueError, match="non-negative"):
            zeropower_via_newtonschulz5(torch.randn(8, 8), steps=-1)

    def test_batched_input(self):
        torch.manual_seed(3)
        G = torch.randn(3, 40, 24)
        W = zeropower_via_newtonschulz5(G)
        for i in range(3):
            assert rel_err(W[i], newton_schulz_reference(G[i].double())) < 1e-4

    def test_different_inputs_differ(self):
        torch.manual_seed(42)
        a, b = torch.randn(64, 64), torch.randn(64, 64)
        assert not torch.allclose(zeropower_via_newtonschulz5(a), zeropower_via_newtonschulz5(b))
