"""The GPT-2 model of this library is the GPT-2 architecture of the reference example (pre-LN,
learned positions, exact-GELU MLP, tied LM head): with the same weights its CPU path gives the
logits of the `transformers` GPT-2 configured with exact GELU (its Conv1D weights are stored
transposed)."""
import pytest
import torch

transformers = pytest.importorskip("transformers")


def test_logits_match_transformers_gpt2():
    from transformers import GPT2Config, GPT2LMHeadModel

    from my_muon_fsdp2_b200.models.gpt2 import GPTConfig, GPTModel

    torch.manual_seed(0)
    ours = GPTModel(GPTConfig(vocab_size=96, n_positions=64, n_embd=64, n_layer=2, n_head=4))
    hf = GPT2LMHeadModel(GPT2Config(vocab_size=96, n_positions=64, n_embd=64, n_layer=2, n_head=4,
                                    activation_function="gelu", resid_pdrop=0.0, embd_pdrop=0.0, attn_pdrop=0.0,
                                    layer_norm_epsilon=1e-5)).eval()
    hp = dict(hf.named_parameters())
    with torch.no_grad():
        for n, p in ours.named_parameters():
            key = "transformer." + n
            tgt = hp[key]
            # transformers' Conv1D keeps weights as [in, out]; nn.Linear as [out, in]
            tgt.copy_(p.t() if (tgt.dim() == 2 and n.startswith("h.") and tgt.shape == p.t().shape) else p)
    torch.manual_seed(1)
    x = torch.randint(0, 96, (2, 40))
    with torch.no_grad():
        want = hf(input_ids=x).logits
        got = ours(x)
    assert torch.allclose(got, want, rtol=1e-4, atol=1e-4), (got - want).abs().max()
