"""The Llama model of this library is the Llama-3 architecture: with the same weights, its CPU
path gives the logits and loss of the `transformers` Llama (rotate-half RoPE with theta 5e5,
GQA, RMSNorm, SwiGLU, untied LM head).  This is what the benchmark's random-init 8B model is."""
import pytest
import torch

transformers = pytest.importorskip("transformers")


def _pair():
    from transformers import LlamaConfig as HFConfig
    from transformers import LlamaForCausalLM

    from my_muon_fsdp2_b200.models.llama import Llama, LlamaConfig

    cfg = LlamaConfig.tiny(dim=64, n_heads=4, n_kv_heads=2, ffn_dim=128, vocab_size=96, n_layers=2,
                           rope_theta=500000.0, norm_eps=1e-5)
    torch.manual_seed(0)
    ours = Llama(cfg)
    for p in ours.parameters():
        torch.nn.init.normal_(p, 0.0, 0.05)
    hf = LlamaForCausalLM(HFConfig(vocab_size=96, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, rope_theta=500000.0,
                                   rms_norm_eps=1e-5, max_position_embeddings=256, tie_word_embeddings=False,
                                   attention_bias=False, mlp_bias=False))
    names = {"tok_embeddings.weight": "model.embed_tokens.weight", "norm.weight": "model.norm.weight",
             "output.weight": "lm_head.weight"}
    for i in range(2):
        a, b = f"layers.{i}.", f"model.layers.{i}."
        names.update({a + "attention.wq.weight": b + "self_attn.q_proj.weight",
                      a + "attention.wk.weight": b + "self_attn.k_proj.weight",
                      a + "attention.wv.weight": b + "self_attn.v_proj.weight",
                      a + "attention.wo.weight": b + "self_attn.o_proj.weight",
                      a + "feed_forward.w1.weight": b + "mlp.gate_proj.weight",
                      a + "feed_forward.w3.weight": b + "mlp.up_proj.weight",
                      a + "feed_forward.w2.weight": b + "mlp.down_proj.weight",
                      a + "attention_norm.weight": b + "input_layernorm.weight",
                      a + "ffn_norm.weight": b + "post_attention_layernorm.weight"})
    hf_params = dict(hf.named_parameters())
    with torch.no_grad():
        for n, p in ours.named_parameters():
            hf_params[names[n]].copy_(p)
    assert set(names.values()) == set(hf_params)
    return ours, hf.eval()


def test_logits_and_loss_match_transformers_llama():
    ours, hf = _pair()
    torch.manual_seed(1)
    tok = torch.randint(0, 96, (2, 33))
    x, y = tok[:, :-1], tok[:, 1:]
    with torch.no_grad():
        want = hf(input_ids=x).logits
        got = ours(x)
        loss = ours(x, y)
    assert torch.allclose(got, want, rtol=1e-4, atol=1e-4), (got - want).abs().max()
    ref_loss = torch.nn.functional.cross_entropy(want.reshape(-1, 96), y.reshape(-1))
    assert abs(float(loss) - float(ref_loss)) < 1e-4
