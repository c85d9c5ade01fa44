"""tcgen05 flash attention vs. a plain PyTorch fp32 causal attention (GQA)."""
import math

import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


def _ref(q, k, v):
    B, T, Hq, D = q.shape
    Hkv = k.shape[2]
    qf, kf, vf = q.float(), k.float(), v.float()
    kf = kf.repeat_interleave(Hq // Hkv, dim=2)
    vf = vf.repeat_interleave(Hq // Hkv, dim=2)
    s = torch.einsum("bqhd,bkhd->bhqk", qf, kf) / math.sqrt(D)
    mask = torch.ones(T, T, dtype=torch.bool, device=q.device).triu(1)
    s = s.masked_fill(mask, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    o = torch.einsum("bhqk,bkhd->bqhd", torch.softmax(s, dim=-1), vf)
    return o, lse


@pytest.mark.parametrize("variant", [0, 1], ids=["three_warpgroups", "two_warpgroups"])
@pytest.mark.parametrize("B,T,Hq,Hkv,D", [(1, 128, 1, 1, 128), (2, 384, 4, 2, 128), (1, 512, 2, 2, 64),
                                          (1, 1024, 8, 2, 128), (1, 640, 2, 1, 64)])
def test_attention_forward_matches_fp32(B, T, Hq, Hkv, D, variant):
    from my_muon_fsdp2_b200._ext import check_device_error, ext

    ext().set_attention_fwd_variant(variant)
    torch.manual_seed(0)
    q = torch.randn(B, T, Hq, D, device="cuda").to(torch.bfloat16)
    k = torch.randn(B, T, Hkv, D, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, T, Hkv, D, device="cuda").to(torch.bfloat16)
    o, lse = ext().attention_fwd(q, k, v, 1.0 / math.sqrt(D))
    torch.cuda.synchronize()
    check_device_error(0)
    ext().set_attention_fwd_variant(0)
    ro, rlse = _ref(q, k, v)
    assert rel_err(o, ro) < 2e-2
    assert rel_err(lse, rlse) < 1e-3


@pytest.mark.parametrize("B,T,Hq,Hkv,D", [(1, 128, 1, 1, 128), (2, 256, 4, 2, 128), (1, 384, 2, 1, 64),
                                          (1, 200, 4, 2, 128)])
def test_attention_backward_matches_fp32(B, T, Hq, Hkv, D):
    from my_muon_fsdp2_b200._ext import check_device_error, ext
    from my_muon_fsdp2_b200.ops.attention import flash_attention

    torch.manual_seed(1)
    q = torch.randn(B, T, Hq, D, device="cuda").to(torch.bfloat16).requires_grad_()
    k = torch.randn(B, T, Hkv, D, device="cuda").to(torch.bfloat16).requires_grad_()
    v = torch.randn(B, T, Hkv, D, device="cuda").to(torch.bfloat16).requires_grad_()
    o = flash_attention(q, k, v)
    do = torch.randn_like(o)
    gq, gk, gv = torch.autograd.grad(o, (q, k, v), do)
    torch.cuda.synchronize()
    check_device_error(0)
    qf, kf, vf = (t.detach().float().requires_grad_() for t in (q, k, v))
    ro, _ = _ref(qf, kf, vf)
    rq, rk, rv = torch.autograd.grad(ro, (qf, kf, vf), do.float())
    assert rel_err(o, ro) < 2e-2
    assert rel_err(gq, rq) < 3e-2, "dq"
    assert rel_err(gk, rk) < 3e-2, "dk"
    assert rel_err(gv, rv) < 3e-2, "dv"
