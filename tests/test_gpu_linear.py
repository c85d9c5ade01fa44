"""Grouped transformer-linear GEMM (csrc/linear_gemm.cu) and the fused linear ops (ops/linear.py)
against plain PyTorch fp32 references of the same math."""
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


def _bf(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


def _check():
    from my_muon_fsdp2_b200._ext import check_device_error

    check_device_error(torch.cuda.current_device())


def _rope_ref(x, T, hd, theta):
    """x [M, H*hd] fp32, rows are b*T + t -> rotate-half RoPE at position t."""
    M, N = x.shape
    half = hd // 2
    inv = theta ** (-torch.arange(half, device=x.device, dtype=torch.float32) * 2.0 / hd)
    pos = (torch.arange(M, device=x.device) % T).float()
    ang = pos[:, None] * inv[None, :]
    cos, sin = ang.cos()[:, None, :], ang.sin()[:, None, :]
    x = x.view(M, N // hd, hd)
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1).reshape(M, N)


SHAPES = [(512, 768, 512), (300, 200, 136), (256, 256, 64), (1000, 1280, 4096)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("bias,resid", [(False, False), (True, True)])
def test_forward_store(M, N, K, bias, resid):
    from my_muon_fsdp2_b200.ops.linear import mm_fwd

    torch.manual_seed(0)
    x, w = _bf(M, K), _bf(N, K, scale=0.05)
    b = _bf(N) if bias else None
    r = _bf(M, N) if resid else None
    (y,) = mm_fwd(x, [w], bias=b, residual=r)
    ref = x.float() @ w.float().T
    if bias:
        ref += b.float()
    if resid:
        ref += r.float()
    _check()
    assert rel_err(y, ref) < 1e-2


def test_forward_residual_in_place():
    from my_muon_fsdp2_b200.ops.linear import EPI_STORE, gemm

    torch.manual_seed(1)
    x, w, r = _bf(384, 512), _bf(640, 512, scale=0.05), _bf(384, 640)
    ref = x.float() @ w.float().T + r.float()
    gemm([x], [w], False, False, [r], EPI_STORE, C=r)
    _check()
    assert rel_err(r, ref) < 1e-2


@pytest.mark.parametrize("M,hd,hq,hkv,T", [(512, 128, 8, 2, 256), (384, 64, 4, 2, 128), (4096, 128, 32, 8, 4096)])
def test_qkv_rope_segments(M, hd, hq, hkv, T):
    from my_muon_fsdp2_b200.ops.linear import EPI_ROPE, gemm

    torch.manual_seed(2)
    D = hq * hd
    x = _bf(M, D)
    ws = [_bf(hq * hd, D, scale=0.03), _bf(hkv * hd, D, scale=0.03), _bf(hkv * hd, D, scale=0.03)]
    outs = [torch.empty(M, w.shape[0], dtype=torch.bfloat16, device="cuda") for w in ws]
    gemm([x], ws, False, False, outs, EPI_ROPE, rope_mask=0b011, seq_len=T, head_dim=hd, rope_theta=500000.0)
    _check()
    refs = [x.float() @ w.float().T for w in ws]
    refs[0] = _rope_ref(refs[0], T, hd, 500000.0)
    refs[1] = _rope_ref(refs[1], T, hd, 500000.0)
    for o, r in zip(outs, refs):
        assert rel_err(o, r) < 1e-2


@pytest.mark.parametrize("M,F_,D", [(512, 768, 512), (300, 200, 136), (4096, 14336, 4096)])
def test_swiglu_forward_and_backward_epilogues(M, F_, D):
    from my_muon_fsdp2_b200.ops.linear import EPI_SWIGLU, EPI_SWIGLU_BWD, gemm

    torch.manual_seed(3)
    x, w1, w3, w2 = _bf(M, D), _bf(F_, D, scale=0.03), _bf(F_, D, scale=0.03), _bf(D, F_, scale=0.03)
    h, g, u = (torch.empty(M, F_, dtype=torch.bfloat16, device="cuda") for _ in range(3))
    gemm([x], [w1, w3], False, False, [h, g, u], EPI_SWIGLU)
    _check()
    gr, ur = x.float() @ w1.float().T, x.float() @ w3.float().T
    assert rel_err(g, gr) < 1e-2 and rel_err(u, ur) < 1e-2
    assert rel_err(h, F.silu(gr) * ur) < 1e-2
    dy = _bf(M, D)
    dg, du = torch.empty_like(g), torch.empty_like(u)
    gemm([dy], [w2], False, True, [dg, du], EPI_SWIGLU_BWD, aux0=g, aux1=u)
    _check()
    dh = dy.float() @ w2.float()
    gf, uf = g.float(), u.float()
    s = torch.sigmoid(gf)
    assert rel_err(dg, dh * uf * s * (1 + gf * (1 - s))) < 1e-2
    assert rel_err(du, dh * gf * s) < 1e-2


@pytest.mark.parametrize("M,N,Ks", [(512, 512, (512, 128, 128)), (300, 136, (200, 64, 72)), (4096, 4096, (14336, 14336))])
def test_input_gradient_k_segments(M, N, Ks):
    from my_muon_fsdp2_b200.ops.linear import mm_dx

    torch.manual_seed(4)
    dys = [_bf(M, k) for k in Ks]
    ws = [_bf(k, N, scale=0.03) for k in Ks]
    dx = mm_dx(dys, ws)
    _check()
    ref = sum(d.float() @ w.float() for d, w in zip(dys, ws))
    assert rel_err(dx, ref) < 1e-2
    acc = _bf(M, N)
    ref2 = acc.float() + ref
    mm_dx(dys, ws, add_to=acc)
    _check()
    assert rel_err(acc, ref2) < 1e-2


@pytest.mark.parametrize("T,Ns,K", [(512, (512, 128, 128), 512), (200, (136, 64), 72), (4096, (14336, 14336), 4096)])
@pytest.mark.parametrize("f32", [False, True])
def test_weight_gradient_m_segments_accumulate(T, Ns, K, f32):
    from my_muon_fsdp2_b200.ops.linear import mm_dw

    torch.manual_seed(5)
    x = _bf(T, K)
    dys = [_bf(T, n, scale=0.1) for n in Ns]
    dt = torch.float32 if f32 else torch.bfloat16
    outs = [torch.empty(n, K, dtype=dt, device="cuda") for n in Ns]
    mm_dw(dys, x, outs, accumulate=False)
    _check()
    refs = [d.float().T @ x.float() for d in dys]
    for o, r in zip(outs, refs):
        assert rel_err(o, r) < 1e-2
    mm_dw(dys, x, outs, accumulate=True)
    _check()
    for o, r in zip(outs, refs):
        assert rel_err(o, 2 * r) < 1e-2


@pytest.mark.parametrize("M,N,K", [(512, 3072, 768), (300, 200, 136)])
def test_gelu_epilogues(M, N, K):
    from my_muon_fsdp2_b200.ops.linear import EPI_GELU, EPI_GELU_BWD, gemm

    torch.manual_seed(6)
    x, w, b = _bf(M, K), _bf(N, K, scale=0.05), _bf(N)
    a, z = torch.empty(M, N, dtype=torch.bfloat16, device="cuda"), torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    gemm([x], [w], False, False, [a, z], EPI_GELU, bias=b)
    _check()
    zr = x.float() @ w.float().T + b.float()
    assert rel_err(z, zr) < 1e-2 and rel_err(a, F.gelu(zr)) < 1e-2
    w2, dy = _bf(K, N, scale=0.05), _bf(M, K)
    dz = torch.empty_like(z)
    gemm([dy], [w2], False, True, [dz], EPI_GELU_BWD, aux0=z)
    _check()
    zf = z.float().requires_grad_()
    (ga,) = torch.autograd.grad(F.gelu(zf), zf, dy.float() @ w2.float())
    assert rel_err(dz, ga) < 1e-2


# ---------------------------------------------------------------- autograd-level fused ops
def _grads(params):
    return [p.grad.detach().clone() for p in params]


def test_fused_llama_block_matches_fp32_autograd():
    """One Llama block (q|k|v + RoPE, attention, wo + residual, SwiGLU FFN + residual) on the
    fused kernels vs the same block in fp32 with PyTorch ops: output and every gradient."""
    from my_muon_fsdp2_b200.models.llama import LlamaConfig, TransformerBlock

    torch.manual_seed(7)
    cfg = LlamaConfig.tiny(dim=512, n_heads=4, n_kv_heads=2, ffn_dim=1024)
    blk = TransformerBlock(cfg)
    ref = TransformerBlock(cfg)
    ref.load_state_dict(blk.state_dict())
    blk = blk.to("cuda", torch.bfloat16)
    ref = ref.to("cuda", torch.float32)
    x = _bf(2, 256, 512)
    xr = x.float().requires_grad_()
    x.requires_grad_()
    y = blk(x)
    # the fp32 reference runs the CPU-style PyTorch paths (not bf16 -> not the native kernels)
    yr = ref(xr)
    dy = _bf(2, 256, 512)
    y.backward(dy)
    yr.backward(dy.float())
    _check()
    assert rel_err(y, yr) < 2e-2
    assert rel_err(x.grad, xr.grad) < 3e-2
    for (n, p), (_, q) in zip(blk.named_parameters(), ref.named_parameters()):
        assert rel_err(p.grad, q.grad) < 3e-2, n


def test_fused_gelu_mlp_and_linear_match_fp32_autograd():
    from my_muon_fsdp2_b200.ops.linear import gelu_mlp, linear

    torch.manual_seed(8)
    fc, proj = nn.Linear(256, 1024), nn.Linear(1024, 256)
    fcr, projr = nn.Linear(256, 1024), nn.Linear(1024, 256)
    fcr.load_state_dict(fc.state_dict())
    projr.load_state_dict(proj.state_dict())
    fc, proj = fc.cuda().bfloat16(), proj.cuda().bfloat16()
    fcr, projr = fcr.cuda(), projr.cuda()
    x, res = _bf(300, 256), _bf(300, 256)
    x.requires_grad_()
    xr = x.detach().float().requires_grad_()
    y = gelu_mlp(x, fc, proj, residual=res)
    yr = projr(F.gelu(fcr(xr))) + res.float()
    dy = _bf(300, 256)
    y.backward(dy)
    yr.backward(dy.float())
    _check()
    assert rel_err(y, yr) < 2e-2 and rel_err(x.grad, xr.grad) < 3e-2
    for p, q in [(fc.weight, fcr.weight), (fc.bias, fcr.bias), (proj.weight, projr.weight), (proj.bias, projr.bias)]:
        assert rel_err(p.grad, q.grad) < 3e-2


def test_fused_linear_with_bias_and_residual_matches_fp32_autograd():
    from my_muon_fsdp2_b200.ops.linear import linear

    torch.manual_seed(9)
    m, mr = nn.Linear(320, 200), nn.Linear(320, 200)
    mr.load_state_dict(m.state_dict())
    m, mr = m.cuda().bfloat16(), mr.cuda()
    x, res = _bf(2, 150, 320), _bf(2, 150, 200)
    x.requires_grad_()
    res.requires_grad_()
    xr, rr = x.detach().float().requires_grad_(), res.detach().float().requires_grad_()
    y = linear(x, m, residual=res)
    yr = mr(xr) + rr
    dy = _bf(2, 150, 200)
    y.backward(dy)
    yr.backward(dy.float())
    _check()
    assert rel_err(y, yr) < 2e-2 and rel_err(x.grad, xr.grad) < 3e-2 and rel_err(res.grad, rr.grad) < 1e-2
    assert rel_err(m.weight.grad, mr.weight.grad) < 3e-2 and rel_err(m.bias.grad, mr.bias.grad) < 3e-2


def test_launch_from_a_thread_without_cuda_context():
    """A thread whose first CUDA work is one of this library's GEMMs (autograd's backward worker
    can be one): the launcher binds the device's context before encoding its tensor maps."""
    import threading

    from my_muon_fsdp2_b200.ops.linear import mm_fwd

    x, w = _bf(256, 512), _bf(384, 512, scale=0.05)
    ref = x.float() @ w.float().T
    out = {}

    def run():
        try:
            (out["y"],) = mm_fwd(x, [w])
            torch.cuda.synchronize()
        except Exception as e:  # reported below
            out["e"] = e

    t = threading.Thread(target=run)
    t.start()
    t.join()
    assert "e" not in out, out.get("e")
    assert rel_err(out["y"], ref) < 1e-2


def test_split_last_wave_matches_whole_tiles():
    """The split last wave (the tail tiles' K-parts on idle CTA pairs with an fp32 fix-up, taken
    when every part keeps >= 8192 of the reduction) gives the whole-tile result for each kernel
    form and epilogue, twice in a row (the flags reset themselves).  4096 x 4096 outputs are 256
    tiles: three full waves of the 74 pairs and 34 tail tiles, split in two along K = 16384."""
    from my_muon_fsdp2_b200._ext import ext
    from my_muon_fsdp2_b200.ops.linear import EPI_GELU, EPI_GELU_BWD, EPI_SWIGLU_BWD, gemm, mm_dw, mm_dx, mm_fwd

    torch.manual_seed(11)
    M, N, K = 4096, 4096, 16384
    x, w = _bf(M, K), _bf(N, K, scale=0.01)
    dy, w2 = _bf(M, K), _bf(K, N, scale=0.01)
    dyt, xt = _bf(K, N, scale=0.1), _bf(K, N)
    g, u, r = _bf(M, N), _bf(M, N), _bf(M, N)
    bias = _bf(N, scale=0.1)
    res = {}
    for split in (False, True):
        ext().set_linear_split_tail(split)
        try:
            for _ in range(2):
                (y,) = mm_fwd(x, [w], residual=r)
                dx = mm_dx([dy], [w2])
                dw = torch.empty(N, N, dtype=torch.bfloat16, device="cuda")
                mm_dw([dyt], xt, [dw], accumulate=False)
                dw32 = torch.ones(N, N, dtype=torch.float32, device="cuda")
                mm_dw([dyt], xt, [dw32], accumulate=True)
                dg, du = torch.empty_like(g), torch.empty_like(u)
                gemm([dy], [w2], False, True, [dg, du], EPI_SWIGLU_BWD, aux0=g, aux1=u)
                a_, z_ = torch.empty_like(g), torch.empty_like(g)
                gemm([x], [w], False, False, [a_, z_], EPI_GELU, bias=bias)
                dz = torch.empty_like(g)
                gemm([dy], [w2], False, True, [dz], EPI_GELU_BWD, aux0=g)
                torch.cuda.synchronize()
                _check()
        finally:
            ext().set_linear_split_tail(True)
        res[split] = (y, dx, dw, dw32, dg, du, a_, z_, dz)
    for i, (a, b) in enumerate(zip(res[False], res[True])):
        assert rel_err(b, a) < 5e-3, f"output {i}"
    ref = x.float() @ w.float().T + r.float()
    assert rel_err(res[True][0], ref) < 1e-2
    assert rel_err(res[True][3], 1.0 + dyt.float().T @ xt.float()) < 1e-2
