"""tcgen05 GEMM kernel vs. a plain PyTorch fp32 reference of the same op."""
import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


def E():
    from my_muon_fsdp2_b200._ext import ext

    return ext()


@pytest.fixture(params=[1, 2], ids=["cta1", "cta_pair"], autouse=True)
def gemm_variant(request):
    """Run every GEMM test with the single-CTA and with the CTA-pair (cta_group::2) kernel."""
    E().set_gemm_variant(request.param)
    yield request.param
    E().set_gemm_variant(0)


def _bf(*shape):
    return torch.randn(*shape, device="cuda").to(torch.bfloat16)


@pytest.mark.parametrize("batch,M,N,K", [(1, 128, 256, 64), (2, 256, 512, 320), (3, 384, 256, 1024),
                                         (1, 512, 768, 4096)])
def test_kmajor_plain(batch, M, N, K):
    A, B = _bf(batch, M, K), _bf(batch, N, K)
    D = torch.empty(batch, M, N, dtype=torch.bfloat16, device="cuda")
    E().tc_gemm_ws(A, B, False, D, None, None, 1.0, None, 0.0, False)
    ref = A.float() @ B.float().transpose(1, 2)
    assert rel_err(D, ref) < 1e-2
    from my_muon_fsdp2_b200._ext import check_device_error

    check_device_error(0)


@pytest.mark.parametrize("batch,M,N,K", [(1, 128, 256, 64), (2, 256, 512, 192), (1, 768, 1024, 512)])
def test_mnmajor_axpby(batch, M, N, K):
    A, Bk = _bf(batch, M, K), _bf(batch, K, N)
    C = _bf(batch, M, N)
    alpha_vec = torch.rand(batch, device="cuda") + 0.5
    D = torch.empty(batch, M, N, dtype=torch.bfloat16, device="cuda")
    E().tc_gemm_ws(A, Bk, True, D, C, alpha_vec, 0.75, None, -1.25, False)
    ref = 0.75 * alpha_vec.view(-1, 1, 1) * (A.float() @ Bk.float()) - 1.25 * C.float()
    assert rel_err(D, ref) < 1e-2


@pytest.mark.parametrize("batch,M,K", [(1, 256, 256), (2, 512, 384), (1, 768, 128), (1, 1024, 2048)])
def test_symmetric_gram(batch, M, K):
    X = _bf(batch, M, K)
    D = torch.full((batch, M, M), float("nan"), dtype=torch.bfloat16, device="cuda")
    s2 = torch.rand(batch, device="cuda") + 0.1
    E().tc_gemm_ws(X, X, False, D, None, s2, 1.0, None, 0.0, True)
    ref = s2.view(-1, 1, 1) * (X.float() @ X.float().transpose(1, 2))
    assert not torch.isnan(D.float()).any(), "symmetric mode left elements unwritten"
    assert rel_err(D, ref) < 1e-2
    assert torch.equal(D, D.transpose(1, 2))


def test_symmetric_square_axpby():
    X = _bf(2, 512, 256)
    A = (X.float() @ X.float().transpose(1, 2) / 256).to(torch.bfloat16)
    Bm = torch.empty_like(A)
    E().tc_gemm_ws(A, A, False, Bm, A, None, 2.0315, None, -4.7750, True)
    ref = 2.0315 * (A.float() @ A.float()) - 4.7750 * A.float()
    assert rel_err(Bm, ref) < 1e-2


@pytest.mark.parametrize("transposed", [False, True])
@pytest.mark.parametrize("out_f32", [False, True])
def test_out_mode_update(transposed, out_f32):
    batch, M, N, K = 2, 256, 512, 256
    m_true, n_true = 200, 450
    A, Bk, C = _bf(batch, M, K), _bf(batch, K, N), _bf(batch, M, N)
    dt = torch.float32 if out_f32 else torch.bfloat16
    shape = (n_true, m_true) if transposed else (m_true, n_true)
    outs = [torch.randn(*shape, device="cuda").to(dt) for _ in range(batch)]
    before = [o.clone() for o in outs]
    ptrs = E().ptr_table(outs)
    ld = shape[1]
    E().tc_gemm_out(A, Bk, True, C, None, 1.0, None, 0.5, ptrs, 1, None, ld, out_f32, transposed, m_true, n_true,
                    None, 0.9, None, -0.1)
    V = (A.float() @ Bk.float() + 0.5 * C.float())[:, :m_true, :n_true]
    for b in range(batch):
        v = V[b].T if transposed else V[b]
        ref = 0.9 * before[b].float() - 0.1 * v
        assert rel_err(outs[b], ref) < 1e-2


def test_out_mode_row_segments():
    """Per-batch (ld, transposed, seg_rows) metadata: each row block lands in its own buffer."""
    batch, M, N, K = 2, 256, 256, 128
    m_true, n_true = 256, 200  # wide result 256 x 200
    A, Bk = _bf(batch, M, K), _bf(batch, K, N)
    nseg = 4
    # batch 0: destination is 256 x 200 (not transposed), 64-row segments
    # batch 1: destination is 200 x 256 (transposed), 50-row segments
    segs0 = [torch.zeros(64, 200, device="cuda") for _ in range(nseg)]
    segs1 = [torch.zeros(50, 256, device="cuda") for _ in range(nseg)]
    ptrs = E().ptr_table(segs0 + segs1)
    meta = torch.tensor([200, 0, 64, 256, 1, 50], dtype=torch.int64, device="cuda")
    E().tc_gemm_out(A, Bk, True, None, None, 1.0, None, 0.0, ptrs, nseg, meta, 0, True, False, m_true, n_true,
                    None, 0.0, None, 1.0)
    V = (A.float() @ Bk.float())[:, :m_true, :n_true]
    assert rel_err(torch.cat(segs0), V[0]) < 1e-2
    assert rel_err(torch.cat(segs1), V[1].T) < 1e-2


@pytest.mark.parametrize("T,N,K", [(64, 128, 256), (256, 512, 512), (4096, 1024, 4096), (320, 768, 256)])
@pytest.mark.parametrize("with_c", [False, True])
def test_wgrad_mnmajor_a_row_segments(T, N, K, with_c):
    """Weight gradient dW = dY^T X (+ C) with both operands MN-major, rows scattered into two
    segments (the reduce-scatter layout of two ranks)."""
    dy, x = _bf(T, N), _bf(T, K)
    C = _bf(N, K) if with_c else None
    half = N // 2
    segs = [torch.full((half, K), float("nan"), device="cuda", dtype=torch.bfloat16) for _ in range(2)]
    ptrs = torch.tensor([s.data_ptr() for s in segs], dtype=torch.int64, device="cuda")
    meta = torch.tensor([K, 0, half], dtype=torch.int64, device="cuda")
    E().wgrad_out(dy, x, ptrs, 2, meta, False, 0.0, C, 1.0)
    ref = dy.float().t() @ x.float()
    if with_c:
        ref = ref + C.float()
    assert rel_err(torch.cat(segs), ref) < 1e-2
    from my_muon_fsdp2_b200._ext import check_device_error

    check_device_error(0)
