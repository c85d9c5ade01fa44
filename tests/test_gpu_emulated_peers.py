"""The kernels of the multi-GPU paths on ONE GPU with an emulated world: every "peer" buffer is a
local allocation, so the kernels take the same pointer tables, segment scatters and rank-order
reductions as over NVLink, without a second GPU.  Each is checked against an fp32 (or fp64)
PyTorch restatement of the collective it fuses:

* ``rs_pull_reduce``: the overlapped reduce-scatter's pull-and-sum of one rank's rows;
* ``wgrad_out`` + ``rs_reduce``: the weight-gradient GEMM whose epilogue stores each rank's row
  block into that rank's receive slot, then the rank-order sum;
* the P2P Muon exchange: momentum into each rank's buffer, the owner's assembly kernel reading
  every rank's shard, and the Newton-Schulz chain whose last epilogue applies the update straight
  into every rank's parameter shard (the direct-update path of ``MuonEngine._sharded_p2p``).
"""
import pytest
import torch

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


def _E():
    from my_muon_fsdp2_b200._ext import ext

    return ext()


def _check():
    from my_muon_fsdp2_b200._ext import check_device_error

    check_device_error(torch.cuda.current_device())


@pytest.mark.parametrize("ws,rank,rows,cols", [(2, 1, 512, 4096), (8, 5, 1792, 4096), (4, 0, 100, 72)])
@pytest.mark.parametrize("accumulate", [False, True])
def test_rs_pull_reduce_emulated(ws, rank, rows, cols, accumulate):
    torch.manual_seed(ws * 10 + rank)
    n_full = ws * rows
    parts = [torch.randn(n_full, cols, device="cuda").to(torch.bfloat16) for _ in range(ws)]
    srcs = torch.tensor([p.data_ptr() for p in parts], dtype=torch.int64, device="cuda")
    out = torch.randn(rows, cols, device="cuda").to(torch.bfloat16)
    ref = sum(p[rank * rows:(rank + 1) * rows].float() for p in parts) / ws
    if accumulate:
        ref = ref + out.float()
    _E().rs_pull_reduce(srcs, rank * rows * cols, out, accumulate, 1.0 / ws)
    torch.cuda.synchronize()
    _check()
    assert rel_err(out, ref) < 1e-2


@pytest.mark.parametrize("kernel", ["linear_scatter", "tc_gemm_out"])
@pytest.mark.parametrize("ws,T,N,K", [(2, 256, 1024, 512), (4, 320, 4096, 1024), (8, 4096, 14336, 4096),
                                      (8, 200, 1024, 136)])
def test_wgrad_epilogue_scatter_then_rank_order_reduce(ws, T, N, K, kernel):
    """Every emulated rank j computes its partial dW_j = dY_j^T X_j; the GEMM epilogue stores rows
    of owner s into slot [j] of owner s; each owner then sums its ws slots (x 1/ws).  Both the
    grouped linear kernel's coalesced scatter and the NS kernel's row-segment output mode."""
    if kernel == "tc_gemm_out" and (T % 64 or K % 256):
        pytest.skip("the NS kernel's output mode takes T % 64 == 0 and K % 256 == 0")
    torch.manual_seed(T + N + ws)
    r = N // ws
    dys = [(torch.randn(T, N, device="cuda") * 0.1).to(torch.bfloat16) for _ in range(ws)]
    xs = [torch.randn(T, K, device="cuda").to(torch.bfloat16) for _ in range(ws)]
    slots = [torch.zeros(ws * r * K, dtype=torch.bfloat16, device="cuda") for _ in range(ws)]  # per owner
    meta = torch.tensor([K, 0, r], dtype=torch.int64, device="cuda")
    for j in range(ws):
        ptrs = torch.tensor([slots[s].data_ptr() + 2 * j * r * K for s in range(ws)], dtype=torch.int64,
                            device="cuda")
        if kernel == "linear_scatter":
            _E().wgrad_scatter(dys[j], xs[j], ptrs, r, None)
        else:
            _E().wgrad_out(dys[j], xs[j], ptrs, ws, meta, False, 0.0, None, 1.0)
    grads = [torch.zeros(r, K, dtype=torch.bfloat16, device="cuda") for _ in range(ws)]
    for s in range(ws):
        _E().rs_reduce(slots[s], ws, r * K, grads[s], False, 1.0 / ws)
    torch.cuda.synchronize()
    _check()
    full = sum(d.float().t() @ x.float() for d, x in zip(dys, xs)) / ws
    for s in range(ws):
        assert rel_err(grads[s], full[s * r:(s + 1) * r]) < 2e-2, f"owner {s}"


@pytest.mark.parametrize("ws", [2, 4, 8])
def test_p2p_muon_exchange_direct_update_emulated(ws):
    """The kernel sequence of the P2P Muon step for one owner, all ranks emulated: per-rank momentum
    into per-rank exchange buffers (with partial sums of squares), the owner's assembly from every
    rank's buffer, the batched NS chain, and the last epilogue applying p <- decay p - lr O into
    every rank's parameter shard.  Compared with the reference Muon step in fp64 on the full
    matrices (parameter CHANGE, so a zero or wrong update fails)."""
    from my_muon_fsdp2_b200.ops.newton_schulz import NS_EPS
    from my_muon_fsdp2_b200.ops.ns_cuda import round_up, run_ns_group, wide_shape
    from my_muon_fsdp2_b200.parallel.comm import chunk_offset, chunk_rows
    from my_muon_fsdp2_b200.parallel.muon_engine import MODE_COPY, MODE_EMA
    from tests.oracle import muon_reference_step

    E = _E()
    torch.manual_seed(ws)
    lr, mu, wd = 0.02, 0.95, 0.01
    shapes = [(ws * 96, 1024), (ws * 160, 384)]  # one wide, one tall (after sharding rows)
    full_p = [torch.randn(*s, dtype=torch.float64) for s in shapes]
    full_g = [torch.randn(*s, dtype=torch.float64) for s in shapes]
    rows_of = [chunk_rows(s[0], ws) for s in shapes]
    # per-rank shards (fp32 params, bf16 grads, fp32 momentum) and exchange buffers
    params = [[full_p[j][chunk_offset(shapes[j][0], ws, r):][:rows_of[j][r]].float().cuda().contiguous()
               for j in range(2)] for r in range(ws)]
    p0 = [[p.clone() for p in pr] for pr in params]
    grads = [[full_g[j][chunk_offset(shapes[j][0], ws, r):][:rows_of[j][r]].to(torch.bfloat16).cuda().contiguous()
              for j in range(2)] for r in range(ws)]
    bufs = [[torch.zeros(rows_of[j][r], shapes[j][1], dtype=torch.float32, device="cuda") for j in range(2)]
            for r in range(ws)]
    cnt = [[rows_of[j][r] * shapes[j][1] for j in range(2)] for r in range(ws)]
    xbuf = [torch.zeros(sum(cnt[r]), dtype=torch.bfloat16, device="cuda") for r in range(ws)]
    off = [[0, cnt[r][0]] for r in range(ws)]
    part = torch.zeros(ws, 2, dtype=torch.float32, device="cuda")
    # 1. every rank: momentum -> own exchange buffer, partial sums of squares
    for r in range(ws):
        sub = torch.zeros(2, dtype=torch.float32, device="cuda")
        E.muon_prep(grads[r], bufs[r], [], xbuf[r], off[r], [0, 0], [0, 0], [shapes[0][1], shapes[1][1]], [], [],
                    MODE_EMA, False, mu, 0.0, sub)
        part[r] = sub
    # 2. the owner (every matrix is its own group here): assembly from all ranks' buffers, NS chain,
    #    direct update of every rank's parameter shard
    for j, (rws, cls) in enumerate(shapes):
        mw, nw, tall = wide_shape(rws, cls)
        Mp, Np = round_up(mw), round_up(nw)
        X0 = torch.zeros(1, Mp, Np, dtype=torch.bfloat16, device="cuda")
        srcs = [xbuf[r][off[r][j]:off[r][j] + cnt[r][j]].view(rows_of[j][r], cls) for r in range(ws)]
        E.muon_prep(srcs, [], [], X0, [0] * ws, [chunk_offset(rws, ws, r) for r in range(ws)], [int(tall)] * ws,
                    [Np], [], [], MODE_COPY, False, 0.0, 0.0, None)
        ssq = part[:, j:j + 1].contiguous()  # [ws, 1]
        s = torch.empty(1, dtype=torch.float32, device="cuda")
        s2 = torch.empty_like(s)
        E.ns_scale(ssq, 1, ws, NS_EPS, s, s2)
        ptrs = torch.tensor([params[r][j].data_ptr() for r in range(ws)], dtype=torch.int64, device="cuda")
        meta = torch.tensor([cls, int(tall), (rws + ws - 1) // ws], dtype=torch.int64, device="cuda")
        pvec = torch.tensor([1 - lr * wd], dtype=torch.float32, device="cuda")
        vvec = torch.tensor([-lr], dtype=torch.float32, device="cuda")
        run_ns_group(X0, s, s2, 5, ptrs, 0, True, False, mw, nw, p_scale=1.0, v_scale=1.0, p_scale_vec=pvec,
                     v_scale_vec=vvec, nseg=ws, out_meta=meta, transposed_dest=tall)
    torch.cuda.synchronize()
    _check()
    # oracle: the reference Muon step (EMA momentum, NS, decoupled wd) on the full matrices, fp64,
    # from the bf16-rounded gradients the kernels saw
    ref = [p.clone() for p in full_p]
    muon_reference_step(ref, [g.to(torch.bfloat16).double() for g in full_g], [torch.zeros_like(p) for p in ref],
                        lr, mu, wd, False, 5)
    for j in range(2):
        d_ours = torch.cat([params[r][j].double().cpu() - p0[r][j].double().cpu() for r in range(ws)])
        d_ref = ref[j] - full_p[j]
        assert rel_err(d_ours, d_ref) < 0.06, f"matrix {j} {shapes[j]}"


def test_wgrad_scatter_adds_the_carry():
    """The scatter epilogue adds the unsharded no-sync accumulator C before storing."""
    torch.manual_seed(3)
    ws, T, N, K = 4, 256, 512, 384
    r = N // ws
    dy = (torch.randn(T, N, device="cuda") * 0.1).to(torch.bfloat16)
    x = torch.randn(T, K, device="cuda").to(torch.bfloat16)
    carry = torch.randn(N, K, device="cuda").to(torch.bfloat16)
    slots = [torch.zeros(r * K, dtype=torch.bfloat16, device="cuda") for _ in range(ws)]
    ptrs = torch.tensor([t.data_ptr() for t in slots], dtype=torch.int64, device="cuda")
    _E().wgrad_scatter(dy, x, ptrs, r, carry)
    torch.cuda.synchronize()
    _check()
    full = dy.float().t() @ x.float() + carry.float()
    got = torch.cat([t.view(r, K) for t in slots])
    assert rel_err(got, full) < 1e-2
