"""Fused FSDP collectives on >= 2 GPUs: the all-gather GEMM and the GEMM -> reduce-scatter
against fp32 references, and SymmFSDP training against plain FSDP2 (skipped with < 2 GPUs)."""
import os
import subprocess
import sys
import tempfile

import pytest
import torch

from tests.conftest import free_port, rel_err

pytestmark = [pytest.mark.gpu, pytest.mark.distributed]

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _run(world, mode, out):
    env = dict(os.environ, PYTHONPATH=ROOT, NCCL_NVLS_ENABLE="0")
    for attempt in range(3):  # a rendezvous port taken meanwhile: pick another
        cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
               f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={free_port()}",
               os.path.join(HERE, "symm_fsdp_worker.py"), "--mode", mode, "--out", out]
        r = subprocess.run(cmd, env=env, capture_output=True, text=True, cwd=ROOT)
        if r.returncode == 0 or "EADDRINUSE" not in r.stderr:
            break
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return torch.load(out)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_allgather_gemm_and_reduce_scatter():
    with tempfile.TemporaryDirectory() as d:
        res = _run(2, "kernels", os.path.join(d, "k.pt"))
    for k, v in res.items():
        if k.startswith("g"):
            assert v, f"{k}: gathered weight differs from the full weight"
        else:
            assert v < 1e-2, f"{k}: relative error {v}"


def test_symm_fsdp_one_rank_training_matches_fsdp2():
    """One rank: SymmFSDP's weight sources and grouped gradient GEMMs (q|k|v, w1|w3 partial sums
    into the gradient shards) against FSDP2's autograd-returned gradients, same fused kernels."""
    with tempfile.TemporaryDirectory() as d:
        res = _run(1, "train", os.path.join(d, "t1.pt"))
    a, b = res["symm"], res["fsdp2"]
    for x, y in zip(a["losses"], b["losses"]):
        assert abs(x - y) < 2e-2 * abs(y), (a["losses"], b["losses"])
    for n in b["params"]:
        assert rel_err(a["params"][n], b["params"][n]) < 2e-2, n


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["train", "train_shard_root"], ids=["root_replicated", "root_fsdp2"])
def test_symm_fsdp_training_matches_fsdp2(mode):
    """SymmFSDP linears with the rest of the model replicated (default) or under FSDP2, against
    plain FSDP2 everywhere, from the same initial weights."""
    with tempfile.TemporaryDirectory() as d:
        res = _run(2, mode, os.path.join(d, "t.pt"))
    a, b = res["symm"], res["fsdp2"]
    assert a["direct_updates"] > 0 and b["direct_updates"] == 0  # in-place peer updates on symm shards only
    for x, y in zip(a["losses"], b["losses"]):
        assert abs(x - y) < 2e-2 * abs(y), (a["losses"], b["losses"])
    for n in b["params"]:
        assert rel_err(a["params"][n], b["params"][n]) < 2e-2, n


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_cooperative_ns_schedule_matches_owner_computes():
    with tempfile.TemporaryDirectory() as d:
        res = _run(2, "split", os.path.join(d, "s.pt"))
    for n in res["never"]:
        assert rel_err(res["always"][n], res["never"][n]) < 2e-2, n


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_mixed_fused_and_nccl_weights_with_bias():
    with tempfile.TemporaryDirectory() as d:
        res = _run(2, "mixed", os.path.join(d, "m.pt"))
    assert res.pop("fused_ok") == [True, False]
    for k, v in res.items():
        if k.startswith("g"):
            assert v, f"{k}: gathered weight differs from the full weight"
        else:
            assert v < 1e-2, f"{k}: relative error {v}"


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs 4 GPUs")
def test_symm_fsdp_hsdp_training_matches_fsdp2_hsdp():
    """2 x 2 mesh: fused collectives inside each shard pair, replica averaging across pairs."""
    with tempfile.TemporaryDirectory() as d:
        res = _run(4, "hsdp", os.path.join(d, "h.pt"))
    a, b = res["symm"], res["fsdp2"]
    for x, y in zip(a["losses"], b["losses"]):
        assert abs(x - y) < 2e-2 * abs(y), (a["losses"], b["losses"])
    for n in b["params"]:
        assert rel_err(a["params"][n], b["params"][n]) < 2e-2, n
