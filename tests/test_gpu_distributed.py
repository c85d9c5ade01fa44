"""Multi-GPU Muon on FSDP2: NCCL all-to-all and symmetric-memory P2P exchanges give the same
parameters, and both match a single-GPU run (needs >= 2 GPUs; skipped otherwise)."""
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


def _run(world, comm, out, extra=()):
    env = dict(os.environ, PYTHONPATH=ROOT, NCCL_NVLS_ENABLE="0")
    for attempt in range(3):  # a rendezvous port taken meanwhile: pick another
        cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
               f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={free_port()}",
               os.path.join(HERE, "dist_gpu_worker.py"), "--comm", comm, "--out", out, *extra]
        r = subprocess.run(cmd, env=env, capture_output=True, text=True, cwd=ROOT)
        if r.returncode == 0 or "EADDRINUSE" not in r.stderr:
            break
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return torch.load(out)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_engine_p2p_bitwise_equals_nccl():
    """Same kernels, different transport: the P2P exchange must reproduce NCCL bit for bit."""
    with tempfile.TemporaryDirectory() as d:
        a = _run(2, "nccl", os.path.join(d, "a.pt"), ["--engine-only"])
        b = _run(2, "p2p", os.path.join(d, "b.pt"), ["--engine-only"])
    for i in a:
        assert torch.equal(a[i], b[i]), f"matrix {i}: p2p differs from nccl"


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_training_matches_single_gpu():
    with tempfile.TemporaryDirectory() as d:
        a = _run(2, "nccl", os.path.join(d, "a.pt"))
        b = _run(2, "p2p", os.path.join(d, "b.pt"))
    for n in a["params"]:
        assert rel_err(a["params"][n], b["params"][n]) < 1e-2, n
    sys.path.insert(0, HERE)
    from dist_gpu_worker import build, train

    model, opts, cfg = build(1, 0, "nccl", sharded=False)
    init = {n: p.detach().float().cpu().clone() for n, p in build(1, 0, "nccl", sharded=False)[0].named_parameters()}
    losses = train(model, opts, cfg, 3, "cuda:0")
    for n, p in model.named_parameters():
        delta_ref = p.detach().float().cpu() - init[n]
        delta = a["params"][n] - init[n]
        assert rel_err(delta, delta_ref) < 0.1, n
    for x, y in zip(a["losses"], losses):
        assert abs(x - y) < 2e-2 * abs(y)
