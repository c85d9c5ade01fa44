"""Every example runs to completion on CPU (gloo for the multi-process ones), so that the
documented entry points do not rot.  GPT-2 small on CPU takes about a minute; it runs with one
short step."""
import os
import subprocess
import sys

import pytest

from tests.conftest import free_port

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(args, nproc=None, timeout=400):
    env = dict(os.environ, PYTHONPATH=ROOT, OMP_NUM_THREADS="2")
    env["CUDA_VISIBLE_DEVICES"] = ""  # the CPU paths, also on a machine with GPUs
    for attempt in range(3):
        if nproc is None:
            cmd = [sys.executable] + args
        else:
            cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
                   "--master-addr=127.0.0.1", f"--master-port={free_port()}"] + args
        r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=timeout)
        # another test process may take the free port before the rendezvous binds it: new port
        if r.returncode != 0 and nproc is not None and "EADDRINUSE" in r.stderr and attempt < 2:
            continue
        break
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-3000:])
    return r.stdout


def test_simple_muon():
    out = _run(["examples/simple_muon.py"])
    assert "step 19 loss" in out


def test_single_process_fsdp2_utils():
    out = _run(["examples/single_gpu.py"])
    assert "world size: 1" in out and "step 3: loss" in out and "single-process example done" in out


def test_sso_vs_muon():
    out = _run(["examples/train_sso.py"])
    assert "muon" in out and "sso" in out


def test_hybrid_muon_adamw():
    out = _run(["examples/mixed_adamw.py", "--steps", "2"])
    assert "muon_ratio" in out and "step 1 loss" in out


@pytest.mark.distributed
def test_gloo_validation_workload():
    out = _run(["examples/gloo_validation.py"], nproc=2)
    assert "median optimizer.step()" in out


@pytest.mark.distributed
def test_hsdp_example():
    out = _run(["examples/hdsp_training.py", "--dp", "2", "--fsdp", "2"], nproc=4)
    assert "step 9 loss" in out


@pytest.mark.distributed
def test_transformer_encoder_fsdp():
    out = _run(["examples/fsdp_distributed.py", "--steps", "2", "--batch", "4", "--seq", "32"], nproc=2)
    assert "step 1 loss" in out


@pytest.mark.distributed
def test_llama_fused_fsdp_and_hsdp(tmp_path):
    out = _run(["examples/llama_symm_fsdp.py", "--steps", "1", "--seq", "32"], nproc=2)
    assert "step 0 loss" in out
    out = _run(["examples/llama_symm_fsdp.py", "--steps", "1", "--seq", "32", "--replicas", "2"], nproc=4)
    assert "step 0 loss" in out


@pytest.mark.distributed
def test_gpt2_fsdp_with_checkpoint(tmp_path):
    out = _run(["examples/train_gpt.py", "--steps", "1", "--batch", "1", "--seq", "32", "--fsdp",
                "--save-dir", str(tmp_path)], nproc=2)
    assert "step 0 loss" in out
