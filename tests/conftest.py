"""Shared pytest configuration.

Markers:
  gpu          needs a CUDA device (B200, sm_100a) and the built native extension
  distributed  spawns several processes (gloo on CPU unless marked gpu as well)
  slow         long-running
"""
import os
import socket

import pytest
import torch


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device and the built sm_100a extension")
    config.addinivalue_line("markers", "distributed: spawns several processes")
    config.addinivalue_line("markers", "slow: long-running test")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if item.get_closest_marker("gpu"):
            item.add_marker(skip)


@pytest.fixture
def seed():
    torch.manual_seed(42)
    return 42


@pytest.fixture
def random_matrix_256():
    return torch.randn(256, 256)


@pytest.fixture
def random_matrix_512():
    return torch.randn(512, 512)


@pytest.fixture
def random_matrix_tall():
    return torch.randn(512, 256)


@pytest.fixture
def random_matrix_wide():
    return torch.randn(256, 512)


@pytest.fixture
def bfloat16_matrix():
    return torch.randn(256, 256, dtype=torch.bfloat16)


MAX_ORTHOGONALITY_ERROR = 15.0  # quintic NS is deliberately not exactly orthogonal


def orthogonality_error(W: torch.Tensor) -> float:
    """||W^T W - I|| for tall W, ||W W^T - I|| otherwise (in fp32)."""
    W = W.float()
    if W.size(0) > W.size(1):
        P = W.T @ W
    else:
        P = W @ W.T
    return (P - torch.eye(P.size(0), device=W.device)).norm().item()


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double()
    b = b.double()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()
