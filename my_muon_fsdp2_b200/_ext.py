"""Loader for the compiled sm_100a extension (``my_muon_fsdp2_b200/_C*.so``).

The extension is built in-tree by ``python setup.py build_ext --inplace`` (``__graft_entry__.build``).
CUDA code paths call :func:`ext`, which raises a clear error when the extension is missing:
a CUDA tensor is never silently routed to a PyTorch fallback.
"""
from __future__ import annotations

import importlib
from typing import Optional

_EXT = None
_ERR: Optional[BaseException] = None


def ext():
    """Return the compiled extension module, importing it on first use (raises if absent)."""
    global _EXT, _ERR
    if _EXT is not None:
        return _EXT
    try:
        import torch  # noqa: F401  (the extension links against libtorch)

        _EXT = importlib.import_module("my_muon_fsdp2_b200._C")
    except ImportError as e:  # pragma: no cover - depends on build state
        _ERR = e
        raise RuntimeError(
            "my_muon_fsdp2_b200: the native sm_100a extension is not built or failed to load "
            f"({e}). Build it with `python setup.py build_ext --inplace`."
        ) from e
    return _EXT


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def launch_count() -> int:
    """Kernels launched by this library in this process (host-side counter)."""
    return int(ext().launch_count()) if available() else 0


def check_device_error(device: int = 0) -> None:
    """Raise if a bounded wait inside one of our kernels timed out (reads and clears the flag)."""
    code = int(ext().device_error(device))
    if code != 0:
        raise RuntimeError(f"my_muon_fsdp2_b200: device-side wait timed out (error code {code}) on cuda:{device}")
