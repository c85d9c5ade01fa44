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


_ERROR_TEXT = {
    1: "a TMA producer's wait for a free stage timed out",
    2: "the MMA issuer's wait for loaded operands timed out",
    3: "the MMA issuer's wait for a free accumulator timed out",
    4: "the epilogue's wait for a finished accumulator timed out",
    5: "a wait on a peer's flag or barrier timed out",
    6: "a kernel rejected its arguments",
    7: "debug check: a TMA innermost coordinate is not on a 16-byte boundary",
    8: "debug check: an index is outside its buffer or segment table",
}


def device_checks() -> bool:
    """True when the extension was built with the device-side debug checks (MMF_DEVICE_CHECKS=1)."""
    return bool(ext().device_checks())


def check_device_error(device: int = 0) -> None:
    """Raise if one of our kernels recorded an error: a bounded wait that timed out, or (debug
    builds) a failed device-side check.  Reads and clears the error word."""
    code = int(ext().device_error(device))
    if code != 0:
        what = _ERROR_TEXT.get(code, "unknown error")
        raise RuntimeError(f"my_muon_fsdp2_b200: device error code {code} on cuda:{device}: {what}")
