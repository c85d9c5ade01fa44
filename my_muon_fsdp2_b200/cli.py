"""Command line interfaces: ``muon-fsdp info [-v] | check [--full]`` and ``fsdp2-utils --info``.

Parity with ``src/muon_fsdp/cli.py:12-91`` and ``src/fsdp2_utils/cli.py:9-35``; ``check`` also
reports whether the sm_100a extension is built and whether a Blackwell GPU is visible.
"""
from __future__ import annotations

import argparse
import sys

from .version import FSDP2_UTILS_VERSION, __version__


def muon_fsdp_main(argv=None) -> int:
    parser = argparse.ArgumentParser(prog="muon-fsdp", description="Muon optimizer with FSDP2 support (B200-native)")
    parser.add_argument("--version", action="version", version=f"%(prog)s {__version__}")
    sub = parser.add_subparsers(dest="command")
    info = sub.add_parser("info", help="show package information")
    info.add_argument("--verbose", "-v", action="store_true")
    check = sub.add_parser("check", help="check installation and dependencies")
    check.add_argument("--full", action="store_true", help="also run a small optimizer step")
    sub.add_parser("configs", help="list the benchmark workloads and the commands that measure them")
    args = parser.parse_args(argv)
    import torch

    if args.command == "info":
        print(f"muon-fsdp version: {__version__}")
        print(f"Python version: {sys.version}")
        print(f"PyTorch version: {torch.__version__}")
        if args.verbose:
            print("\nAvailable components:")
            for line in ("MuonOptimizer", "FSDPMuonOptimizer", "HDSPMuonOptimizer", "SpectralSphereOptimizer",
                         "HybridMuonAdamW", "Newton-Schulz (tcgen05 chain on sm_100a)",
                         "distributed primitives (NCCL / symmetric-memory P2P)"):
                print(f"  - {line}")
        return 0
    if args.command == "configs":
        from .configs import WORKLOADS

        for w in WORKLOADS.values():
            print(f"{w.name}: {w.model}\n  gpus: {w.gpus}; dtype: {w.dtype}; batch/GPU: {w.batch_per_gpu}\n"
                  f"  optimizer: {w.optimizer}\n  run: {w.command}")
        return 0
    if args.command == "check":
        print(f"OK PyTorch {torch.__version__}")
        try:
            from . import FSDPMuonOptimizer, MuonOptimizer  # noqa: F401
            from .ops.newton_schulz import zeropower_via_newtonschulz5  # noqa: F401

            print("OK muon-fsdp components import")
        except ImportError as e:
            print(f"FAIL import: {e}")
            return 1
        from ._ext import available

        print(("OK" if available() else "MISSING") + " native sm_100a extension")
        if torch.cuda.is_available():
            cap = torch.cuda.get_device_capability()
            print(f"GPU: {torch.cuda.get_device_name()} (sm_{cap[0]}{cap[1]})")
        if args.full:
            from . import MuonOptimizer

            m = torch.nn.Linear(128, 128)
            opt = MuonOptimizer(m.parameters(), lr=0.01)
            m(torch.randn(4, 128)).sum().backward()
            opt.step()
            print("OK MuonOptimizer step")
        print("\nAll checks passed!")
        return 0
    parser.print_help()
    return 0


def fsdp2_utils_main(argv=None) -> int:
    parser = argparse.ArgumentParser(prog="fsdp2-utils", description="FSDP2 utilities (B200-native)")
    parser.add_argument("--version", "-v", action="version", version=f"%(prog)s {FSDP2_UTILS_VERSION}")
    parser.add_argument("--info", action="store_true", help="show package information")
    args = parser.parse_args(argv)
    if args.info:
        print("FSDP2 utilities")
        print(f"version: {FSDP2_UTILS_VERSION}")
        print("description: DTensor / collective helpers and FSDP2-aware optimizers")
        return 0
    parser.print_help()
    return 0


if __name__ == "__main__":  # pragma: no cover
    sys.exit(muon_fsdp_main())
