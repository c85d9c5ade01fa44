"""``muon-fsdp`` command line entry point."""
from ..cli import muon_fsdp_main as main

__all__ = ["main"]
