"""``muon-fsdp`` command line entry point (the reference's public names of src/muon_fsdp/cli.py:12-91)."""
from ..cli import muon_fsdp_main as main

__all__ = ["main"]
