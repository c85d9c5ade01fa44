"""``fsdp2-utils`` command line entry point (the reference's public names of src/fsdp2_utils/cli.py:9-35)."""
from ..cli import fsdp2_utils_main as main

__all__ = ["main"]
