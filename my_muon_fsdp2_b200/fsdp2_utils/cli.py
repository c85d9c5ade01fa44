"""``fsdp2-utils`` command line entry point."""
from ..cli import fsdp2_utils_main as main

__all__ = ["main"]
