"""Version strings: the package, and the two API namespaces it mirrors."""
__version__ = "0.1.0"
FSDP2_UTILS_VERSION = "0.2.0"
