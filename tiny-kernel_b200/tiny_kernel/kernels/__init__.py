"""Kernel wrappers, one module per reference file (src/kernels/*.zig)."""
from . import fused, quantized, rmsnorm  # noqa: F401
