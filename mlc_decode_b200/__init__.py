"""B200 (sm_100a) absorbed-MLA decode: split-KV decode + LSE combine kernels.

The drop-in module with the reference's public names is ``mla_decode`` at the
repository root; this package holds the C-ABI binding (``capi``), the kernel
object (``decode``), the planner/config table (``plan``) and the multi-GPU
partitioning (``dist``).
"""
from .decode import MlaDecodeKernel, MlaPagedDecodeKernel, combine  # noqa: F401

__all__ = ["MlaDecodeKernel", "MlaPagedDecodeKernel", "combine"]
