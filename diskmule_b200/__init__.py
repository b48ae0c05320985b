"""diskmule_b200 -- a B200 (sm_100a) implementation of DiskMule's routed-expert path.

The product is the CUDA shared library `libdiskmule_cuda.so` (C ABI in
include/diskmule_cuda.h). This package is its host-side mirror: `CudaContext`
mirrors the reference's `MetalContext`, `MoeLayer` the batched MoE block.
"""
from ._native import DmError, lib  # noqa: F401
from .moe import Buffer, CudaContext, MoeLayer  # noqa: F401

__all__ = ["Buffer", "CudaContext", "DmError", "MoeLayer", "lib"]
