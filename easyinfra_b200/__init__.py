"""B200 (sm_100a) expert-parallel MoE layer forward for EasyInfra.

Host code in Python/PyTorch over a C-ABI library of hand-written CUDA kernels
(libb200moe.so, include/b200moe.h): router, permute, grouped tcgen05 SwiGLU/down
GEMMs, combine; dispatch/combine all-to-all over NCCL.  There is no CPU fallback.
"""
from . import _lib, ops  # noqa: F401
from .layer import LayerParams, MoELayer, forward_ep_single_device  # noqa: F401
from .placement import Placement  # noqa: F401

__all__ = ["ops", "MoELayer", "LayerParams", "Placement", "forward_ep_single_device"]
