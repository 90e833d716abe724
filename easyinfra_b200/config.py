"""Plugin selection mirroring EasyInfra's env-var switches.

get_moe_impl() mirrors easyinfra/generation/modules/moe/config.py:4-15 (MOE_IMPL)
and get_moe_block() mirrors easyinfra/generation/blocks/__init__.py:4-12
(MOE_COMM_MODE) for the implementation this package provides: MOE_IMPL=b200 with
the all-to-all communication mode.
"""
from __future__ import annotations

import os


def get_moe_impl():
    impl = os.getenv("MOE_IMPL", "b200").lower()
    if impl == "b200":
        from .experts import B200MoE
        return B200MoE
    raise ValueError(f"Unrecognized MoE Implementation {impl} (this package provides MOE_IMPL=b200)")


def get_moe_block():
    mode = os.getenv("MOE_COMM_MODE", "all2all")
    if mode == "all2all":
        from .block import B200MoeAll2AllBlock
        return B200MoeAll2AllBlock
    raise ValueError(f"Unsupported moe communication mode {mode} (this package provides all2all)")
