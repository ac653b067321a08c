"""beatlm-b200: a B200 (sm_100a) backend for beatlm's ViT attention hot path.

The compute runs in ``libbeatlm_b200.so`` (hand-written tcgen05/TMA kernels
behind the C ABI of ``include/beatlm_b200.h``); this package is the host-side
mirror of the reference's operator interface for that path. There is no CPU
or PyTorch fallback: when the library is missing every op raises.
"""
from ._native import BackendError, BL_BF16, BL_F16, BL_F32, lib, status  # noqa: F401
from .ops import attention, pack_qkv  # noqa: F401

__all__ = ["attention", "pack_qkv", "status", "BackendError", "lib"]
