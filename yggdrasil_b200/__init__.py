"""yggdrasil_b200: Yggdrasil's int8 streaming inference step on NVIDIA B200 (sm_100a).

The compute path is libygg_b200.so (hand-written CUDA behind a C-ABI, include/ygg_b200.h); this package is its
Python host side, shaped as the reference's inference API (``Yggdrasil.load(path, backend="b200")``).
"""
from .inference import B200Yggdrasil, Yggdrasil  # noqa: F401

__all__ = ["Yggdrasil", "B200Yggdrasil"]
