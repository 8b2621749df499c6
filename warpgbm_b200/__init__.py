"""B200-native (sm_100a) implementation of WarpGBM's tree-growing hot path.

``from warpgbm_b200 import WarpGBM`` is a drop-in for ``from warpgbm import
WarpGBM``; ``warpgbm_b200.node_kernel`` is a drop-in for the reference's
``warpgbm.cuda.node_kernel`` extension.  All compute runs in the in-tree
CUDA library libwgb_b200.so (C ABI: include/warpgbm_b200.h).
"""
from .core import WarpGBM

__all__ = ["WarpGBM"]
__version__ = "0.1.0"
