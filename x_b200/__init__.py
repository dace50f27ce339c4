"""x_b200 -- B200-native (sm_100a) implementation of the anchored transport score path of
KAVYANSHTYAGI/x (package ``atl``): a drop-in for ``atl.ops`` (splat / gather / ats_pair_sums /
build_pair_plan / window_counts / voxel_grid) and the anchored objectives built on them.

Kernels live in libatlb200.so (C ABI: include/atl_b200.h, sources: x_b200/csrc/).  Build it with
``python -m x_b200.build``.  There is no CPU path.
"""
from .events import EventPacket
from .functional import (PairPlan, ats_pair_sums, blur, build_pair_plan, gather, gaussian_kernel1d, splat,
                         voxel_grid, window_counts)
from ._ext import ext_supports, get_ext

__all__ = ["EventPacket", "PairPlan", "ats_pair_sums", "blur", "build_pair_plan", "gather", "gaussian_kernel1d",
           "splat", "voxel_grid", "window_counts", "ext_supports", "get_ext"]
