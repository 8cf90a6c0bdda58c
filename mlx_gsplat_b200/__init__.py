"""B200-native (sm_100a) training hot path of 3D Gaussian Splatting with the
reference's Python API (mlx_gsplat/__init__.py): the allocator, the fused
Adam, the cull and the differentiable rasterizer keep their names.

Importing the package needs no GPU; every compute call goes to
``libgsplat_b200.so`` (built by ``python -m mlx_gsplat_b200.build``) and
fails loudly without it.
"""
from .allocator import PointerStableChunkedAllocator
from .dataset import Dataset, Parser
from .optimizer import FusedMLXAdam
from .rendering import RasterSettings, bilinear_resize_mlx, frustum_culling_mlx, rasterize_gaussians_mlx

__all__ = [
    "PointerStableChunkedAllocator",
    "FusedMLXAdam",
    "frustum_culling_mlx",
    "rasterize_gaussians_mlx",
    "bilinear_resize_mlx",
    "RasterSettings",
    "Parser",
    "Dataset",
]
