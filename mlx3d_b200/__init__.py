"""mlx3d_b200: B200-native (sm_100a) Gaussian-splatting rasterizer with mlx3D's API.

The compute path is the C-ABI library ``_lib/libgsplat_b200.so`` (hand-written
CUDA, see include/gsplat_b200.h); tensors are torch CUDA tensors.
"""

__version__ = "0.1.0"

from . import cameras, losses, renderer, splatting  # noqa: E402
from .cameras import Camera  # noqa: E402

__all__ = ["Camera", "cameras", "losses", "renderer", "splatting", "__version__"]
