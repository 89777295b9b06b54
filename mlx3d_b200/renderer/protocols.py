"""The renderer convention (src/mlx3d/renderer/protocols.py:32-62).

A renderer is any callable ``renderer(camera, *scene) -> RenderOutput``; the
output dict carries ``image`` (H, W, 3), ``alpha`` (H, W) and optionally
``depth`` (H, W), plus renderer-specific extras read by key.
"""

from __future__ import annotations

from typing import Protocol, TypedDict, runtime_checkable

import torch

from ..cameras import Camera

__all__ = ["RenderOutput", "Renderer"]


class RenderOutput(TypedDict, total=False):
    image: torch.Tensor
    alpha: torch.Tensor
    depth: torch.Tensor


@runtime_checkable
class Renderer(Protocol):
    def __call__(self, camera: Camera, *args: object, **kwargs: object) -> RenderOutput: ...
