from .protocols import Renderer, RenderOutput
from .rasterizer import Fragments, interpolate_face_attributes, rasterize_meshes

__all__ = ["Fragments", "RenderOutput", "Renderer", "interpolate_face_attributes", "rasterize_meshes"]
