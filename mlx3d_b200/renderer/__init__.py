from .protocols import Renderer, RenderOutput

__all__ = ["RenderOutput", "Renderer"]
