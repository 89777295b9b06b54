"""Gaussian splatting on sm_100a: the drop-in counterpart of ``mlx3d.splatting``."""

from .model import GaussianModel
from .projection import project_gaussians, project_gaussians_ut, quat_scale_to_cov3d
from .rasterize import rasterize, rasterize_depth, rasterize_features
from .render import render_gaussian_depth, render_gaussian_features, render_gaussians
from .sh import eval_sh, num_sh_bases, rgb_to_sh, sh_to_rgb
from .tiles import TILE_SIZE, bin_gaussians
from .trainer import GaussianTrainer, TrainerConfig

__all__ = [
    "GaussianModel",
    "GaussianTrainer",
    "TILE_SIZE",
    "TrainerConfig",
    "bin_gaussians",
    "eval_sh",
    "num_sh_bases",
    "project_gaussians",
    "project_gaussians_ut",
    "quat_scale_to_cov3d",
    "rasterize",
    "rasterize_depth",
    "rasterize_features",
    "render_gaussian_depth",
    "render_gaussian_features",
    "render_gaussians",
    "rgb_to_sh",
    "sh_to_rgb",
]
