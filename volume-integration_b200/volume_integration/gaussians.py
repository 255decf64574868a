"""Gaussian-attribute front end (extension; no counterpart in the reference).

The reference renderer's primitives are cubes of one fixed world size, projected
by centre and bounding radius only (cuda_integrator/forward.cu:82-87, :100-102 of
the reference).  This module adds the standard per-Gaussian front end of
splatting on the same CUDA library:

* ``preprocess_gaussians``: projection, 3D covariance from scale and rotation,
  2D covariance (EWA, with the 0.3 pixel low-pass), conic, screen radius and
  tiles touched, and colour from real spherical harmonics of degree 0..3, as a
  differentiable function (the backward is the exact derivative);
* ``bin_gaussians``: the tile binning of the projected Gaussians, a point list
  sorted by (tile, depth, index) and per-tile ranges, as the reference renderer
  bins its primitives (integrator_impl.cu:106-178).

There is no CPU fallback: without the CUDA library the import fails.
"""
from dataclasses import dataclass
from typing import NamedTuple

import torch

from . import _C


@dataclass
class GaussianCamera:
    """Camera of the Gaussian front end, in the renderer's conventions.

    ``viewmatrix`` is world->view transposed and ``projmatrix`` is
    (proj @ view) transposed, both stored row-major (as ``IntegrationSettings``);
    ``campos`` is the camera centre, kept on the host (the kernels take it by
    value, so a device tensor is copied once here rather than at every call).
    """
    image_height: int
    image_width: int
    tanfovx: float
    tanfovy: float
    viewmatrix: torch.Tensor
    projmatrix: torch.Tensor
    campos: torch.Tensor
    sh_degree: int = 3
    scale_modifier: float = 1.0
    near_plane: float = 0.2

    def __post_init__(self):
        self.campos = torch.as_tensor(self.campos).detach().to("cpu", torch.float32).reshape(3)


class ProjectedGaussians(NamedTuple):
    radii: torch.Tensor          # [P] int32, 0 = culled
    means2D: torch.Tensor        # [P, 2] pixel coordinates
    depths: torch.Tensor         # [P] view-space z
    cov3D: torch.Tensor          # [P, 6] xx, xy, xz, yy, yz, zz
    conic_opacity: torch.Tensor  # [P, 4] inverse 2D covariance (a, b, c) and opacity
    rgb: torch.Tensor            # [P, 3]
    tiles_touched: torch.Tensor  # [P] int32


class _PreprocessGaussians(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means3D, scales, rotations, opacities, shs, cam):
        op = opacities.reshape(-1)
        radii, means2D, depths, cov3D, conic, rgb, clamped, tiles = _C.preprocess_gaussians(
            means3D, scales, rotations, op, shs, cam.sh_degree, cam.scale_modifier, cam.viewmatrix,
            cam.projmatrix, cam.campos, cam.image_width, cam.image_height, cam.tanfovx, cam.tanfovy,
            cam.near_plane)
        ctx.cam = cam
        ctx.op_shape = opacities.shape
        ctx.save_for_backward(means3D, scales, rotations, shs, radii, clamped)
        ctx.mark_non_differentiable(radii, tiles)
        return radii, means2D, depths, cov3D, conic, rgb, tiles

    @staticmethod
    def backward(ctx, g_radii, g_means2D, g_depths, g_cov3D, g_conic, g_rgb, g_tiles):
        cam = ctx.cam
        means3D, scales, rotations, shs, radii, clamped = ctx.saved_tensors
        P = means3D.shape[0]

        def grad(g, *shape):
            return torch.zeros(*shape, device=means3D.device) if g is None else g.contiguous()
        gm2, gd = grad(g_means2D, P, 2), grad(g_depths, P)
        gcov, gco, grgb = grad(g_cov3D, P, 6), grad(g_conic, P, 4), grad(g_rgb, P, 3)
        dm, ds, dq, dsh = _C.preprocess_gaussians_backward(
            means3D, scales, rotations, shs, cam.sh_degree, cam.scale_modifier, cam.viewmatrix, cam.projmatrix,
            cam.campos, cam.image_width, cam.image_height, cam.tanfovx, cam.tanfovy, cam.near_plane, radii,
            clamped, gm2, gd, gcov, gco, grgb)
        dop = torch.where(radii > 0, gco[:, 3], torch.zeros_like(gco[:, 3])).reshape(ctx.op_shape)
        return dm, ds, dq, dop, dsh, None


def preprocess_gaussians(means3D, scales, rotations, opacities, shs, cam: GaussianCamera) -> ProjectedGaussians:
    """Per-Gaussian projection, covariances, conic, radius, tiles touched and colour.

    means3D, scales: [P, 3]; rotations: [P, 4] quaternions (r, x, y, z), normalised
    inside; opacities: [P] or [P, 1] (passed through as conic_opacity[:, 3]);
    shs: [P, M, 3] with (sh_degree + 1)^2 <= M <= 16.  Gradients flow to every
    float input from means2D, depths, cov3D, conic_opacity and rgb.
    """
    return ProjectedGaussians(*_PreprocessGaussians.apply(means3D, scales, rotations, opacities, shs, cam))


class GaussianBins(NamedTuple):
    point_list: torch.Tensor  # [R] int32 Gaussian ids, sorted by (tile, depth, index)
    tile_ids: torch.Tensor    # [R] int32 tile of each entry
    ranges: torch.Tensor      # [tiles, 2] int32 [start, end) of each tile in point_list


def bin_gaussians(proj: ProjectedGaussians, image_width: int, image_height: int) -> GaussianBins:
    """Tile binning of projected Gaussians (16x16 tiles, row-major tile ids)."""
    pl, tiles, ranges = _C.bin_gaussians(proj.radii, proj.means2D.detach(), proj.depths.detach(),
                                         proj.tiles_touched, image_width, image_height)
    return GaussianBins(pl, tiles, ranges)
