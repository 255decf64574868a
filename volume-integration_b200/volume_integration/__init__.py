"""Differentiable tile-binned volume integration on B200 (sm_100a).

Drop-in for the reference package of the same name (reference
``volume_integration/__init__.py``): the same ``IntegrationSettings`` fields and
defaults (``:27-64``), the same autograd Function contract (``:66-344``) and the
same ``VolumeIntegrator`` module (``:346-389``).  All work runs in the compiled
extension ``_C`` over ``libvi_b200.so``; importing fails loudly if it is absent.
"""
from dataclasses import dataclass, field
from typing import Optional, Sequence

import torch
import torch.nn as nn
from torch.autograd import Function

try:
    from . import _C
except ImportError as e:  # no silent fallback: the CUDA extension is the product
    raise ImportError(
        "volume_integration._C is not built; run `python volume-integration_b200/build.py` "
        "(or __graft_entry__.build()) first") from e

__all__ = ["IntegrationSettings", "VolumeIntegrator", "integrate_primitives"]


@dataclass
class IntegrationSettings:
    # camera
    viewmatrix: torch.Tensor = field(default_factory=lambda: torch.eye(4))
    projmatrix: torch.Tensor = field(default_factory=lambda: torch.eye(4))
    cam_pos: torch.Tensor = field(default_factory=lambda: torch.zeros(3))
    tanfovx: float = 1.0
    tanfovy: float = 1.0
    image_height: int = 512
    image_width: int = 512
    near_plane: float = 0.1
    max_distance: float = 100.0
    # primitives: axis-aligned cubes sharing one edge length
    primitive_scale: float = 0.01
    # hashgrid: flat table laid out [entry][level][feature]
    feature_table: torch.Tensor = field(default_factory=lambda: torch.empty(0))
    resolution: torch.Tensor = field(default_factory=lambda: torch.empty(0, dtype=torch.int32))
    do_hash: torch.Tensor = field(default_factory=lambda: torch.empty(0, dtype=torch.int32))
    primes: torch.Tensor = field(default_factory=lambda: torch.empty(0, dtype=torch.int32))
    feature_offset: int = 0  # entries per level (T)
    # linear layer: weights [O][D] flat, bias [O]
    linear_weights: torch.Tensor = field(default_factory=lambda: torch.empty(0))
    linear_bias: torch.Tensor = field(default_factory=lambda: torch.empty(0))
    # integration
    stencil_genus: int = 1
    grid_size: int = 3
    max_primitives_per_ray: int = 64
    occupancy_threshold: float = 0.5
    bg_color: torch.Tensor = field(default_factory=lambda: torch.zeros(3))
    # dimensions
    input_feature_dim: int = 2
    output_feature_dim: int = 8
    intermediate_feature_dim: int = 32
    hashgrid_levels: int = 16
    num_output_channels: int = 3
    debug: bool = False
    # Extension (no counterpart in the reference, which fixes the hashgrid box
    # at [-1.3, 1.3]^3, hashgrid.h:23-24): (lo_x, lo_y, lo_z, hi_x, hi_y, hi_z)
    # of the box positions are normalised to, or None for the reference's box.
    hash_bounds: Optional[Sequence[float]] = None
    # Extension: when True the backward is the derivative of the forward
    # (including dL/dmeans3D and dL/dvisibility_info) instead of the reference's
    # formula, which is not (no transmittance factor, another occupancy, no
    # delta-t terms).  Off by default: the reference's gradients.
    exact_gradients: bool = False


def _flat_confidences(conf, P, G):
    """(P, G, G, G) or (P, G^3) -> (P, G^3); returns (flat, original 4-D shape or None)."""
    if conf.dim() == 4:
        assert conf.shape[0] == P, f"Primitive count mismatch: means3D ({P}) vs confidences ({conf.shape[0]})"
        assert tuple(conf.shape[1:]) == (G, G, G), \
            f"Confidence grid dimensions mismatch: expected {G}, got {tuple(conf.shape[1:])}"
        return conf.reshape(P, -1).contiguous(), conf.shape
    if conf.dim() == 2:
        assert conf.shape[0] == P, f"Primitive count mismatch: means3D ({P}) vs confidences ({conf.shape[0]})"
        assert conf.shape[1] == G ** 3, \
            f"Confidence grid flat dimension mismatch: expected {G ** 3}, got {conf.shape[1]}"
        return conf, None
    raise ValueError(f"primitive_confidences has unexpected shape: {conf.shape}")


def _hash_bounds(s):
    """The settings' hashgrid box as 6 floats, or None for the reference's fixed box."""
    hb = getattr(s, "hash_bounds", None)
    if hb is None:
        return None
    vals = [float(v) for v in (hb.flatten().tolist() if isinstance(hb, torch.Tensor) else hb)]
    if len(vals) != 6:
        raise ValueError(f"hash_bounds needs 6 values (lo xyz, hi xyz), got {len(vals)}")
    return vals


def _flags(s):
    return int(_C.FLAG_EXACT_GRADIENTS) if getattr(s, "exact_gradients", False) else 0


class _IntegratePrimitives(Function):
    @staticmethod
    def forward(ctx, means3D, primitive_confidences, feature_table, linear_weights, linear_bias,
                integration_settings):
        s = integration_settings
        means3D = means3D.contiguous().float()
        primitive_confidences = primitive_confidences.contiguous().float()
        feature_table = feature_table.contiguous().float()
        linear_weights = linear_weights.contiguous().float()
        linear_bias = linear_bias.contiguous().float()
        conf_flat, conf_shape = _flat_confidences(primitive_confidences, means3D.shape[0], s.grid_size)

        resolution = s.resolution.contiguous().int()
        do_hash = s.do_hash.contiguous().int()
        primes = s.primes.contiguous().int()
        bg_color = s.bg_color.contiguous().float()
        viewmatrix = s.viewmatrix.contiguous().float()
        projmatrix = s.projmatrix.contiguous().float()
        cam_pos = s.cam_pos
        if not isinstance(cam_pos, torch.Tensor):
            raise TypeError(f"cam_pos must be a torch.Tensor, got {type(cam_pos)}")
        if not cam_pos.is_cuda:
            raise TypeError(f"cam_pos must be a CUDA tensor, but device is {cam_pos.device}")
        if cam_pos.numel() < 3:
            raise ValueError(f"cam_pos must have at least 3 elements, but has shape {cam_pos.shape}")
        cam_pos = cam_pos.contiguous().float()

        args = (means3D, conf_flat, s.primitive_scale, viewmatrix, projmatrix, cam_pos, s.tanfovx, s.tanfovy,
                s.image_height, s.image_width, s.near_plane, s.max_distance, feature_table, resolution, do_hash,
                primes, s.feature_offset, linear_weights, linear_bias, s.stencil_genus, s.grid_size,
                s.max_primitives_per_ray, s.occupancy_threshold, bg_color, s.input_feature_dim,
                s.output_feature_dim, s.intermediate_feature_dim, s.hashgrid_levels, s.num_output_channels,
                s.debug)
        hb, flags = _hash_bounds(s), _flags(s)
        if hb is None and not flags:
            res = _C.integrate_primitives(*args)
        else:
            res = _C.integrate_primitives_ex(*args, hb or [], flags)
        num_rendered, out_color, out_features, visibility_info, geom, binning, img = res

        ctx.save_for_backward(means3D, conf_flat, feature_table, linear_weights, linear_bias, viewmatrix,
                              projmatrix, cam_pos, resolution, do_hash, primes, bg_color, geom, binning, img,
                              visibility_info)
        ctx.integration_settings = s
        ctx.num_rendered = num_rendered
        ctx.original_confidences_shape = conf_shape
        return out_color, out_features, visibility_info

    @staticmethod
    def backward(ctx, grad_out_color, grad_out_features, grad_out_visibility):
        (means3D, conf_flat, feature_table, linear_weights, linear_bias, viewmatrix, projmatrix, cam_pos,
         resolution, do_hash, primes, bg_color, geom, binning, img, _visibility) = ctx.saved_tensors
        s = ctx.integration_settings
        needs = ctx.needs_input_grad
        if not any(needs[:5]):
            return (None, None, None, None, None, None)
        args = (grad_out_color.contiguous(), grad_out_features.contiguous(), geom, binning, img, means3D,
                conf_flat, s.primitive_scale, viewmatrix, projmatrix, cam_pos, s.tanfovx, s.tanfovy,
                s.image_height, s.image_width, s.near_plane, s.max_distance, feature_table, resolution, do_hash,
                primes, s.feature_offset, linear_weights, linear_bias, s.stencil_genus, s.grid_size,
                s.max_primitives_per_ray, s.occupancy_threshold, bg_color, s.input_feature_dim,
                s.output_feature_dim, s.hashgrid_levels, s.num_output_channels, feature_table.numel(),
                means3D.shape[0], ctx.num_rendered, s.debug)
        hb, flags = _hash_bounds(s), _flags(s)
        if hb is None and not flags:
            dmeans, dconf, dtable, dW, db = _C.integrate_primitives_backward(*args)
        else:
            gv = grad_out_visibility if (flags and grad_out_visibility is not None) else torch.empty(0)
            dmeans, dconf, dtable, dW, db = _C.integrate_primitives_backward_ex(*args, hb or [], flags,
                                                                                gv.contiguous())
        if ctx.original_confidences_shape is not None:
            dconf = dconf.view(ctx.original_confidences_shape)
        return (dmeans if needs[0] else None, dconf if needs[1] else None, dtable if needs[2] else None,
                dW if needs[3] else None, db if needs[4] else None, None)


def integrate_primitives(means3D, primitive_confidences, feature_table, linear_weights, linear_bias,
                         integration_settings):
    """Functional form of ``VolumeIntegrator.forward``: (out_color, out_features, visibility)."""
    return _IntegratePrimitives.apply(means3D, primitive_confidences, feature_table, linear_weights,
                                      linear_bias, integration_settings)


class VolumeIntegrator(nn.Module):
    def __init__(self, integration_settings: IntegrationSettings):
        super().__init__()
        self.integration_settings = integration_settings

    def markVisible(self, positions):
        """bool[P]: view-space z > 0.2 (the reference's frustum test)."""
        with torch.no_grad():
            s = self.integration_settings
            return _C.mark_visible(positions.contiguous().float(), s.viewmatrix.contiguous().float(),
                                   s.projmatrix.contiguous().float())

    def forward(self, means3D, primitive_confidences):
        s = self.integration_settings
        return _IntegratePrimitives.apply(means3D, primitive_confidences, s.feature_table, s.linear_weights,
                                          s.linear_bias, s)
