"""Test helpers for the Gaussian front end: seeded scenes and a float64 torch
restatement of the forward whose autograd derivative is the oracle of the
CUDA backward.

The restatement follows the same mathematics as oracle/gaussians.py (EWA
splatting; real spherical harmonics of degree 0..3) without its float32
operation order.  Culling (radii == 0) and the colour clamp are taken from the
forward under test, so the two differentiate the same piecewise-smooth function.
"""
import math

import numpy as np
import torch

import vi_workloads as wl

C0 = 0.28209479177387814
C1 = 0.4886025119029199
C2 = (1.0925484305920792, -1.0925484305920792, 0.31539156525252005, -1.0925484305920792, 0.5462742152960396)
C3 = (-0.5900435899266435, 2.890611442640554, -0.4570457994644658, 0.3731763325901154, -0.4570457994644658,
      1.445305721320277, -0.5900435899266435)


def scene(P, sh_degree, seed=0, extent=1.0, mu_scale=-3.0, sigma_scale=0.5, width=128, height=96, fov=60.0,
          dist=4.0, M=None, layout="box"):
    """Seeded Gaussians (CPU float32 tensors) and a camera dict."""
    g = torch.Generator().manual_seed(seed)
    if layout == "box":
        means = (torch.rand(P, 3, generator=g) * 2 - 1) * extent
    else:
        means = wl.mixture(P, 256, extent, g)
    scales = torch.exp(mu_scale + sigma_scale * torch.randn(P, 3, generator=g))
    q = torch.randn(P, 4, generator=g)
    q = q / q.norm(dim=1, keepdim=True) * (0.5 + torch.rand(P, 1, generator=g))  # not unit: normalised inside
    opac = torch.sigmoid(torch.randn(P, 1, generator=g))
    M = M or (sh_degree + 1) ** 2
    shs = 0.2 * torch.randn(P, M, 3, generator=g)
    cam = wl.camera((0.3, -0.2, -dist), width, height, fov)
    return means, scales, q, opac, shs, cam


def sh_eval(d, shs, deg):
    x, y, z = d[:, 0], d[:, 1], d[:, 2]
    Y = [torch.full_like(x, C0)]
    if deg >= 1:
        Y += [-C1 * y, C1 * z, -C1 * x]
    if deg >= 2:
        xx, yy, zz = x * x, y * y, z * z
        Y += [C2[0] * x * y, C2[1] * y * z, C2[2] * (2 * zz - xx - yy), C2[3] * x * z, C2[4] * (xx - yy)]
    if deg >= 3:
        Y += [C3[0] * y * (3 * xx - yy), C3[1] * x * y * z, C3[2] * y * (4 * zz - xx - yy),
              C3[3] * z * (2 * zz - 3 * xx - 3 * yy), C3[4] * x * (4 * zz - xx - yy), C3[5] * z * (xx - yy),
              C3[6] * x * (xx - 3 * yy)]
    return sum(Yk[:, None] * shs[:, k, :] for k, Yk in enumerate(Y)) + 0.5


def forward64(means, scales, rots, shs, cam, sh_degree, scale_modifier, live, clamped):
    """(means2D, depths, cov3D, conic[:, :3], rgb) in float64, differentiable."""
    V = cam["viewmatrix"].double().reshape(16)
    Pm = cam["projmatrix"].double().reshape(16)
    cp = cam["cam_pos"].double().reshape(3)
    W, H = cam["image_width"], cam["image_height"]
    tx_, ty_ = float(np.float32(cam["tanfovx"])), float(np.float32(cam["tanfovy"]))
    fx, fy = W / (2 * tx_), H / (2 * ty_)
    limx, limy = 1.3 * tx_, 1.3 * ty_
    p = means
    t = torch.stack([p[:, 0] * V[r] + p[:, 1] * V[4 + r] + p[:, 2] * V[8 + r] + V[12 + r] for r in range(3)], 1)
    h = torch.stack([p[:, 0] * Pm[r] + p[:, 1] * Pm[4 + r] + p[:, 2] * Pm[8 + r] + Pm[12 + r] for r in (0, 1, 3)], 1)
    pw = 1.0 / (h[:, 2] + 1e-7)
    m2 = torch.stack([((h[:, 0] * pw + 1) * W - 1) * 0.5, ((h[:, 1] * pw + 1) * H - 1) * 0.5], 1)
    qn = rots / rots.norm(dim=1, keepdim=True)
    r, x, y, z = qn.unbind(1)
    R = torch.stack([1 - 2 * (y * y + z * z), 2 * (x * y - r * z), 2 * (x * z + r * y),
                     2 * (x * y + r * z), 1 - 2 * (x * x + z * z), 2 * (y * z - r * x),
                     2 * (x * z - r * y), 2 * (y * z + r * x), 1 - 2 * (x * x + y * y)], 1).view(-1, 3, 3)
    Mm = R * (scale_modifier * scales)[:, None, :]
    Sig = Mm @ Mm.transpose(1, 2)
    iu = [(0, 0), (0, 1), (0, 2), (1, 1), (1, 2), (2, 2)]
    cov3D = torch.stack([Sig[:, a, b] for a, b in iu], 1)
    tz = t[:, 2]
    txc = torch.clamp(t[:, 0] / tz, -limx, limx) * tz
    tyc = torch.clamp(t[:, 1] / tz, -limy, limy) * tz
    zero = torch.zeros_like(tz)
    J = torch.stack([torch.stack([fx / tz, zero, -fx * txc / tz ** 2], 1),
                     torch.stack([zero, fy / tz, -fy * tyc / tz ** 2], 1)], 1)  # [P, 2, 3]
    Wr = torch.stack([V[0:12:4], V[1:12:4], V[2:12:4]], 0)  # rows of the view rotation
    U = J @ Wr
    cov2 = U @ Sig @ U.transpose(1, 2)
    a, b, c = cov2[:, 0, 0] + 0.3, cov2[:, 0, 1], cov2[:, 1, 1] + 0.3
    det = a * c - b * b
    conic = torch.stack([c / det, -b / det, a / det], 1)
    d = p - cp
    d = d / d.norm(dim=1, keepdim=True)
    col = sh_eval(d, shs, sh_degree)
    rgb = torch.where(clamped, torch.zeros_like(col), col)
    lv = live[:, None]
    return (torch.where(lv, m2, 0 * m2), torch.where(live, tz, 0 * tz), torch.where(lv, cov3D, 0 * cov3D),
            torch.where(lv, conic, 0 * conic), torch.where(lv, rgb, 0 * rgb))


def autograd_grads(means, scales, rots, shs, cam, sh_degree, scale_modifier, live, clamped, g_m2, g_d, g_cov, g_con,
                   g_rgb):
    """float64 autograd gradients of <outputs, incoming gradients>."""
    leaves = [x.detach().double().clone().requires_grad_(True) for x in (means, scales, rots, shs)]
    outs = forward64(*leaves, cam, sh_degree, scale_modifier, live, clamped)
    loss = sum((o * gi.double()).sum() for o, gi in zip(outs, (g_m2, g_d, g_cov, g_con, g_rgb)))
    grads = torch.autograd.grad(loss, leaves, allow_unused=True)
    return [gr if gr is not None else torch.zeros_like(l) for gr, l in zip(grads, leaves)]


def rel_close(a, b, rtol=1e-3, atol_frac=1e-4):
    """max |a - b| <= rtol * |b| + atol_frac * max |b| element-wise."""
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    scale = max(float(np.abs(b).max()) if b.size else 0.0, 1e-30)
    ok = np.abs(a - b) <= rtol * np.abs(b) + atol_frac * scale
    return bool(ok.all()), float((np.abs(a - b) / (np.abs(b) + atol_frac * scale)).max()) if b.size else 0.0


def camera_args(cam):
    return dict(viewmatrix=cam["viewmatrix"].numpy(), projmatrix=cam["projmatrix"].numpy(),
                campos=cam["cam_pos"].numpy(), W=cam["image_width"], H=cam["image_height"],
                tanfovx=cam["tanfovx"], tanfovy=cam["tanfovy"])


def fov_of(tan_half):
    return 2 * math.degrees(math.atan(tan_half))
