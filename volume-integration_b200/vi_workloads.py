"""Seeded synthetic workloads with the shapes of the renderer's benchmark scenes.

There is no dataset: every scene is drawn from a fixed seed.  The mapping of a
scene description onto the renderer's real inputs is:

* primitive centres   -> ``means3D`` (uniform box or a mixture of anisotropic clusters);
* median cube scale   -> the single ``primitive_scale`` (6 x the log-normal median,
  i.e. +-3 sigma of the footprint), because every primitive shares one edge length;
* opacity-logit mean  -> mean of the confidence grids, ``conf ~ N(mu, 1)``;
* hashgrid            -> ``res_l = floor(base * growth**l)``, a level is hashed when
  ``(res_l + 1)**3 > T``, primes (1, 2654435761, 805459861) as int32 bit patterns;
* linear layer        -> ``W, b ~ U(+-1/sqrt(D))`` with ``W`` laid out ``[O][D]``.

Cameras follow the convention the kernels read (``auxiliary.h:67-86`` of the
reference): ``viewmatrix`` is world->view transposed, ``projmatrix`` is
(proj @ view) transposed, both stored row-major, view-space +z in front.
"""
import math

import torch

PRIMES = (1, 2654435761, 805459861)


def _i32(v):
    return v - (1 << 32) if v >= (1 << 31) else v


def hashgrid(levels, feats, log2_T, base, growth):
    T = 1 << log2_T
    res = [int(math.floor(base * growth ** l)) for l in range(levels)]
    do_hash = [1 if (r + 1) ** 3 > T else 0 for r in res]
    return dict(
        resolution=torch.tensor(res, dtype=torch.int32),
        do_hash=torch.tensor(do_hash, dtype=torch.int32),
        primes=torch.tensor([_i32(p) for p in PRIMES], dtype=torch.int32),
        feature_offset=T,
        hashgrid_levels=levels,
        input_feature_dim=feats,
        intermediate_feature_dim=levels * feats,
    )


def perspective(znear, zfar, tan_x, tan_y):
    top, right = tan_y * znear, tan_x * znear
    P = torch.zeros(4, 4, dtype=torch.float64)
    P[0, 0] = 2.0 * znear / (2 * right)
    P[1, 1] = 2.0 * znear / (2 * top)
    P[3, 2] = 1.0
    P[2, 2] = zfar / (zfar - znear)
    P[2, 3] = -(zfar * znear) / (zfar - znear)
    return P


def look_at(eye, target=(0.0, 0.0, 0.0), up=(0.0, 1.0, 0.0)):
    """World->camera 4x4 (camera +z forward, +x right, +y down)."""
    eye = torch.tensor(eye, dtype=torch.float64)
    fwd = torch.tensor(target, dtype=torch.float64) - eye
    fwd = fwd / fwd.norm()
    upv = torch.tensor(up, dtype=torch.float64)
    if abs(float(fwd @ upv)) > 0.999:
        upv = torch.tensor((0.0, 0.0, 1.0), dtype=torch.float64)
    right = torch.linalg.cross(fwd, -upv)
    right = right / right.norm()
    down = torch.linalg.cross(fwd, right)
    M = torch.eye(4, dtype=torch.float64)
    M[0, :3], M[1, :3], M[2, :3] = right, down, fwd
    M[:3, 3] = -M[:3, :3] @ eye
    return M


def camera(eye, width, height, fov_y_deg, znear=0.01, zfar=100.0, target=(0.0, 0.0, 0.0)):
    tan_y = math.tan(math.radians(fov_y_deg) / 2)
    tan_x = tan_y * width / height
    V = look_at(eye, target)
    P = perspective(znear, zfar, tan_x, tan_y)
    return dict(
        viewmatrix=V.t().contiguous().float(),
        projmatrix=(P @ V).t().contiguous().float(),
        cam_pos=torch.tensor(eye, dtype=torch.float32),
        tanfovx=tan_x, tanfovy=tan_y, image_width=width, image_height=height,
    )


def orbit(n, radius, width, height, fov_y_deg, elevation_deg=20.0, seed=0):
    """n cameras on a circle of the given radius, all looking at the origin."""
    out = []
    el = math.radians(elevation_deg)
    for i in range(n):
        a = 2 * math.pi * i / n + 0.1 * seed
        eye = (radius * math.cos(el) * math.cos(a), -radius * math.sin(el), radius * math.cos(el) * math.sin(a))
        out.append(camera(eye, width, height, fov_y_deg))
    return out


def sphere_cameras(n, radius, width, height, fov_y_deg, gen):
    out = []
    for _ in range(n):
        v = torch.randn(3, generator=gen, dtype=torch.float64)
        v = v / v.norm() * radius
        out.append(camera(tuple(v.tolist()), width, height, fov_y_deg))
    return out


def mixture(P, clusters, extent, gen):
    """Centres from a mixture of anisotropic Gaussian clusters clipped to [-extent, extent]^3."""
    centers = (torch.rand(clusters, 3, generator=gen) * 2 - 1) * 0.8 * extent
    sig = (0.02 + 0.13 * torch.rand(clusters, 3, generator=gen)) * extent
    q = torch.randn(clusters, 4, generator=gen)
    q = q / q.norm(dim=1, keepdim=True)
    w, x, y, z = q.unbind(1)
    Rm = torch.stack([
        1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
        2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
        2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], 1).view(clusters, 3, 3)
    idx = torch.randint(0, clusters, (P,), generator=gen)
    local = torch.randn(P, 3, generator=gen) * sig[idx]
    pts = centers[idx] + torch.einsum("pij,pj->pi", Rm[idx], local)
    return pts.clamp(-extent, extent).contiguous()


def linear_layer(D, O, gen):
    bound = 1.0 / math.sqrt(max(D, 1))
    W = (torch.rand(O * D, generator=gen) * 2 - 1) * bound
    b = (torch.rand(O, generator=gen) * 2 - 1) * bound
    return W, b


# name -> description of the scene (shapes and distributions of the benchmark configs)
CONFIGS = {
    "tiny": dict(P=4096, layout="box", extent=1.0, mu_scale=-3.0, mu_conf=0.0, width=128, height=128,
                 fov=60.0, dist=4.0, views=1, L=4, F=2, log2_T=14, base=16, growth=2.0),
    "mid": dict(P=100_000, layout="mix", clusters=32, extent=3.0, mu_scale=-4.5, mu_conf=0.0,
                width=800, height=800, fov=50.0, dist=5.0, views=8, L=16, F=2, log2_T=19, base=16,
                growth=1.447),
    "headline": dict(P=1_000_000, layout="mix", clusters=256, extent=10.0, mu_scale=-5.0, mu_conf=0.0,
                     width=1920, height=1080, fov=50.0, dist=12.0, views=1, L=16, F=2, log2_T=19,
                     base=16, growth=1.447),
    # the headline scene and camera with a quarter of the primitives (profiling case)
    "headline_q": dict(P=250_000, layout="mix", clusters=256, extent=10.0, mu_scale=-5.0, mu_conf=0.0,
                       width=1920, height=1080, fov=50.0, dist=12.0, views=1, L=16, F=2, log2_T=19,
                       base=16, growth=1.447),
    "multiview": dict(P=3_000_000, layout="mix", clusters=256, extent=10.0, mu_scale=-5.0, mu_conf=0.0,
                      width=1920, height=1080, fov=50.0, dist=12.0, views=32, L=16, F=2, log2_T=19,
                      base=16, growth=1.447),
    "stress": dict(P=6_000_000, layout="mix", clusters=256, extent=10.0, mu_scale=-3.0, mu_conf=1.0,
                   width=3840, height=2160, fov=50.0, dist=14.0, views=1, L=16, F=4, log2_T=21,
                   base=16, growth=1.447),
}
SEEDS = {"tiny": 1000, "mid": 1001, "headline": 1002, "multiview": 1003, "stress": 1004, "headline_q": 1002}


def make(name, table_range=1e-4, seed=None, **over):
    """Returns (means3D, confidences, settings_kwargs, cameras) on the CPU.

    ``settings_kwargs`` holds every ``IntegrationSettings`` field except the camera,
    which comes from one entry of ``cameras``.
    """
    c = dict(CONFIGS[name])
    c.update(over)
    gen = torch.Generator().manual_seed(SEEDS.get(name, 999) if seed is None else seed)
    P, G = c["P"], 3
    if c["layout"] == "box":
        means = (torch.rand(P, 3, generator=gen) * 2 - 1) * c["extent"]
    else:
        means = mixture(P, c["clusters"], c["extent"], gen)
    conf = torch.randn(P, G ** 3, generator=gen) + c["mu_conf"]
    hg = hashgrid(c["L"], c["F"], c["log2_T"], c["base"], c["growth"])
    D, Fout = c["L"] * c["F"], 4
    O = 3 + Fout + 1
    table = (torch.rand(hg["feature_offset"] * c["L"] * c["F"], generator=gen) * 2 - 1) * table_range
    W, b = linear_layer(D, O, gen)
    if c["views"] == 1:
        cams = [camera((0.0, 0.0, -c["dist"]), c["width"], c["height"], c["fov"])]
    elif name == "mid":
        cams = sphere_cameras(c["views"], c["dist"], c["width"], c["height"], c["fov"], gen)
    else:
        cams = orbit(c["views"], c["dist"], c["width"], c["height"], c["fov"])
    kw = dict(
        near_plane=0.01, max_distance=100.0,
        primitive_scale=6.0 * math.exp(c["mu_scale"]),
        feature_table=table, linear_weights=W, linear_bias=b,
        stencil_genus=1, grid_size=G, max_primitives_per_ray=64, occupancy_threshold=0.5,
        bg_color=torch.zeros(3), output_feature_dim=Fout, num_output_channels=3, debug=False,
    )
    kw.update({k: v for k, v in hg.items()})
    return means, conf, kw, cams


def gaussians(name="headline", seed=None, sh_degree=3):
    """Seeded Gaussian attributes of a scene's shape (the Gaussian front end's workload).

    Centres as ``make(name)``; log-normal scales per axis (mu = the scene's
    mu_scale, sigma 0.7); random unit quaternions (r, x, y, z); opacity
    sigmoid(N(0, 1)); SH coefficients N(0, 0.2) of the given degree.  Returns
    (means3D, scales, rotations, opacities [P, 1], shs [P, (deg+1)^2, 3], camera).
    """
    c = dict(CONFIGS[name])
    gen = torch.Generator().manual_seed((SEEDS.get(name, 999) if seed is None else seed) + 7)
    P = c["P"]
    if c["layout"] == "box":
        means = (torch.rand(P, 3, generator=gen) * 2 - 1) * c["extent"]
    else:
        means = mixture(P, c["clusters"], c["extent"], gen)
    scales = torch.exp(c["mu_scale"] + 0.7 * torch.randn(P, 3, generator=gen))
    q = torch.randn(P, 4, generator=gen)
    q = q / q.norm(dim=1, keepdim=True)
    opac = torch.sigmoid(torch.randn(P, 1, generator=gen))
    shs = 0.2 * torch.randn(P, (sh_degree + 1) ** 2, 3, generator=gen)
    cam = camera((0.0, 0.0, -c["dist"]), c["width"], c["height"], c["fov"])
    return means, scales, q, opac, shs, cam
