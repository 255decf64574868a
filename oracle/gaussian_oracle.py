"""CPU restatement of the Gaussian-attribute front end -- test infrastructure.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU baseline import this
module; the product library never does.

The reference has no Gaussian front end (its primitives are cubes:
``cuda_integrator/forward.cu:82-87``, ``:100-102``), so this restatement follows
the published mathematics (EWA splatting, Zwicker et al. 2001; 3D Gaussian
splatting, Kerbl et al. 2023) in the operation order the CUDA kernels use,
with every operation rounded to float32 (numpy evaluates each operator
separately, with no fused multiply-add), so radii, tile counts and every float
output are reproduced bit for bit.  The conversions that the cube renderer
copies from the reference are shared: ``transformPoint4x3/4x4`` order
(``auxiliary.h:67-86``), ``ndc2Pix`` in double (``auxiliary.h:50-53``) and
``getRect`` (``auxiliary.h:55-65``).

``preprocess`` returns the outputs of ``vi_preprocess_gaussians``; ``binning``
those of ``vi_bin_gaussians`` (a stable sort of tile << 32 | depth bits, as the
reference renderer's duplicateWithKeys + radix sort, ``integrator_impl.cu:106-178``).
"""
import numpy as np

f32 = np.float32
C0 = f32(0.28209479177387814)
C1 = f32(0.4886025119029199)
C2 = [f32(v) for v in (1.0925484305920792, -1.0925484305920792, 0.31539156525252005, -1.0925484305920792,
                       0.5462742152960396)]
C3 = [f32(v) for v in (-0.5900435899266435, 2.890611442640554, -0.4570457994644658, 0.3731763325901154,
                       -0.4570457994644658, 1.445305721320277, -0.5900435899266435)]
TILE = 16


def _t43(p, m):
    x, y, z = p[:, 0], p[:, 1], p[:, 2]
    return [((m[0 + r] * x + m[4 + r] * y) + m[8 + r] * z) + m[12 + r] for r in range(3)]


def _t44_xyw(p, m):
    x, y, z = p[:, 0], p[:, 1], p[:, 2]
    return [((m[0 + r] * x + m[4 + r] * y) + m[8 + r] * z) + m[12 + r] for r in (0, 1, 3)]


def _ndc2pix(v, S):
    return (((v.astype(np.float64) + 1.0) * float(S) - 1.0) * 0.5).astype(np.float32)


def _get_rect(mx, my, r, gx, gy):
    rf = r.astype(np.float32)
    def cvt(v):
        return np.trunc(v).astype(np.int64)
    x0 = np.minimum(gx, np.maximum(0, cvt((mx - rf) * f32(0.0625))))
    y0 = np.minimum(gy, np.maximum(0, cvt((my - rf) * f32(0.0625))))
    x1 = np.minimum(gx, np.maximum(0, cvt((((mx + rf) + f32(TILE)) - f32(1)) * f32(0.0625))))
    y1 = np.minimum(gy, np.maximum(0, cvt((((my + rf) + f32(TILE)) - f32(1)) * f32(0.0625))))
    return x0, y0, x1, y1


def sh_basis(x, y, z, deg):
    """The 16 real SH basis values at unit directions, in the kernel's order."""
    Y = [np.full_like(x, C0)]
    if deg >= 1:
        Y += [(-C1) * y, C1 * z, (-C1) * x]
    if deg >= 2:
        xx, yy, zz = x * x, y * y, z * z
        xy, yz, xz = x * y, y * z, x * z
        Y += [C2[0] * xy, C2[1] * yz, C2[2] * ((f32(2) * zz - xx) - yy), C2[3] * xz, C2[4] * (xx - yy)]
    if deg >= 3:
        Y += [(C3[0] * y) * (f32(3) * xx - yy), (C3[1] * xy) * z, (C3[2] * y) * ((f32(4) * zz - xx) - yy),
              (C3[3] * z) * ((f32(2) * zz - f32(3) * xx) - f32(3) * yy), (C3[4] * x) * ((f32(4) * zz - xx) - yy),
              (C3[5] * z) * (xx - yy), (C3[6] * x) * (xx - f32(3) * yy)]
    return Y


def preprocess(means3D, scales, rotations, opacities, shs, sh_degree, scale_modifier, viewmatrix, projmatrix,
               campos, W, H, tanfovx, tanfovy, near_plane=0.2):
    """Returns dict(radii, means2D, depths, cov3D, conic_opacity, rgb, clamped, tiles_touched)."""
    p = np.asarray(means3D, np.float32).reshape(-1, 3)
    P = p.shape[0]
    s_in = np.asarray(scales, np.float32).reshape(P, 3)
    q = np.asarray(rotations, np.float32).reshape(P, 4)
    op = np.asarray(opacities, np.float32).reshape(P)
    sh = np.asarray(shs, np.float32).reshape(P, -1, 3)
    V = np.asarray(viewmatrix, np.float32).reshape(16)
    Pm = np.asarray(projmatrix, np.float32).reshape(16)
    cam = np.asarray(campos, np.float32).reshape(3)
    mod = f32(scale_modifier)
    gx, gy = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
    fx = f32(W) / (f32(2) * f32(tanfovx))
    fy = f32(H) / (f32(2) * f32(tanfovy))
    limx, limy = f32(1.3) * f32(tanfovx), f32(1.3) * f32(tanfovy)

    with np.errstate(all="ignore"):
        tx, ty, tz = _t43(p, V)
        hx, hy, hw = _t44_xyw(p, Pm)
        pw = f32(1) / (hw + f32(1e-7))
        n = np.sqrt(((q[:, 0] * q[:, 0] + q[:, 1] * q[:, 1]) + q[:, 2] * q[:, 2]) + q[:, 3] * q[:, 3])
        r, x, y, z = q[:, 0] / n, q[:, 1] / n, q[:, 2] / n, q[:, 3] / n
        R = [[f32(1) - f32(2) * (y * y + z * z), f32(2) * (x * y - r * z), f32(2) * (x * z + r * y)],
             [f32(2) * (x * y + r * z), f32(1) - f32(2) * (x * x + z * z), f32(2) * (y * z - r * x)],
             [f32(2) * (x * z - r * y), f32(2) * (y * z + r * x), f32(1) - f32(2) * (x * x + y * y)]]
        s = [mod * s_in[:, k] for k in range(3)]
        M = [[R[j][k] * s[k] for k in range(3)] for j in range(3)]
        pairs = [(0, 0), (0, 1), (0, 2), (1, 1), (1, 2), (2, 2)]
        S = [(M[a][0] * M[b][0] + M[a][1] * M[b][1]) + M[a][2] * M[b][2] for a, b in pairs]
        idx = {(0, 0): 0, (0, 1): 1, (0, 2): 2, (1, 1): 3, (1, 2): 4, (2, 2): 5}

        def sym(i, j):
            return S[idx[(min(i, j), max(i, j))]]
        txtz, tytz = tx / tz, ty / tz
        txc = np.minimum(limx, np.maximum(-limx, txtz)) * tz
        tyc = np.minimum(limy, np.maximum(-limy, tytz)) * tz
        tz2 = tz * tz
        J00, J02 = fx / tz, -((fx * txc) / tz2)
        J11, J12 = fy / tz, -((fy * tyc) / tz2)
        u0 = [J00 * V[4 * k] + J02 * V[4 * k + 2] for k in range(3)]
        u1 = [J11 * V[4 * k + 1] + J12 * V[4 * k + 2] for k in range(3)]
        v = [(sym(i, 0) * u0[0] + sym(i, 1) * u0[1]) + sym(i, 2) * u0[2] for i in range(3)]
        w = [(sym(i, 0) * u1[0] + sym(i, 1) * u1[1]) + sym(i, 2) * u1[2] for i in range(3)]
        a = ((u0[0] * v[0] + u0[1] * v[1]) + u0[2] * v[2]) + f32(0.3)
        b = (u1[0] * v[0] + u1[1] * v[1]) + u1[2] * v[2]
        c = ((u1[0] * w[0] + u1[1] * w[1]) + u1[2] * w[2]) + f32(0.3)
        det = a * c - b * b
        idet = f32(1) / det
        mid = f32(0.5) * (a + c)
        disc = np.sqrt(np.maximum(f32(0.1), mid * mid - det))
        l1, l2 = mid + disc, mid - disc
        rad = np.ceil(f32(3) * np.sqrt(np.maximum(l1, l2)))
        m2x, m2y = _ndc2pix(hx * pw, W), _ndc2pix(hy * pw, H)

        front = tz > f32(near_plane)
        ok = front & (det != 0) & np.isfinite(rad)
        radi = np.where(ok, rad, 0).astype(np.int64)
        x0, y0, x1, y1 = _get_rect(m2x, m2y, radi, gx, gy)
        area = (x1 - x0) * (y1 - y0)
        ok &= area != 0

        dx, dy, dz = p[:, 0] - cam[0], p[:, 1] - cam[1], p[:, 2] - cam[2]
        ln = np.sqrt((dx * dx + dy * dy) + dz * dz)
        Y = sh_basis(dx / ln, dy / ln, dz / ln, sh_degree)
        col = np.zeros((P, 3), np.float32)
        for k, Yk in enumerate(Y):
            col = col + Yk[:, None] * sh[:, k, :]
        col = col + f32(0.5)

    out = dict(
        radii=np.where(ok, radi, 0).astype(np.int32),
        means2D=np.where(ok[:, None], np.stack([m2x, m2y], 1), f32(0)).astype(np.float32),
        depths=np.where(ok, tz, f32(0)).astype(np.float32),
        cov3D=np.where(ok[:, None], np.stack(S, 1), f32(0)).astype(np.float32),
        conic_opacity=np.where(ok[:, None], np.stack([c * idet, (-b) * idet, a * idet, op], 1), f32(0)).astype(
            np.float32),
        rgb=np.where(ok[:, None], np.maximum(col, f32(0)), f32(0)).astype(np.float32),
        clamped=np.where(ok[:, None], col < 0, False).astype(np.uint8),
        tiles_touched=np.where(ok, area, 0).astype(np.int32),
    )
    return out


def binning(radii, means2D, depths, tiles_touched, W, H):
    """(point_list, tile_ids, ranges [tiles, 2]) of a stable sort of tile << 32 | depth bits."""
    gx, gy = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
    radii = np.asarray(radii).astype(np.int64)
    m2 = np.asarray(means2D, np.float32).reshape(-1, 2)
    dbits = np.asarray(depths, np.float32).view(np.uint32).astype(np.uint64)
    x0, y0, x1, y1 = _get_rect(m2[:, 0], m2[:, 1], radii, gx, gy)
    keys, vals = [], []
    for i in np.nonzero(np.asarray(tiles_touched) > 0)[0]:
        ty, tx = np.meshgrid(np.arange(y0[i], y1[i]), np.arange(x0[i], x1[i]), indexing="ij")
        t = (ty * gx + tx).reshape(-1).astype(np.uint64)
        keys.append((t << np.uint64(32)) | dbits[i])
        vals.append(np.full(t.shape, i, np.int64))
    tiles = gx * gy
    if not keys:
        return np.zeros(0, np.int32), np.zeros(0, np.int32), np.zeros((tiles, 2), np.int32)
    keys, vals = np.concatenate(keys), np.concatenate(vals)
    order = np.argsort(keys, kind="stable")
    keys, vals = keys[order], vals[order]
    tid = (keys >> np.uint64(32)).astype(np.int64)
    ranges = np.zeros((tiles, 2), np.int64)
    starts = np.searchsorted(tid, np.arange(tiles), "left")
    ends = np.searchsorted(tid, np.arange(tiles), "right")
    ranges[:, 0], ranges[:, 1] = starts, ends
    ranges[starts == ends] = 0
    return vals.astype(np.int32), tid.astype(np.int32), ranges.astype(np.int32)
