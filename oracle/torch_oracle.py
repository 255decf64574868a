"""Vectorised PyTorch-on-CPU restatement of the reference algorithm -- TEST
INFRASTRUCTURE and the timed CPU baseline; the product never imports it.

It computes what oracle/vi_oracle.c computes (the reference extension's
forward and backward, paths relative to that project), with torch tensor
operations on the host cores instead of scalar loops:

  preprocess           cuda_integrator/forward.cu:27-110, auxiliary.h:50-86,148-175
  binning              integrator_impl.cu:306-365 (scan, duplicateWithKeys, stable
                       sort of tile|depth keys -- torch.sort(stable=True) gives the
                       permutation of CUB's stable LSD radix sort -- identifyTileRanges)
  render               forward.cu:296-791, hashgrid.h:207-299
  backward             backward.cu:107-791, hashgrid.h:9-96 (the reference's formula,
                       which is not the derivative of the forward)

Arrangement: stage 1 of the reference (grid point positions, screen points,
hashgrid features, linear layer) depends only on the primitive, so it is
computed once per primitive that the requested tiles list, not once per (tile,
primitive).  Stage 2 becomes one record per (primitive, pixel) whose occupancy
sum passes the reference's 1e-7 test, summed with index_add_ in grid-point
order.  Compositing runs over all pixels at once, one list entry of every
pixel per iteration.  The backward aggregates each grid point's table
coefficient over the pixels before one scatter per (grid point, level, corner)
-- the same sums in another order.

Floating point: element-wise float32 tensor operations round each operation
separately, as the C oracle (compiled without contraction); ndc2Pix and the
radius' 1e-6 are evaluated in float64 as the reference's double literals make
them.  The linear layer is a matrix product, so images and gradients agree
with the C oracle to rounding (tests/test_torch_oracle.py), integers exactly.
Stage-1 work is chunked to bound host memory.
"""
import math

import numpy as np
import torch

TILE = 16
_CHUNK = 1 << 17  # primitives per stage-1 chunk


def _f(x):
    return torch.as_tensor(np.asarray(x), dtype=torch.float32)


def _i(x):
    return torch.as_tensor(np.asarray(x), dtype=torch.int64)


def _t43(p, m):
    """transformPoint4x3 (auxiliary.h:67-75): ((m0 x + m4 y) + m8 z) + m12."""
    x, y, z = p[..., 0], p[..., 1], p[..., 2]
    return (m[0] * x + m[4] * y + m[8] * z + m[12], m[1] * x + m[5] * y + m[9] * z + m[13],
            m[2] * x + m[6] * y + m[10] * z + m[14])


def _t44_xyw(p, m):
    x, y, z = p[..., 0], p[..., 1], p[..., 2]
    return (m[0] * x + m[4] * y + m[8] * z + m[12], m[1] * x + m[5] * y + m[9] * z + m[13],
            m[3] * x + m[7] * y + m[11] * z + m[15])


def _ndc2pix(v, S):
    """auxiliary.h:50-53 in double: ((v + 1) * S - 1) * 0.5."""
    return (((v.double() + 1.0) * float(S) - 1.0) * 0.5).float()


def _rect(px, py, r, gx, gy):
    """getRect (auxiliary.h:55-65) with float arithmetic and truncation."""
    rf = r.float()

    def clampi(v, g):
        a = torch.trunc(v).clamp(min=-2.0 ** 31, max=2.0 ** 31 - 1).to(torch.int64)
        return torch.minimum(torch.clamp(a, min=0), torch.tensor(g))
    x0 = clampi((px - rf) / 16.0, gx)
    y0 = clampi((py - rf) / 16.0, gy)
    x1 = clampi((px + rf + 16.0 - 1.0) / 16.0, gx)
    y1 = clampi((py + rf + 16.0 - 1.0) / 16.0, gy)
    return x0, y0, x1, y1


class Scene:
    """Torch views of an oracle.Scene (the same fields, float32/int64 tensors)."""

    def __init__(self, s):
        self.s = s
        self.P, self.W, self.H, self.G = s.P, s.W, s.H, s.G
        self.V = s.G ** 3
        self.means = _f(s.means).reshape(-1, 3)
        self.conf = _f(s.conf).reshape(self.P, self.V)
        self.scale = float(s.scale)
        self.view = _f(s.view).reshape(16)
        self.proj = _f(s.proj).reshape(16)
        self.table = _f(s.table).reshape(-1)
        self.res = [int(r) for r in np.asarray(s.res)]
        self.do_hash = [int(h) for h in np.asarray(s.do_hash)]
        self.primes = [int(np.uint32(np.int32(p))) for p in np.asarray(s.primes)]
        self.T = int(s.T)
        self.L, self.F, self.Fout = s.L, s.F, s.Fout
        self.D, self.O = s.L * s.F, 3 + s.Fout + 1
        self.Wl = _f(s.Wl).reshape(self.O, self.D)
        self.bl = _f(s.bl).reshape(self.O)
        self.bg = _f(s.bg).reshape(-1)
        self.K, self.genus = s.K, s.genus
        self.near_plane, self.max_distance = float(s.near_plane), float(s.max_distance)
        self.hlo = torch.tensor([float(v) for v in s.hlo], dtype=torch.float32)
        self.hext = torch.tensor([float(v) for v in s.hext], dtype=torch.float32)
        self.gx, self.gy = (s.W + 15) // 16, (s.H + 15) // 16
        self.tanfovx, self.tanfovy = float(s.tanfovx), float(s.tanfovy)
        g = torch.arange(self.V)
        self.gz, self.gyy, self.gxx = g // (self.G * self.G), (g % (self.G * self.G)) // self.G, g % self.G
        step = self.scale / float(self.G - 1) if self.G > 1 else self.scale
        self.step = float(np.float32(step))
        gof = float(np.float32((self.G - 1) / 2.0))
        self.rel = torch.stack([(self.gxx.float() - gof) * self.step, (self.gyy.float() - gof) * self.step,
                                (self.gz.float() - gof) * self.step], 1)  # [V, 3], forward.cu:421-428
        c = [1.0 / 12.0, -2.0 / 3.0, 0.0, 2.0 / 3.0, -1.0 / 12.0] if self.genus == 2 else [-0.5, 0.0, 0.5]
        self.taps = [float(np.float32(v)) for v in c]


# ---------------------------------------------------------------------------
# preprocess and binning
# ---------------------------------------------------------------------------
def preprocess(sc):
    P, W, H = sc.P, sc.W, sc.H
    fy = float(np.float32(H) / (np.float32(2.0) * np.float32(sc.tanfovy)))
    fx = float(np.float32(W) / (np.float32(2.0) * np.float32(sc.tanfovx)))
    vx, vy, vz = _t43(sc.means, sc.view)
    hx, hy, hw = _t44_xyw(sc.means, sc.proj)
    pw = 1.0 / (hw + 1e-7)
    wr = float(np.float32(sc.scale) * np.float32(0.86602540378))
    vd = (vz.abs().double() + 1e-6).float()
    r = torch.ceil(torch.maximum(wr * fx / vd, wr * fy / vd))
    r = torch.where(torch.isfinite(r), r, torch.zeros_like(r)).clamp(-2.0 ** 31, 2.0 ** 31 - 1).to(torch.int64)
    mx, my = _ndc2pix(hx * pw, W), _ndc2pix(hy * pw, H)
    x0, y0, x1, y1 = _rect(mx, my, r, sc.gx, sc.gy)
    tiles = (x1 - x0) * (y1 - y0)
    vis = (vz > 0.2) & (tiles > 0) & (r > 0)
    z = torch.zeros_like(vz)
    return dict(radii=torch.where(vis, r, 0).to(torch.int32), depths=torch.where(vis, vz, z),
                means2D=torch.stack([torch.where(vis, mx, z), torch.where(vis, my, z)], 1),
                tiles_touched=torch.where(vis, tiles, 0), rect=(x0, y0, x1, y1), visible=vis)


def binning(sc, pre):
    vis = pre["visible"]
    idx = torch.nonzero(vis).flatten()
    x0, y0, x1, y1 = [t[idx] for t in pre["rect"]]
    w, h = x1 - x0, y1 - y0
    n = w * h
    R = int(n.sum())
    q = torch.repeat_interleave(idx, n)
    start = torch.cumsum(n, 0) - n
    k = torch.arange(R) - torch.repeat_interleave(start, n)
    wq = torch.repeat_interleave(w, n)
    tx = torch.repeat_interleave(x0, n) + k % wq
    ty = torch.repeat_interleave(y0, n) + k // wq
    tile = ty * sc.gx + tx
    dbits = pre["depths"].view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    keys = (tile << 32) | dbits[q]
    keys_sorted, order = torch.sort(keys, stable=True)
    point_list = q[order]
    tiles_sorted = keys_sorted >> 32
    ntiles = sc.gx * sc.gy
    counts = torch.bincount(tiles_sorted, minlength=ntiles)
    ends = torch.cumsum(counts, 0)
    starts = ends - counts
    ranges = torch.stack([torch.where(counts > 0, starts, 0), torch.where(counts > 0, ends, 0)], 1)
    return dict(num_rendered=R, keys=keys_sorted, point_list=point_list, ranges=ranges)


# ---------------------------------------------------------------------------
# stage 1 per primitive (hoisted)
# ---------------------------------------------------------------------------
def _corner_entries(sc, b, l):
    """Table rows of the 8 corners (dx, dy, dz nesting order) of base cells b
    [..., 3] at level l, or -1 (hashgrid.h:258-275)."""
    res = sc.res[l]
    out = []
    for dx in (0, 1):
        for dy in (0, 1):
            for dz in (0, 1):
                cx, cy, cz = b[..., 0] + dx, b[..., 1] + dy, b[..., 2] + dz
                if sc.do_hash[l]:
                    h = ((cx * sc.primes[0]) & 0xFFFFFFFF) ^ ((cy * sc.primes[1]) & 0xFFFFFFFF) ^ \
                        ((cz * sc.primes[2]) & 0xFFFFFFFF)
                    e = h % sc.T
                else:
                    inb = (cx >= 0) & (cx < res) & (cy >= 0) & (cy < res) & (cz >= 0) & (cz < res)
                    e = (cz * res * res + cy * res + cx) & 0xFFFFFFFF
                    e = torch.where(inb & (e < sc.T), e, torch.full_like(e, -1))
                out.append(e)
    return out


def _level_setup(sc, pos, l):
    n = ((pos - sc.hlo) / sc.hext).clamp(0.0, 1.0)
    p = n * float(sc.res[l])
    fl = torch.floor(p)
    return fl.to(torch.int64), p - fl


def stage1(sc, q, fwd):
    """For primitives q [n]: positions [n,V,3], screen points [n,V,2] (forward
    1/(w+1e-7) or backward 1/w), features phi [n,V,D], linear layer mlp [n,V,O]."""
    c = sc.means[q]
    pos = c[:, None, :] + sc.rel[None, :, :]
    hx, hy, hw = _t44_xyw(pos, sc.proj)
    pw = 1.0 / (hw + 1e-7) if fwd else 1.0 / hw
    scr = torch.stack([_ndc2pix(hx * pw, sc.W), _ndc2pix(hy * pw, sc.H)], -1)
    n = q.numel()
    phi = torch.zeros(n, sc.V, sc.D)
    tab = sc.table.view(-1, sc.L, sc.F)
    for l in range(sc.L):
        b, t = _level_setup(sc, pos, l)
        acc = torch.zeros(n, sc.V, sc.F)
        ents = _corner_entries(sc, b, l)
        k = 0
        for dx in (0, 1):
            wx = t[..., 0] if dx else 1.0 - t[..., 0]
            for dy in (0, 1):
                wy = t[..., 1] if dy else 1.0 - t[..., 1]
                for dz in (0, 1):
                    wz = t[..., 2] if dz else 1.0 - t[..., 2]
                    w = wx * wy * wz
                    e = ents[k]
                    k += 1
                    ok = e >= 0
                    v = tab[e.clamp(min=0), l, :] * w[..., None]
                    acc = acc + torch.where(ok[..., None], v, torch.zeros_like(v))
        phi[:, :, l * sc.F:(l + 1) * sc.F] = acc
    mlp = phi @ sc.Wl.t()
    return pos, scr, phi, mlp


def _stencil_mag(sc, occ):
    """|d/dx| + |d/dy| + |d/dz| of a boolean occupancy [..., V] with the
    reference's taps, summed in tap order (forward.cu:557-611)."""
    G = sc.G
    o = occ.reshape(*occ.shape[:-1], G, G, G).float()  # [..., z, y, x]
    S = len(sc.taps)
    off = (S - 1) // 2
    out = []
    for axis in (-1, -2, -3):  # x, y, z
        acc = torch.zeros_like(o)
        for s in range(S):
            r = s - off
            sh = torch.zeros_like(o)
            src = [slice(None)] * o.dim()
            dst = [slice(None)] * o.dim()
            if r >= 0:
                src[axis], dst[axis] = slice(r, G), slice(0, G - r)
            else:
                src[axis], dst[axis] = slice(0, G + r), slice(-r, G)
            sh[tuple(dst)] = o[tuple(src)]
            acc = acc + sh * sc.taps[s]
        out.append(acc.abs())
    return (out[0] + out[1] + out[2]).reshape(occ.shape)


# ---------------------------------------------------------------------------
# render
# ---------------------------------------------------------------------------
def _records(sc, q, pre, fwd=True):
    """(primitive, pixel) records of primitives q: key = q * N + pixel, the
    occupancy sum, the pre-activation sums of the linear layer and (for the
    backward) of the features, and per grid point the pixel and magnitude."""
    N = sc.W * sc.H
    pos, scr, phi, mlp = stage1(sc, q, fwd)
    conf = sc.conf[q]
    mag = _stencil_mag(sc, conf > 0)
    px, py = torch.floor(scr[..., 0]), torch.floor(scr[..., 1])
    inside = (px >= 0) & (px < sc.W) & (py >= 0) & (py < sc.H)
    x0, y0, x1, y1 = [t[q][:, None] for t in pre["rect"]]
    pxi, pyi = px.clamp(-1, sc.W).to(torch.int64), py.clamp(-1, sc.H).to(torch.int64)
    tx, ty = pxi.div(16, rounding_mode="floor"), pyi.div(16, rounding_mode="floor")
    ok = inside & (conf > 0) & (tx >= x0) & (tx < x1) & (ty >= y0) & (ty < y1)
    pix = pyi * sc.W + pxi
    key = q[:, None] * N + pix
    sel = ok.flatten()
    k = key.flatten()[sel]
    uk, inv = torch.unique(k, return_inverse=True)
    m = mag.flatten()[sel]
    w = (conf * mag).flatten()[sel]
    use = (m > 1e-7)
    ogs = torch.zeros(uk.numel()).index_add_(0, inv, m)
    contrib = mlp.reshape(-1, sc.O)[sel] * w[:, None]
    contrib = torch.where(use[:, None], contrib, torch.zeros_like(contrib))
    agg = torch.zeros(uk.numel(), sc.O).index_add_(0, inv, contrib)
    out = dict(key=uk, ogs=ogs, agg=agg)
    if not fwd:
        fi = phi.reshape(-1, sc.D)[sel] * w[:, None]
        fi = torch.where(use[:, None], fi, torch.zeros_like(fi))
        out["in"] = torch.zeros(uk.numel(), sc.D).index_add_(0, inv, fi)
        out["pos"], out["scr"], out["phi"], out["conf"] = pos, scr, phi, conf
    return out


def _tiles_of(mask, sc):
    return torch.ones(sc.gx * sc.gy, dtype=torch.bool) if mask is None else torch.as_tensor(np.asarray(mask) != 0)


def render(sc, pre, b, tile_mask=None):
    """Images and contributor lists (pixels of the masked tiles only)."""
    N, K, O = sc.W * sc.H, sc.K, sc.O
    tm = _tiles_of(tile_mask, sc)
    rng = b["ranges"]
    ent_tile = torch.repeat_interleave(torch.arange(rng.shape[0]), rng[:, 1] - rng[:, 0])
    ent_j = torch.cat([torch.arange(int(a), int(c)) for a, c in rng.tolist() if c > a]) if b["num_rendered"] else \
        torch.zeros(0, dtype=torch.int64)
    sel = tm[ent_tile]
    ent_tile, ent_j = ent_tile[sel], ent_j[sel]
    ent_q = b["point_list"][ent_j]
    prims = torch.unique(ent_q)
    # records of those primitives, chunked
    rk, rogs, ragg = [], [], []
    for i in range(0, prims.numel(), _CHUNK):
        r = _records(sc, prims[i:i + _CHUNK], pre)
        rk.append(r["key"])
        rogs.append(r["ogs"])
        ragg.append(r["agg"])
    rkey = torch.cat(rk) if rk else torch.zeros(0, dtype=torch.int64)
    keep = torch.cat(rogs) >= 1e-7 if rk else torch.zeros(0, dtype=torch.bool)
    rkey = rkey[keep]
    pre_act = (torch.cat(ragg)[keep] + sc.bl) if rk else torch.zeros(0, O)
    props = torch.cat([torch.sigmoid(pre_act[:, :O - 1]), torch.exp(pre_act[:, O - 1:])], 1)
    rq, rpix = rkey // N, rkey % N
    rtile = (rpix // sc.W // 16) * sc.gx + (rpix % sc.W) // 16
    # list position of each record: the entry (tile, primitive)
    P = sc.P
    ekey = ent_tile * P + ent_q
    eorder = torch.argsort(ekey)
    ek_sorted = ekey[eorder]
    look = rtile * P + rq
    pos = torch.searchsorted(ek_sorted, look)
    found = (pos < ek_sorted.numel()) & (ek_sorted[pos.clamp(max=max(ek_sorted.numel() - 1, 0))] == look)
    rpix, rq, props = rpix[found], rq[found], props[found]
    rj = ent_j[eorder[pos[found]]]
    # events per pixel in list order
    order = torch.argsort(rpix * (b["num_rendered"] + 1) + rj)
    rpix, rq, props, rj = rpix[order], rq[order], props[order], rj[order]
    depth_all = _t43(sc.means, sc.view)[2]
    rdepth = depth_all[rq]
    upix, counts = torch.unique_consecutive(rpix, return_counts=True)
    first = torch.cumsum(counts, 0) - counts
    npx = upix.numel()
    Tt = torch.ones(npx)
    C = torch.zeros(npx, 3)
    Fe = torch.zeros(npx, sc.Fout)
    cnt = torch.zeros(npx, dtype=torch.int64)
    has_p = torch.zeros(npx, dtype=torch.bool)
    done = torch.zeros(npx, dtype=torch.bool)
    pend = torch.zeros(npx, O)
    pdepth = torch.full((npx,), sc.near_plane)
    Tp = torch.zeros(npx)
    pidx = torch.zeros(npx, dtype=torch.int64)
    contrib_idx = torch.full((N, K), -1, dtype=torch.int64)
    delta_t = torch.zeros(N, K)

    def composite(ids, dt):
        a = 1.0 - torch.exp(-pend[ids, O - 1] * dt)
        a = a.clamp(0.0, 1.0)
        wgt = Tp[ids] * a
        C[ids] += wgt[:, None] * pend[ids, :3]
        Fe[ids] += wgt[:, None] * pend[ids, 3:3 + sc.Fout]
        Tt[ids] = Tp[ids] * (1.0 - a)
        contrib_idx[upix[ids], cnt[ids]] = pidx[ids]
        delta_t[upix[ids], cnt[ids]] = dt
        cnt[ids] += 1

    active = torch.arange(npx)
    step = 0
    while active.numel():
        ev = first[active] + step
        ids = active
        d = rdepth[ev]
        hp = has_p[ids]
        dt = torch.clamp(d - pdepth[ids], min=0.0)
        c1 = hp & (dt > 1e-5) & (cnt[ids] < K)
        if c1.any():
            composite(ids[c1], dt[c1])
        ok = (Tt[ids] >= 1e-4) & (cnt[ids] < K)
        sel_ok = ids[ok]
        pend[sel_ok] = props[ev[ok]]
        pdepth[sel_ok] = d[ok]
        pidx[sel_ok] = rj[ev[ok]]
        has_p[sel_ok] = True
        Tp[sel_ok] = Tt[sel_ok]
        bad = ids[~ok]
        has_p[bad] = False
        done[bad] = True
        done[ids] |= (Tt[ids] < 1e-4) | (cnt[ids] >= K)
        step += 1
        active = active[(~done[active]) & (step < counts[active])]
    fin = has_p & (Tt >= 1e-4) & (cnt < K)
    dtf = torch.clamp(sc.max_distance - pdepth, min=0.0)
    fin &= dtf > 1e-5
    ids = torch.nonzero(fin).flatten()
    if ids.numel():
        composite(ids, dtf[ids])
    # images of the masked tiles
    allpix = torch.arange(N)
    ptile = (allpix // sc.W // 16) * sc.gx + (allpix % sc.W) // 16
    inmask = tm[ptile]
    T_img = torch.ones(N)
    C_img = torch.zeros(N, 3)
    F_img = torch.zeros(N, sc.Fout)
    n_img = torch.zeros(N, dtype=torch.int64)
    T_img[upix], C_img[upix], F_img[upix], n_img[upix] = Tt, C, Fe, cnt
    color = (C_img + T_img[:, None] * sc.bg).clamp(0.0, 1.0)
    z = lambda x: torch.where(inmask.reshape(-1, *([1] * (x.dim() - 1))), x, torch.zeros_like(x))  # noqa: E731
    out = dict(out_color=z(color).t().reshape(3, sc.H, sc.W), out_features=z(F_img).t().reshape(sc.Fout, sc.H, sc.W),
               visibility=z(1.0 - T_img).reshape(sc.H, sc.W), final_T=z(T_img), n_contrib=z(n_img),
               contrib_idx=torch.where(inmask[:, None], contrib_idx, -1).reshape(-1),
               delta_t=z(delta_t).reshape(-1))
    return out


# ---------------------------------------------------------------------------
# backward (the reference's formula)
# ---------------------------------------------------------------------------
def backward(sc, pre, b, fwd, dL_dcolor, dL_dfeat, tile_mask=None):
    N, K, O, D, V = sc.W * sc.H, sc.K, sc.O, sc.D, sc.V
    B = O - 1
    g = dict(dL_dmeans3D=torch.zeros(sc.P, 3), dL_dconfidences=torch.zeros(sc.P, V),
             dL_dfeature_table=torch.zeros(sc.table.numel()), dL_dlinear_weights=torch.zeros(O * D),
             dL_dlinear_bias=torch.zeros(O))
    if b["num_rendered"] == 0:
        return g
    tm = _tiles_of(tile_mask, sc)
    nc = fwd["n_contrib"].clamp(max=K)
    allpix = torch.arange(N)
    ptile = (allpix // sc.W // 16) * sc.gx + (allpix % sc.W) // 16
    pix = allpix[tm[ptile] & (nc > 0)]
    if pix.numel() == 0:
        return g
    nc = nc[pix]
    cidx = fwd["contrib_idx"].reshape(N, K)[pix]
    dts = fwd["delta_t"].reshape(N, K)[pix]
    cq = b["point_list"][cidx.clamp(min=0)]
    # per contribution: backward-projection records of its primitive at its pixel
    prims = torch.unique(cq[torch.arange(K)[None, :] < nc[:, None]])
    rk, rin, ragg = [], [], []
    pos_l, scr_l, phi_l, conf_l = [], [], [], []
    for i in range(0, prims.numel(), _CHUNK):
        r = _records(sc, prims[i:i + _CHUNK], pre, fwd=False)
        rk.append(r["key"])
        rin.append(r["in"])
        ragg.append(r["agg"])
        pos_l.append(r["pos"])
        scr_l.append(r["scr"])
        phi_l.append(r["phi"])
        conf_l.append(r["conf"])
    rkey, rin, ragg = torch.cat(rk), torch.cat(rin), torch.cat(ragg)
    ppos, pscr, pphi, pconf = torch.cat(pos_l), torch.cat(scr_l), torch.cat(phi_l), torch.cat(conf_l)
    slot_of = torch.full((sc.P,), -1, dtype=torch.int64)
    slot_of[prims] = torch.arange(prims.numel())
    dOut = torch.cat([dL_dcolor.reshape(3, N)[:, pix].t(),
                      (dL_dfeat.reshape(sc.Fout, N)[:, pix].t() if sc.Fout else torch.zeros(pix.numel(), 0))], 1)
    after = torch.cat([sc.bg.expand(pix.numel(), 3), torch.zeros(pix.numel(), sc.Fout)], 1)
    # contributions in reverse per pixel: k = nc-1 .. 0
    rows = []  # (pixel row, contribution k, dpre, in)
    Wl = sc.Wl
    for k in range(K - 1, -1, -1):
        act = nc > k
        if not act.any():
            continue
        ids = torch.nonzero(act).flatten()
        q = cq[ids, k]
        look = q * N + pix[ids]
        pos = torch.searchsorted(rkey, look)
        hit = (pos < rkey.numel()) & (rkey[pos.clamp(max=rkey.numel() - 1)] == look)
        agg = torch.where(hit[:, None], ragg[pos.clamp(max=rkey.numel() - 1)], torch.zeros(ids.numel(), O))
        inn = torch.where(hit[:, None], rin[pos.clamp(max=rkey.numel() - 1)], torch.zeros(ids.numel(), D))
        pre_act = agg + sc.bl
        blend = torch.sigmoid(pre_act[:, :B])
        dens = torch.exp(pre_act[:, B])
        dO, af = dOut[ids], after[ids]
        dbl = dO * blend
        dalpha = (dbl * (blend - af)).sum(1)
        dpre = torch.cat([dO * blend * blend * (1.0 - blend), (dalpha * dens * dts[ids, k] * dens)[:, None]], 1)
        rows.append((ids, q, dpre, inn))
        dOut[ids] = dO * blend
        after[ids] = blend + af * (1.0 - blend)
    ids = torch.cat([r[0] for r in rows])
    q = torch.cat([r[1] for r in rows])
    dpre = torch.cat([r[2] for r in rows])
    inn = torch.cat([r[3] for r in rows])
    g["dL_dlinear_bias"] += dpre.sum(0)
    g["dL_dlinear_weights"] += (dpre.t() @ inn).reshape(-1)
    dIn = dpre @ Wl  # [C, D]
    # (C) per contribution and grid point: g' from neighbours whose backward
    # screen point lies in this pixel (backward.cu:644-689)
    s = slot_of[q]
    cpix = pix[ids]
    cx, cy = (cpix % sc.W).float(), (cpix // sc.W).float()
    scr = pscr[s]  # [C, V, 2]
    inpix = (scr[..., 0] >= cx[:, None]) & (scr[..., 0] < cx[:, None] + 1.0) & \
            (scr[..., 1] >= cy[:, None]) & (scr[..., 1] < cy[:, None] + 1.0)
    m2 = _stencil_mag(sc, inpix)  # [C, V]
    use = m2 > 1e-7
    phi = pphi[s]  # [C, V, D]
    dX = (phi * dIn[:, None, :]).sum(-1) * m2
    dX = torch.where(use, dX, torch.zeros_like(dX))
    g["dL_dconfidences"].view(-1).index_add_(0, (q[:, None] * V + torch.arange(V)).flatten(), dX.flatten())
    wg = m2 * pconf[s]
    usea = use & (wg.abs() > 1e-9)
    coef = torch.where(usea[..., None], dIn[:, None, :] * wg[..., None], torch.zeros(1))  # [C, V, D]
    # sum per (primitive, grid point) before scattering: the corners depend on (q, g) only
    A = torch.zeros(prims.numel(), V, D).index_add_(0, s, coef)
    gpos = ppos  # [np, V, 3]
    tab_grad = g["dL_dfeature_table"]
    for l in range(sc.L):
        bcell, t = _level_setup(sc, gpos, l)
        ents = _corner_entries(sc, bcell, l)
        a = A[:, :, l * sc.F:(l + 1) * sc.F]
        k = 0
        for dx in (0, 1):
            for dy in (0, 1):
                for dz in (0, 1):
                    w = (t[..., 0] if dx else 1.0 - t[..., 0]) * (t[..., 1] if dy else 1.0 - t[..., 1]) * \
                        (t[..., 2] if dz else 1.0 - t[..., 2])
                    e = ents[k]
                    k += 1
                    ok = (e >= 0)
                    v = a * w[..., None]
                    idx = (e.clamp(min=0)[..., None] * sc.L + l) * sc.F + torch.arange(sc.F)
                    m = ok[..., None].expand_as(idx) & (v != 0)
                    tab_grad.index_add_(0, idx[m], v[m])
    return g


def forward(s, tile_mask=None):
    """Forward of an oracle.Scene; returns (torch scene, dict of tensors)."""
    sc = Scene(s)
    pre = preprocess(sc)
    b = binning(sc, pre)
    out = render(sc, pre, b, tile_mask=tile_mask)
    res = dict(pre)
    res.update(b)
    res.update(out)
    return sc, res


def run(s, dL_dcolor, dL_dfeat, tile_mask=None):
    """Forward + backward; numpy outputs like oracle.forward / oracle.backward."""
    sc, f = forward(s, tile_mask)
    pre = {k: f[k] for k in ("radii", "depths", "means2D", "tiles_touched", "rect", "visible")}
    b = {k: f[k] for k in ("num_rendered", "keys", "point_list", "ranges")}
    grads = backward(sc, pre, b, f, torch.as_tensor(np.asarray(dL_dcolor), dtype=torch.float32),
                     torch.as_tensor(np.asarray(dL_dfeat), dtype=torch.float32), tile_mask=tile_mask)
    np_f = {k: (v.numpy() if torch.is_tensor(v) else v) for k, v in f.items() if k not in ("rect",)}
    return np_f, {k: v.numpy() for k, v in grads.items()}
