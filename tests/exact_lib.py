"""Oracle of the exact-gradient mode: the forward restated in float64 torch on
the discrete structure of the oracle's own forward, differentiated by autograd.

The forward is piecewise smooth: which grid points land in which pixel, the
stencil magnitudes, the pixels' contributor lists and their order are discrete
and held fixed; everything else is a smooth function of the inputs:

* grid point positions = centre + fixed offsets; hashgrid trilinear features
  (hashgrid.h:207-299) of the clamped normalised position;
* record pre-activation = sum over its grid points of conf * mag * (W phi) + b,
  then sigmoid (colour, features) and exp (density) (forward.cu:481-643);
* compositing (forward.cu:649-785): alpha = 1 - exp(-sigma dt) with
  dt = depth(next covering primitive) - depth, or max_distance - depth for the
  last; C = clamp(sum T alpha c + T_n bg, 0, 1), F = sum T alpha f,
  visibility = 1 - T_n; depth = view-space z of the centre.

The structure comes from the C oracle (contributor lists, delta t, and the grid
points of each record through vio_record_lanes), so it is the reference's.
"""
import numpy as np
import torch

import oracle as orc


def _struct(sc, f):
    """Per pixel: list of (q, lanes, mags, trigger q or -1), from the oracle's forward f."""
    W, H, K = sc.W, sc.H, sc.K
    pl = f["point_list"].astype(np.int64)
    ci = f["contrib_idx"].reshape(-1, K)
    nc = f["n_contrib"].reshape(-1)
    ranges = f["ranges"].reshape(-1, 2)
    gx = (W + 15) // 16
    cache = {}

    def lanes(q, px, py):
        key = (q, px, py)
        if key not in cache:
            cache[key] = orc.record_lanes(sc, q, px, py)
        return cache[key]

    out = {}
    for pix in np.nonzero(nc)[0]:
        px, py = int(pix % W), int(pix // W)
        t = (py // 16) * gx + (px // 16)
        r1 = int(ranges[t, 1])
        seq = []
        for k in range(int(nc[pix])):
            j = int(ci[pix, k])
            q = int(pl[j])
            ln, mg = lanes(q, px, py)
            trig = -1  # the first covering entry after j composited this one
            for jj in range(j + 1, r1):
                if len(lanes(int(pl[jj]), px, py)[0]):
                    trig = int(pl[jj])
                    break
            seq.append((q, ln, mg, trig))
        out[int(pix)] = seq
    return out


def _hashgrid(pos, table, s, lo, ext):
    """(N, 3) float64 positions -> (N, L*F) trilinear hashgrid features (hashgrid.h:207-299)."""
    L, F, T = s.hashgrid_levels, s.input_feature_dim, s.feature_offset
    res = [int(r) for r in np.asarray(s.resolution.cpu()).reshape(-1)]
    do_hash = [int(h) for h in np.asarray(s.do_hash.cpu()).reshape(-1)]
    primes = [int(p) & 0xFFFFFFFF for p in np.asarray(s.primes.cpu()).reshape(-1)]
    tab = table.view(-1, L, F)
    n = torch.clamp((pos - lo) / ext, 0.0, 1.0)
    feats = []
    for l in range(L):
        x = n * res[l]
        b = torch.floor(x).detach()
        t = x - b
        bi = b.long()
        acc = torch.zeros(pos.shape[0], F, dtype=pos.dtype)
        for dx in (0, 1):
            for dy in (0, 1):
                for dz in (0, 1):
                    cx, cy, cz = bi[:, 0] + dx, bi[:, 1] + dy, bi[:, 2] + dz
                    if do_hash[l]:
                        h = ((cx * primes[0]) & 0xFFFFFFFF) ^ ((cy * primes[1]) & 0xFFFFFFFF) ^ \
                            ((cz * primes[2]) & 0xFFFFFFFF)
                        idx = h % T
                        valid = torch.ones_like(idx, dtype=torch.bool)
                    else:
                        r = res[l]
                        valid = (cx >= 0) & (cx < r) & (cy >= 0) & (cy < r) & (cz >= 0) & (cz < r)
                        idx = (cz * r * r + cy * r + cx) & 0xFFFFFFFF
                        valid = valid & (idx < T)
                        idx = torch.where(valid, idx, torch.zeros_like(idx))
                    w = (t[:, 0] if dx else 1 - t[:, 0]) * (t[:, 1] if dy else 1 - t[:, 1]) * \
                        (t[:, 2] if dz else 1 - t[:, 2])
                    w = torch.where(valid, w, torch.zeros_like(w))
                    acc = acc + w[:, None] * tab[idx, l, :]
        feats.append(acc)
    return torch.cat(feats, dim=1)


def exact_grads(means, conf, s, dcolor, dfeat, dvis, threads=8):
    """(images, gradients) of the forward in float64 on the oracle's structure."""
    sc = orc.Scene.from_settings(means, conf, s)
    f = orc.forward(sc, threads=threads)
    st = _struct(sc, f)
    G, V, O = s.grid_size, s.grid_size ** 3, 3 + s.output_feature_dim + 1
    Fout, H, W = s.output_feature_dim, s.image_height, s.image_width
    dev = torch.device("cpu")
    m = torch.tensor(np.asarray(means.detach().cpu()), dtype=torch.float64, device=dev, requires_grad=True)
    c = torch.tensor(np.asarray(conf.detach().cpu()).reshape(-1, V), dtype=torch.float64, requires_grad=True)
    tab = torch.tensor(np.asarray(s.feature_table.detach().cpu()).reshape(-1), dtype=torch.float64,
                       requires_grad=True)
    Wl = torch.tensor(np.asarray(s.linear_weights.detach().cpu()).reshape(-1), dtype=torch.float64,
                      requires_grad=True)
    bl = torch.tensor(np.asarray(s.linear_bias.detach().cpu()).reshape(-1), dtype=torch.float64, requires_grad=True)
    view = torch.tensor(np.asarray(s.viewmatrix.cpu()).reshape(16), dtype=torch.float64)
    bg = torch.tensor(np.asarray(s.bg_color.cpu()).reshape(-1), dtype=torch.float64)
    hb = s.hash_bounds
    if hb is None:
        lo = torch.full((3,), -1.3, dtype=torch.float64)
        ext = torch.full((3,), 2.6, dtype=torch.float64)
    else:
        hb = [float(v) for v in hb]
        lo = torch.tensor(hb[:3], dtype=torch.float64)
        ext = torch.tensor(hb[3:], dtype=torch.float64) - lo
    step = s.primitive_scale / (G - 1) if G > 1 else s.primitive_scale
    gof = (G - 1) / 2.0
    g = np.arange(V)
    offs = torch.tensor(np.stack([(g % G - gof), (g // G % G - gof), (g // (G * G) - gof)], 1) * step,
                        dtype=torch.float64)
    D = s.hashgrid_levels * s.input_feature_dim
    Wm = Wl.view(O, D)

    # records used by the contributions, all grid points in one hashgrid call
    recs, rid = [], {}
    for pix, seq in st.items():
        for (q, ln, mg, _) in seq:
            if (q, pix) not in rid:
                rid[(q, pix)] = len(recs)
                recs.append((q, ln, mg))
    if not recs:
        recs.append((0, np.zeros(0, np.int32), np.zeros(0, np.float32)))  # keeps the shapes below non-empty
    lane_rec = np.concatenate([np.full(len(ln), r, np.int64) for r, (q, ln, mg) in enumerate(recs)])
    lane_q = np.concatenate([np.full(len(ln), q, np.int64) for (q, ln, mg) in recs])
    lane_g = np.concatenate([ln.astype(np.int64) for (q, ln, mg) in recs])
    lane_m = np.concatenate([mg.astype(np.float64) for (q, ln, mg) in recs])
    lq, lg = torch.tensor(lane_q), torch.tensor(lane_g)
    pos = m[lq] + offs[lg]
    phi = _hashgrid(pos, tab, s, lo, ext)
    w = c[lq, lg] * torch.tensor(lane_m, dtype=torch.float64)
    pre = torch.zeros(len(recs), O, dtype=torch.float64).index_add(0, torch.tensor(lane_rec),
                                                                   w[:, None] * (phi @ Wm.t())) + bl
    props = torch.cat([torch.sigmoid(pre[:, :O - 1]), torch.exp(pre[:, O - 1:])], 1)
    # compositing, all pixels at once, contributor slot by slot
    dep = view[2] * m[:, 0] + view[6] * m[:, 1] + view[10] * m[:, 2] + view[14]
    pixels = sorted(st)
    Kmax = max((len(st[p]) for p in pixels), default=0)
    npx = len(pixels)
    rec_ix = np.zeros((npx, Kmax), np.int64)
    q_ix = np.zeros((npx, Kmax), np.int64)
    tq_ix = np.zeros((npx, Kmax), np.int64)
    has_t = np.zeros((npx, Kmax), bool)
    valid = np.zeros((npx, Kmax), bool)
    for a, pix in enumerate(pixels):
        for k, (q, ln, mg, trig) in enumerate(st[pix]):
            rec_ix[a, k], q_ix[a, k], valid[a, k] = rid[(q, pix)], q, True
            tq_ix[a, k], has_t[a, k] = max(trig, 0), trig >= 0
    T = torch.ones(npx, dtype=torch.float64)
    C = torch.zeros(npx, 3, dtype=torch.float64)
    Fe = torch.zeros(npx, Fout, dtype=torch.float64)
    for k in range(Kmax):
        vk = torch.tensor(valid[:, k])
        pk = props[torch.tensor(rec_ix[:, k])]
        far = torch.full((npx,), float(s.max_distance), dtype=torch.float64)
        d_next = torch.where(torch.tensor(has_t[:, k]), dep[torch.tensor(tq_ix[:, k])], far)
        dt = d_next - dep[torch.tensor(q_ix[:, k])]
        a = torch.clamp(1 - torch.exp(-pk[:, O - 1] * dt), 0, 1)
        a = torch.where(vk, a, torch.zeros_like(a))
        C = C + (T * a)[:, None] * pk[:, :3]
        Fe = Fe + (T * a)[:, None] * pk[:, 3:3 + Fout]
        T = T * (1 - a)
    outC = bg.clamp(0, 1)[:, None].repeat(1, H * W).clone()
    outF = torch.zeros(Fout, H * W, dtype=torch.float64)
    vis = torch.zeros(H * W, dtype=torch.float64)
    if npx:
        ii = torch.tensor(pixels, dtype=torch.long)
        outC = outC.index_copy(1, ii, torch.clamp(C + T[:, None] * bg, 0, 1).t())
        if Fout:
            outF = outF.index_copy(1, ii, Fe.t())
        vis = vis.index_copy(0, ii, 1 - T)
    gc = torch.tensor(np.asarray(dcolor.detach().cpu()).reshape(3, -1), dtype=torch.float64)
    gf = torch.tensor(np.asarray(dfeat.detach().cpu()).reshape(Fout, H * W), dtype=torch.float64)
    gv = torch.tensor(np.asarray(dvis.detach().cpu()).reshape(-1), dtype=torch.float64)
    loss = (outC * gc).sum() + (outF * gf).sum() + (vis * gv).sum()
    loss.backward()
    images = dict(out_color=outC.detach().numpy().reshape(3, H, W),
                  out_features=outF.detach().numpy().reshape(Fout, H, W),
                  visibility=vis.detach().numpy().reshape(H, W))
    grads = dict(dL_dmeans3D=m.grad.numpy(), dL_dconfidences=c.grad.numpy(), dL_dfeature_table=tab.grad.numpy(),
                 dL_dlinear_weights=Wl.grad.numpy(), dL_dlinear_bias=bl.grad.numpy())
    return images, grads, f
