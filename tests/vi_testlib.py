"""Helpers shared by the tests: build a scene, run the CUDA path and the CPU
oracle on the same inputs, and compare them with the stated tolerances:

* integer state (radii, tiles, sorted keys / point list, tile ranges, per-pixel
  contributor lists) and depths / delta_t: bit-exact;
* images and final transmittance: max |a - b| <= 1e-4 (fp32);
* gradients: ||a - b|| / ||b|| <= 1e-3 and per element
  |a - b| <= 1e-3 * max|b| + 1e-6, because atomic summation order differs.
"""
import numpy as np
import torch

import oracle as orc
import vi_workloads as wl

IMG_TOL = 1e-4
GRAD_REL = 1e-3


def settings_from(kw, cam, device):
    import volume_integration as vi
    d = {}
    for k, v in kw.items():
        d[k] = v.to(device) if isinstance(v, torch.Tensor) else v
    for k, v in cam.items():
        d[k] = v.to(device) if isinstance(v, torch.Tensor) else v
    return vi.IntegrationSettings(**d)


def scene(name="tiny", view=0, device="cuda", table_range=1e-4, seed=None, **over):
    means, conf, kw, cams = wl.make(name, table_range=table_range, seed=seed, **over)
    s = settings_from(kw, cams[view], device)
    return means.to(device), conf.to(device), s


def custom_scene(P=300, W=64, H=48, L=16, F=2, log2_T=12, base=4, growth=1.5, Fout=4, G=3, genus=1, K=64,
                 scale=0.25, extent=1.0, dist=3.0, fov=50.0, mu_conf=0.5, table_range=1.0, bg=(0.0, 0.0, 0.0),
                 seed=0, T=None, device="cuda"):
    """A small random scene with every knob exposed (for edge-case parity tests)."""
    import math
    gen = torch.Generator().manual_seed(seed)
    means = (torch.rand(P, 3, generator=gen) * 2 - 1) * extent
    conf = torch.randn(P, G ** 3, generator=gen) + mu_conf
    hg = wl.hashgrid(L, F, log2_T, base, growth)
    if T is not None:  # arbitrary (non power of two) table size
        hg["feature_offset"] = T
        hg["do_hash"] = torch.tensor([1 if (r + 1) ** 3 > T else 0 for r in hg["resolution"].tolist()],
                                     dtype=torch.int32)
    D, O = L * F, Fout + 4
    table = (torch.rand(hg["feature_offset"] * L * F, generator=gen) * 2 - 1) * table_range
    Wl, bl = wl.linear_layer(D, O, gen)
    cam = wl.camera((0.3, -0.4, -dist), W, H, fov)
    kw = dict(near_plane=0.01, max_distance=100.0, primitive_scale=scale, feature_table=table,
              linear_weights=Wl, linear_bias=bl, stencil_genus=genus, grid_size=G, max_primitives_per_ray=K,
              occupancy_threshold=0.5, bg_color=torch.tensor(bg, dtype=torch.float32),
              output_feature_dim=Fout, num_output_channels=3, debug=True)
    kw.update(hg)
    s = settings_from(kw, cam, device)
    return means.to(device), conf.to(device), s


def oracle_scene(means, conf, s):
    return orc.Scene.from_settings(means, conf, s)


def run_gpu(means, conf, s, dcolor=None, dfeat=None, state=True):
    """Forward (+ backward if dcolor is given) through the autograd Function."""
    import volume_integration as vi
    from volume_integration import _C
    m = means.clone().requires_grad_(True)
    c = conf.clone().requires_grad_(True)
    t = s.feature_table.clone().requires_grad_(True)
    Wl = s.linear_weights.clone().requires_grad_(True)
    bl = s.linear_bias.clone().requires_grad_(True)
    out_color, out_feat, vis = vi.integrate_primitives(m, c, t, Wl, bl, s)
    res = dict(out_color=out_color.detach().cpu().numpy(), out_features=out_feat.detach().cpu().numpy(),
               visibility=vis.detach().cpu().numpy())
    if state:
        res.update(gpu_state(means, conf, s))
    if dcolor is not None:
        loss = (out_color * dcolor).sum() + (out_feat * dfeat).sum()
        loss.backward()
        res["grads"] = dict(dL_dmeans3D=m.grad.cpu().numpy(), dL_dconfidences=c.grad.cpu().numpy(),
                            dL_dfeature_table=t.grad.cpu().numpy(), dL_dlinear_weights=Wl.grad.cpu().numpy(),
                            dL_dlinear_bias=bl.grad.cpu().numpy())
    torch.cuda.synchronize()
    return res


def raw_forward(means, conf, s):
    """Positional call of _C.integrate_primitives, exactly as the reference's Python layer makes it
    (integrate_primitives_ex with the same arguments when the settings carry the hash_bounds or
    exact_gradients extensions)."""
    import volume_integration as vi
    from volume_integration import _C
    G = s.grid_size
    hb, flags = vi._hash_bounds(s), vi._flags(s)
    fn = _C.integrate_primitives if hb is None and not flags else \
        (lambda *a: _C.integrate_primitives_ex(*a, hb or [], flags))
    return fn(
        means.contiguous().float(), conf.reshape(means.shape[0], G ** 3).contiguous().float(), s.primitive_scale,
        s.viewmatrix, s.projmatrix, s.cam_pos, s.tanfovx, s.tanfovy, s.image_height, s.image_width, s.near_plane,
        s.max_distance, s.feature_table, s.resolution, s.do_hash, s.primes, s.feature_offset, s.linear_weights,
        s.linear_bias, s.stencil_genus, s.grid_size, s.max_primitives_per_ray, s.occupancy_threshold, s.bg_color,
        s.input_feature_dim, s.output_feature_dim, s.intermediate_feature_dim, s.hashgrid_levels,
        s.num_output_channels, s.debug)


def gpu_state(means, conf, s):
    from volume_integration import _C
    R, oc, of, vis, geom, binning, img = raw_forward(means, conf, s)
    v = _C.state_views(geom, binning, img, means.shape[0], R, s.image_height, s.image_width,
                       s.max_primitives_per_ray, s.grid_size, s.output_feature_dim)
    out = {k: t.cpu().numpy() for k, t in v.items()}
    out["num_rendered"] = R
    if R > 0:
        pl = out["point_list"].astype(np.int64)
        dbits = out["depths"].view(np.uint32).astype(np.uint64)
        out["keys"] = (out["sorted_tiles"].astype(np.uint64) << np.uint64(32)) | dbits[pl]
    return out


def oracle_run(means, conf, s, dcolor=None, dfeat=None, threads=0, tile_mask=None):
    sc = oracle_scene(means, conf, s)
    f = orc.forward(sc, tile_mask=tile_mask, threads=threads)
    if dcolor is not None:
        dc = dcolor.detach().cpu().numpy() if torch.is_tensor(dcolor) else dcolor
        df = dfeat.detach().cpu().numpy() if torch.is_tensor(dfeat) else dfeat
        f["grads"] = orc.backward(sc, f, f, dc, df, tile_mask=tile_mask, threads=threads)
    return sc, f


def assert_integer_state(g, o, K):
    assert g["num_rendered"] == o["num_rendered"], (g["num_rendered"], o["num_rendered"])
    np.testing.assert_array_equal(g["radii"], o["radii"])
    np.testing.assert_array_equal(g["tiles_touched"].view(np.uint32), o["tiles_touched"])
    vis = o["radii"] > 0
    np.testing.assert_array_equal(g["depths"][vis].view(np.uint32), o["depths"][vis].view(np.uint32))
    np.testing.assert_array_equal(g["means2D"][vis].view(np.uint32), o["means2D"][vis].view(np.uint32))
    if o["num_rendered"] > 0:
        np.testing.assert_array_equal(g["keys"], o["keys"])
        np.testing.assert_array_equal(g["point_list"].view(np.uint32), o["point_list"])
    np.testing.assert_array_equal(g["ranges"].view(np.uint32), o["ranges"])
    np.testing.assert_array_equal(g["n_contrib"], o["n_contrib"])
    N = g["n_contrib"].shape[0]
    k = np.arange(K)[None, :]
    used = (k < o["n_contrib"][:, None]).reshape(-1)
    np.testing.assert_array_equal(g["contrib_idx"].reshape(N * K)[used], o["contrib_idx"][used])
    np.testing.assert_array_equal(g["delta_t"].reshape(N * K)[used].view(np.uint32),
                                  o["delta_t"][used].view(np.uint32))


def assert_images(g, o):
    for k in ("out_color", "out_features", "visibility"):
        a, b = np.asarray(g[k]), np.asarray(o[k])
        assert a.shape == b.shape, (k, a.shape, b.shape)
        if a.size:
            err = float(np.abs(a - b).max())
            assert err <= IMG_TOL, f"{k}: max abs err {err}"
    if "final_T" in g:
        err = float(np.abs(g["final_T"] - o["final_T"]).max()) if g["final_T"].size else 0.0
        assert err <= IMG_TOL, f"final_T: max abs err {err}"


def grad_errors(a, b):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    nb = np.linalg.norm(b)
    rel = np.linalg.norm(a - b) / nb if nb > 0 else np.linalg.norm(a - b)
    scale = np.abs(b).max() if b.size else 0.0
    elem = np.abs(a - b).max() / (scale + 1e-12) if b.size else 0.0
    return rel, elem, scale


def assert_grads(g, o):
    for k in ("dL_dmeans3D", "dL_dconfidences", "dL_dfeature_table", "dL_dlinear_weights", "dL_dlinear_bias"):
        a, b = g[k], o[k]
        assert np.asarray(a).size == np.asarray(b).size, k
        rel, elem, scale = grad_errors(a, b)
        if scale == 0.0:
            assert np.abs(np.asarray(a)).max() <= 1e-6 if np.asarray(a).size else True, k
            continue
        assert rel <= GRAD_REL, f"{k}: relative error {rel}"
        absdiff = np.abs(np.asarray(a, np.float64).reshape(-1) - np.asarray(b, np.float64).reshape(-1)).max()
        assert absdiff <= GRAD_REL * scale + 1e-6, f"{k}: max abs diff {absdiff} (scale {scale})"


def random_grads(s, seed=0, device="cuda"):
    gen = torch.Generator().manual_seed(seed)
    dc = torch.randn(3, s.image_height, s.image_width, generator=gen)
    df = torch.randn(s.output_feature_dim, s.image_height, s.image_width, generator=gen)
    return dc.to(device), df.to(device)
