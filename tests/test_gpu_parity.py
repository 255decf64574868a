"""CUDA path vs the CPU oracle on the same seeded inputs (needs a B200).

Integer state bit-exact, images within 1e-4, gradients within 1e-3 relative
(tolerances in vi_testlib).  The cases cover the configurations and edge cases
the renderer's settings allow: both stencils, every grid size the kernels map,
feature widths 1-8, 0-8 output features, the per-ray cap, background colour,
non power-of-two and dense-only tables, partial tiles, near-camera primitives
(forward and backward projections disagree), empty and culled scenes.
"""
import zlib

import numpy as np
import pytest
import torch

import vi_testlib as tl

pytestmark = pytest.mark.gpu


def _check(means, conf, s, seed=0, grads=True):
    dc, df = tl.random_grads(s, seed=seed)
    g = tl.run_gpu(means, conf, s, dc if grads else None, df if grads else None)
    _, o = tl.oracle_run(means, conf, s, dc if grads else None, df if grads else None, threads=8)
    tl.assert_integer_state(g, o, s.max_primitives_per_ray)
    tl.assert_images(g, o)
    if grads:
        tl.assert_grads(g["grads"], o["grads"])
    return g, o


@pytest.mark.parametrize("table_range", [1e-4, 1.0])
def test_tiny_config(table_range):
    means, conf, s = tl.scene("tiny", table_range=table_range)
    g, o = _check(means, conf, s)
    assert g["num_rendered"] > 10000


CUSTOM = {
    "default": {},
    "genus2": dict(genus=2),
    "grid2": dict(G=2),
    "grid1": dict(G=1),
    "F4L8": dict(F=4, L=8),
    "F4L16_D64": dict(F=4, L=16),
    "F1L16": dict(F=1, L=16),
    "F8L4": dict(F=8, L=4),
    "fout0": dict(Fout=0),
    "fout2": dict(Fout=2),
    "fout8_o12": dict(Fout=8),
    "K1": dict(K=1),
    "K3": dict(K=3),
    "bg": dict(bg=(0.2, 0.5, 0.9)),
    "T_not_pow2": dict(T=3001, log2_T=11),
    "dense_levels": dict(L=4, base=4, growth=1.5, log2_T=16),
    "ragged_image": dict(W=70, H=45),
    "neg_conf": dict(mu_conf=-1.5),
    "pos_conf": dict(mu_conf=3.0),
    "big_primitives": dict(scale=0.9, P=120),
    "near_camera": dict(dist=1.2, extent=0.8, scale=0.3),
    "dense_overlap": dict(P=2000, scale=0.15, extent=0.7),
    "tiny_table_range": dict(table_range=1e-4),
    # grids of 4^3 and 5^3 points (the reference's MAX_GRID_SIZE is 5)
    "grid4": dict(G=4),
    "grid5": dict(G=5),
    "grid4_genus2": dict(G=4, genus=2),
    "grid5_genus2": dict(G=5, genus=2, P=150),
    "grid5_F4L16_D64": dict(G=5, F=4, L=16),
    "grid4_fout8_o12": dict(G=4, Fout=8),
    "grid4_K3": dict(G=4, K=3),
    "grid5_near_camera": dict(G=5, dist=1.2, extent=0.8, scale=0.3),
    "grid4_dense_overlap": dict(G=4, P=1500, scale=0.15, extent=0.7),
    "grid5_T_not_pow2": dict(G=5, T=3001, log2_T=11),
}


@pytest.mark.parametrize("name", sorted(CUSTOM))
def test_custom(name):
    means, conf, s = tl.custom_scene(seed=zlib.crc32(name.encode()) % 1000, **CUSTOM[name])
    _check(means, conf, s, seed=3)


def _projection_crossings(s, n=4_000_000, seed=0):
    """World points (float32) whose pixel under the forward's 1/(w + 1e-7)
    projection differs from the backward's 1/w one (forward.cu:432,
    backward.cu:325), found by sampling the view at depths 0.25-0.6 with the
    kernels' float32 operation order."""
    f32 = np.float32
    W, H = s.image_width, s.image_height
    pm = s.projmatrix.cpu().numpy().reshape(16).astype(np.float32)
    vm = s.viewmatrix.cpu().numpy().reshape(16).astype(np.float32)
    eye = s.cam_pos.cpu().numpy().astype(np.float64)
    rows = np.array([[vm[0], vm[4], vm[8]], [vm[1], vm[5], vm[9]], [vm[2], vm[6], vm[10]]], np.float64)
    rng = np.random.default_rng(seed)
    d = rng.uniform(0.25, 0.6, n)
    cam = np.stack([rng.uniform(-1, 1, n) * d * s.tanfovx, rng.uniform(-1, 1, n) * d * s.tanfovy, d], 1)
    p = (eye[None, :] + cam @ rows).astype(np.float32)

    def pixel(fwd):
        hx = ((pm[0] * p[:, 0] + pm[4] * p[:, 1]) + pm[8] * p[:, 2]) + pm[12]
        hy = ((pm[1] * p[:, 0] + pm[5] * p[:, 1]) + pm[9] * p[:, 2]) + pm[13]
        hw = ((pm[3] * p[:, 0] + pm[7] * p[:, 1]) + pm[11] * p[:, 2]) + pm[15]
        pw = f32(1) / (hw + f32(1e-7)) if fwd else f32(1) / hw
        n2p = lambda q, S: (((q.astype(np.float64) + 1) * S - 1) * 0.5).astype(np.float32)
        return np.floor(n2p(hx * pw, W)), np.floor(n2p(hy * pw, H))
    (ax, ay), (bx, by) = pixel(True), pixel(False)
    return p[(ax != bx) | (ay != by)]


def test_backward_recompute_of_records_whose_projection_differs():
    # Primitives centred on points that the backward's 1/w projection puts in
    # another pixel than the forward's 1/(w + 1e-7): their records are
    # re-derived before the per-pixel pass (recompute_records_kernel), and the
    # gradients must match the oracle's backward, which recomputes them too.
    means, conf, s = tl.custom_scene(seed=41, P=300, W=256, H=256, fov=90.0, dist=0.05, extent=0.4, scale=0.05,
                                     mu_conf=1.5)
    pts = _projection_crossings(s)
    assert len(pts) >= 20
    means = means.clone()
    means[:20] = torch.from_numpy(pts[:20]).to(means.device)
    g, o = _check(means, conf, s, seed=5)
    flagged = (g["rec_cnt"].view(np.uint32) >> 31) & 1
    assert flagged[:20].sum() >= 10, flagged[:20]


def test_single_primitive():
    means, conf, s = tl.custom_scene(P=1, scale=0.8, mu_conf=2.0)
    g, o = _check(means, conf, s)
    assert g["num_rendered"] >= 1


def test_empty_scene():
    means, conf, s = tl.custom_scene(P=0)
    import volume_integration as vi
    oc, of, vis = vi.integrate_primitives(means, conf, s.feature_table, s.linear_weights, s.linear_bias, s)
    assert float(oc.abs().sum()) == 0.0 and float(vis.abs().sum()) == 0.0
    R = tl.raw_forward(means, conf, s)[0]
    assert R == 0


def test_all_behind_camera():
    means, conf, s = tl.custom_scene(P=50)
    means = means.clone()
    means[:, 2] = -10.0  # camera sits at z=-3 looking at +z: all primitives are behind it
    g, o = _check(means, conf, s)
    assert g["num_rendered"] == 0
    assert np.all(g["n_contrib"] == 0)


def test_depth_ties_keep_index_order():
    # Every primitive at the same depth: ties must keep primitive-index order (stable sort).
    means, conf, s = tl.custom_scene(P=400, scale=0.2)
    means = means.clone()
    means[:, 2] = 0.25
    _check(means, conf, s)


def test_4d_confidences_and_needs_grad_subset():
    import volume_integration as vi
    means, conf, s = tl.custom_scene(P=200)
    G = s.grid_size
    c4 = conf.view(-1, G, G, G).clone().requires_grad_(True)
    t = s.feature_table.clone().requires_grad_(True)
    oc, of, vis = vi.integrate_primitives(means, c4, t, s.linear_weights, s.linear_bias, s)
    (oc.sum() + of.sum()).backward()
    assert c4.grad.shape == c4.shape and t.grad.shape == t.shape


def test_module_and_mark_visible():
    import volume_integration as vi
    import oracle as orc
    means, conf, s = tl.custom_scene(P=500, extent=3.0)
    mod = vi.VolumeIntegrator(s)
    got = mod.markVisible(means).cpu().numpy()
    exp = orc.mark_visible(means.cpu().numpy(), s.viewmatrix.cpu().numpy())
    np.testing.assert_array_equal(got, exp)
    oc, of, vis = mod(means, conf)
    assert oc.shape == (3, s.image_height, s.image_width)


def test_repeat_calls_are_deterministic_forward():
    means, conf, s = tl.scene("tiny", table_range=1.0)
    a = tl.gpu_state(means, conf, s)
    b = tl.gpu_state(means, conf, s)
    for k in ("keys", "point_list", "ranges", "n_contrib", "final_T"):
        np.testing.assert_array_equal(a[k], b[k])


@pytest.mark.parametrize("n,begin,end", [(1, 0, 64), (1000, 0, 45), (100_000, 0, 64), (262_144, 8, 40),
                                         (1_000_003, 0, 37)])
def test_sort_pairs_matches_stable_argsort(n, begin, end):
    from volume_integration import _C
    gen = torch.Generator().manual_seed(n)
    keys = torch.randint(-(2 ** 62), 2 ** 62, (n,), generator=gen, dtype=torch.int64)
    keys[: n // 3] = keys[0]  # many duplicates to exercise stability
    vals = torch.arange(n, dtype=torch.int32)
    ks, vs = _C.sort_pairs(keys.cuda(), vals.cuda(), begin, end)
    k = keys.numpy().view(np.uint64)
    width = end - begin
    digit = (k >> np.uint64(begin)) & (np.uint64((1 << width) - 1) if width < 64 else np.uint64(0xFFFFFFFFFFFFFFFF))
    order = np.argsort(digit, kind="stable")
    np.testing.assert_array_equal(vs.cpu().numpy(), vals.numpy()[order])
    np.testing.assert_array_equal(ks.cpu().numpy().view(np.uint64), k[order])


# Hashgrid box other than the reference's fixed [-1.3, 1.3]^3 (an extension):
# parity with the oracle under the same box, and the reference box given
# explicitly must reproduce the default call bit for bit.
HASH_BOUNDS = {
    "inside": dict(extent=1.0, bounds=(-1.1, -1.2, -1.0, 1.05, 1.15, 0.9)),
    # big overlapping primitives: table values of the benchmark scenes keep the
    # densities (and with them the transmittance cut-offs) away from saturation
    "scene_aabb": dict(extent=3.0, scale=0.4, dist=8.0, table_range=1e-4, bounds=None),
    "anisotropic": dict(extent=1.0, bounds=(-0.5, -2.0, -1.0, 0.5, 2.0, 3.0)),
}


@pytest.mark.parametrize("name", sorted(HASH_BOUNDS))
def test_hash_bounds(name):
    import dataclasses
    cfg = dict(HASH_BOUNDS[name])
    bounds = cfg.pop("bounds")
    means, conf, s = tl.custom_scene(seed=zlib.crc32(name.encode()) % 1000, **cfg)
    if bounds is None:  # the scene's own box, padded by half a primitive
        lo = (means.min(0).values - s.primitive_scale).tolist()
        hi = (means.max(0).values + s.primitive_scale).tolist()
        bounds = tuple(lo + hi)
    s = dataclasses.replace(s, hash_bounds=bounds)
    g, o = _check(means, conf, s, seed=5)
    assert g["num_rendered"] > 0


def test_hash_bounds_reference_box_is_the_default():
    import dataclasses
    means, conf, s = tl.custom_scene(seed=11, extent=2.0)
    dc, df = tl.random_grads(s, seed=2)
    a = tl.run_gpu(means, conf, s, dc, df, state=False)
    b = tl.run_gpu(means, conf, dataclasses.replace(s, hash_bounds=(-1.3, -1.3, -1.3, 1.3, 1.3, 1.3)), dc, df,
                   state=False)
    for k in ("out_color", "out_features", "visibility"):
        np.testing.assert_array_equal(a[k], b[k])
    tl.assert_grads(a["grads"], b["grads"])  # atomic summation order differs between calls


def test_hash_bounds_rejects_an_empty_box():
    import dataclasses
    import volume_integration as vi
    means, conf, s = tl.custom_scene(seed=12)
    s = dataclasses.replace(s, hash_bounds=(0.0, 0.0, 0.0, 1.0, -1.0, 1.0))
    with pytest.raises(RuntimeError, match="hash_bounds"):
        vi.integrate_primitives(means, conf, s.feature_table, s.linear_weights, s.linear_bias, s)


# The backward reads the hashgrid features of each position class from a cache
# the feature stage fills; primitives that find no room gather them again.
# VI_PHI_CACHE_BYTES bounds the cache: 0 = no cache, a small bound = a mix.
@pytest.mark.parametrize("limit", ["0", "20000"])
def test_feature_cache_fallback(limit, monkeypatch):
    monkeypatch.setenv("VI_PHI_CACHE_BYTES", limit)
    means, conf, s = tl.custom_scene(seed=21, P=400, extent=1.0)
    _check(means, conf, s, seed=7)
    means, conf, s = tl.scene("tiny", table_range=1.0)
    _check(means, conf, s, seed=8)


@pytest.mark.parametrize("name", ["default", "dense_overlap", "fout8_o12", "K3"])
def test_render_with_record_staging(name, monkeypatch):
    # the render reads records from global memory by default; the form that
    # stages each batch's records with bulk copies (VI_RENDER_TMA=1, read at
    # every launch) must give the same results
    monkeypatch.setenv("VI_RENDER_TMA", "1")
    means, conf, s = tl.custom_scene(seed=zlib.crc32(name.encode()) % 1000, **CUSTOM[name])
    _check(means, conf, s, seed=3)


@pytest.mark.parametrize("name", ["default", "grid5", "T_not_pow2", "F4L16_D64", "dense_levels"])
def test_feature_stage_on_callers_table_layout(name, monkeypatch):
    # the feature stage reads a level-major copy of the table by default; with
    # VI_TABLE_LAYOUT=entry (read at every forward) it reads the caller's
    # entry-major table, with the same results
    monkeypatch.setenv("VI_TABLE_LAYOUT", "entry")
    means, conf, s = tl.custom_scene(seed=zlib.crc32(name.encode()) % 1000, **CUSTOM[name])
    _check(means, conf, s, seed=5)


# Primitives spread over [-3, 3]^3 with the reference's fixed hashgrid box
# [-1.3, 1.3]^3: about one in seven has every grid point clamped to one corner of
# the box.  The backward hands those to backward_corner_kernel and the rest to
# backward_prim_kernel; these cases run both across grid sizes, feature widths
# and output widths (the benchmark scenes cover G = 3, F = 2 and 4, O = 8 only).
CORNER = {
    "corner_G3": dict(),
    "corner_G2": dict(G=2),
    "corner_G1": dict(G=1),
    "corner_fout8_o12": dict(Fout=8),
    "corner_F4L16_D64": dict(F=4, L=16),
    "corner_F1L16": dict(F=1, L=16),
    "corner_F8L4": dict(F=8, L=4),
    "corner_K3": dict(K=3),
}


@pytest.mark.parametrize("name", sorted(CORNER))
def test_box_corner_primitives(name):
    kw = dict(P=600, extent=3.0, dist=9.0, scale=0.25, W=96, H=72)
    kw.update(CORNER[name])
    means, conf, s = tl.custom_scene(seed=zlib.crc32(name.encode()) % 1000, **kw)
    # every grid point lies within scale/2 of the centre on each axis
    clamped = (means.abs().cpu() > 1.3 + 0.5 * kw["scale"] + 1e-4).all(dim=1)
    assert int(clamped.sum()) > 40
    _check(means, conf, s, seed=11)
