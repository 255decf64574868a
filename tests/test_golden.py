"""Pins the CPU oracle to the reference extension itself (CPU only).

The fixtures hold the outputs of the reference's own CUDA kernels, compiled from
its sources as shipped (-G) and with -O3, on fixed inputs (see
tests/golden/make_golden.py).  Binning fixtures cover preprocess, the offsets
scan, duplicateWithKeys, the CUB radix sort, identifyTileRanges and
checkFrustum; full fixtures cover the whole forward and backward on scenes on
which the reference render kernel is free of its barrier race.
"""
import numpy as np
import pytest

import golden_lib as gl
import oracle as orc
import vi_testlib as tl

B = gl.files("b")
F = gl.files("f")


def _oracle_binning(d):
    s = orc.Scene(d["means"], np.zeros((d["means"].shape[0], 27), np.float32), float(d["scale"]), d["viewmatrix"],
                  d["projmatrix"], float(d["tanfovx"]), float(d["tanfovy"]), int(d["height"]), int(d["width"]),
                  0.01, 100.0, np.zeros(8, np.float32), np.ones(1, np.int32), np.zeros(1, np.int32),
                  np.ones(3, np.int32), 1, np.zeros(8, np.float32), np.zeros(8, np.float32), 1, 3, 64,
                  np.zeros(3, np.float32), 2, 4, 1)
    pre = orc.preprocess(s)
    b = orc.binning(s, pre)
    b.update(pre)
    b["present"] = orc.mark_visible(d["means"], d["viewmatrix"])
    return b


@pytest.mark.skipif(not B, reason="no binning fixtures")
@pytest.mark.parametrize("path", B, ids=[gl.name(p) for p in B])
@pytest.mark.parametrize("build", gl.REF_BUILDS)
def test_oracle_binning_matches_reference(path, build):
    """Bit-exact against the reference as shipped (-G: no multiply-add
    contraction, the oracle's own arithmetic).  Against -O3, where nvcc fuses
    a*b+c, the integer results are still exact and only float bits move: depths
    (and so the low half of the keys) by at most 2 ulp, screen positions by a
    tiny absolute amount."""
    d = gl.load(path)
    o = _oracle_binning(d)
    R = int(d[f"{build}_num_rendered"])
    assert o["num_rendered"] == R
    np.testing.assert_array_equal(o["radii"], d[f"{build}_radii"])
    np.testing.assert_array_equal(o["tiles_touched"], d[f"{build}_tiles_touched"])
    np.testing.assert_array_equal(o["point_list"], d[f"{build}_point_list"])
    np.testing.assert_array_equal(o["ranges"], d[f"{build}_ranges"])
    np.testing.assert_array_equal(o["present"], d[f"{build}_present"])
    vis = o["radii"] > 0
    od, rd = o["depths"][vis], d[f"{build}_depths"][vis]
    om, rm = o["means2D"][vis], d[f"{build}_means2D"][vis]
    if build == "G":
        np.testing.assert_array_equal(od.view(np.uint32), rd.view(np.uint32))
        np.testing.assert_array_equal(om.view(np.uint32), rm.view(np.uint32))
        np.testing.assert_array_equal(o["keys"], d[f"{build}_keys"])
    else:
        ulp = np.abs(od.view(np.int32).astype(np.int64) - rd.view(np.int32).astype(np.int64))
        assert ulp.max(initial=0) <= 2
        assert np.abs(om - rm).max(initial=0.0) <= 1e-4
        ok, rk = o["keys"].astype(np.int64), d[f"{build}_keys"].astype(np.int64)
        np.testing.assert_array_equal(ok >> 32, rk >> 32)
        assert np.abs((ok & 0xFFFFFFFF) - (rk & 0xFFFFFFFF)).max(initial=0) <= 2


def _ref_state(d, build, K):
    g = {k: d[f"{build}_{k}"] for k in ("out_color", "out_features", "visibility", "final_T", "n_contrib",
                                         "contrib_idx", "delta_t", "ranges", "keys", "point_list", "radii")}
    g["num_rendered"] = int(d[f"{build}_num_rendered"])
    return g


@pytest.mark.skipif(not F, reason="no full fixtures")
@pytest.mark.parametrize("path", F, ids=[gl.name(p) for p in F])
@pytest.mark.parametrize("build", gl.REF_BUILDS)
def test_oracle_full_matches_reference(path, build):
    d = gl.load(path)
    s = orc.Scene(*gl.full_scene_args(d))
    f = orc.forward(s)
    assert int(f["skips"].sum()) == 0  # the scene is race-free for the reference kernel
    r = _ref_state(d, build, s.K)
    assert f["num_rendered"] == r["num_rendered"]
    np.testing.assert_array_equal(f["keys"], r["keys"])
    np.testing.assert_array_equal(f["point_list"], r["point_list"])
    np.testing.assert_array_equal(f["ranges"], r["ranges"])
    np.testing.assert_array_equal(f["n_contrib"], r["n_contrib"])
    used = (np.arange(s.K)[None, :] < f["n_contrib"][:, None]).reshape(-1)
    np.testing.assert_array_equal(f["contrib_idx"][used], r["contrib_idx"][used])
    np.testing.assert_allclose(f["delta_t"][used], r["delta_t"][used], rtol=0, atol=1e-6)
    tl.assert_images(f, r)
    g = orc.backward(s, f, f, d["dL_dcolor"], d["dL_dfeatures"], threads=1)
    ref_g = {k: d[f"{build}_{k}"] for k in ("dL_dmeans3D", "dL_dconfidences", "dL_dfeature_table",
                                            "dL_dlinear_weights", "dL_dlinear_bias")}
    tl.assert_grads(g, ref_g)
