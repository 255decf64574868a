"""CPU tests of the Gaussian front end's oracle (oracle/gaussian_oracle.py):
known answers of the EWA projection and the spherical harmonics, agreement with
the float64 torch restatement whose autograd checks the CUDA backward, culling,
and the binning's sort order."""
import numpy as np
import torch

import gaussian_lib as gl
import gaussian_oracle as go
import vi_workloads as wl


def _run(means, scales, q, opac, shs, cam, deg, mod=1.0, near=0.2):
    return go.preprocess(means.numpy(), scales.numpy(), q.numpy(), opac.numpy(), shs.numpy(), deg, mod,
                         cam["viewmatrix"].numpy(), cam["projmatrix"].numpy(), cam["cam_pos"].numpy(),
                         cam["image_width"], cam["image_height"], cam["tanfovx"], cam["tanfovy"], near)


def test_isotropic_gaussian_on_the_axis_known_answer():
    # camera on -z looking at the origin; an isotropic Gaussian at the origin:
    # Sigma = s^2 I, so cov2D = diag(fx^2, fy^2) s^2 / d^2 + 0.3 and b = 0
    d, s, W, H = 4.0, 0.05, 160, 120
    cam = wl.camera((0.0, 0.0, -d), W, H, 60.0)
    means = torch.zeros(1, 3)
    scales = torch.full((1, 3), s)
    q = torch.tensor([[1.0, 0.0, 0.0, 0.0]])
    shs = torch.zeros(1, 1, 3)
    out = _run(means, scales, q, torch.ones(1, 1), shs, cam, 0)
    fx = W / (2 * cam["tanfovx"])
    fy = H / (2 * cam["tanfovy"])
    a, c = fx ** 2 * s ** 2 / d ** 2 + 0.3, fy ** 2 * s ** 2 / d ** 2 + 0.3
    np.testing.assert_allclose(out["conic_opacity"][0], [1 / a, 0.0, 1 / c, 1.0], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(out["cov3D"][0], [s * s, 0, 0, s * s, 0, s * s], rtol=1e-6, atol=1e-9)
    assert out["radii"][0] == int(np.ceil(3 * np.sqrt(max(a, c))))
    np.testing.assert_allclose(out["means2D"][0], [(W - 1) / 2, (H - 1) / 2], atol=1e-4)
    assert out["depths"][0] == np.float32(d)
    # degree 0: rgb = C0 * 0 + 0.5
    np.testing.assert_array_equal(out["rgb"][0], [0.5, 0.5, 0.5])


def test_sh_degree_zero_and_clamp():
    means, scales, q, opac, shs, cam = gl.scene(64, 0, seed=3)
    shs = shs * 20  # drives some channels below zero
    out = _run(means, scales, q, opac, shs, cam, 0)
    live = out["radii"] > 0
    col = go.C0 * shs.numpy()[:, 0, :] + np.float32(0.5)
    np.testing.assert_array_equal(out["rgb"][live], np.maximum(col, 0)[live])
    np.testing.assert_array_equal(out["clamped"][live], (col < 0)[live].astype(np.uint8))
    assert out["clamped"][live].any()


def test_oracle_matches_float64_restatement():
    for deg in range(4):
        means, scales, q, opac, shs, cam = gl.scene(300, deg, seed=10 + deg)
        out = _run(means, scales, q, opac, shs, cam, deg, mod=1.3)
        live = torch.from_numpy(out["radii"] > 0)
        assert 50 < int(live.sum()) <= 300
        clamped = torch.from_numpy(out["clamped"].astype(bool))
        m2, dep, cov, con, rgb = gl.forward64(means.double(), scales.double(), q.double(), shs.double(), cam, deg,
                                              1.3, live, clamped)
        np.testing.assert_allclose(out["means2D"], m2.numpy(), rtol=1e-5, atol=1e-3)
        np.testing.assert_allclose(out["depths"], dep.numpy(), rtol=1e-6)
        np.testing.assert_allclose(out["cov3D"], cov.numpy(), rtol=1e-4, atol=1e-5 * np.abs(cov.numpy()).max())
        np.testing.assert_allclose(out["conic_opacity"][:, :3], con.numpy(), rtol=2e-3,
                                   atol=2e-4 * np.abs(con.numpy()).max())
        np.testing.assert_allclose(out["rgb"], rgb.numpy(), rtol=1e-5, atol=1e-6)


def test_culling_behind_camera_and_outputs_zero():
    means, scales, q, opac, shs, cam = gl.scene(200, 1, seed=5, extent=8.0)
    out = _run(means, scales, q, opac, shs, cam, 1)
    dead = out["radii"] == 0
    assert dead.any() and (~dead).any()
    for k in ("means2D", "depths", "cov3D", "conic_opacity", "rgb", "clamped", "tiles_touched"):
        assert not np.any(out[k][dead]), k
    # everything behind the camera (view z <= near) is culled
    V = cam["viewmatrix"].numpy().reshape(16)
    tz = means.numpy() @ V[[2, 6, 10]] + V[14]
    assert np.all(dead[tz <= 0.2])


def test_binning_order_and_ranges():
    means, scales, q, opac, shs, cam = gl.scene(400, 0, seed=7, mu_scale=-2.5)
    out = _run(means, scales, q, opac, shs, cam, 0)
    W, H = cam["image_width"], cam["image_height"]
    pl, tid, ranges = go.binning(out["radii"], out["means2D"], out["depths"], out["tiles_touched"], W, H)
    assert pl.size == int(out["tiles_touched"].sum())
    assert np.all(np.diff(tid) >= 0)
    dep = out["depths"][pl]
    for t in np.unique(tid):
        a, b = ranges[t]
        assert np.all(tid[a:b] == t)
        seg, ids = dep[a:b], pl[a:b]
        assert np.all((np.diff(seg) > 0) | ((np.diff(seg) == 0) & (np.diff(ids) > 0)))
    assert int((ranges[:, 1] - ranges[:, 0]).sum()) == pl.size


def test_c_abi_rejects_bad_sh_settings_without_gpu():
    import ctypes
    import os
    lib = ctypes.CDLL(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                   "volume-integration_b200", "volume_integration", "libvi_b200.so"))
    lib.vi_last_error.restype = ctypes.c_char_p
    f = ctypes.c_float
    cam = (f * 3)(0.0, 0.0, 0.0)
    null = ctypes.c_void_p(None)

    def call(deg, M):
        return lib.vi_preprocess_gaussians(1, deg, M, null, null, null, null, null, f(1.0), null, null, cam,
                                           64, 64, f(0.5), f(0.5), f(0.2), null, null, null, null, null, null,
                                           null, null, null)
    assert call(4, 25) == 2 and b"sh_degree" in lib.vi_last_error()          # VI_ERR_UNSUPPORTED
    assert call(2, 4) == 1 and b"SH coefficients" in lib.vi_last_error()     # VI_ERR_INVALID_ARGUMENT
    assert call(1, 4) == 1 and b"pointer" in lib.vi_last_error()             # camera pointers NULL
