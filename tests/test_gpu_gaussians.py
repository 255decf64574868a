"""GPU parity of the Gaussian front end (extension): the CUDA preprocess against
the oracle bit for bit, its backward against float64 autograd of the forward,
and the binning against the oracle's stable sort of tile << 32 | depth bits."""
import ctypes
import os

import numpy as np
import pytest
import torch

import gaussian_lib as gl
import gaussian_oracle as go

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "volume-integration_b200", "volume_integration", "libvi_b200.so")

# (P, sh_degree, M, seed, scene keyword arguments, scale_modifier)
CASES = [
    (1, 0, 1, 0, dict(), 1.0),
    (129, 1, 4, 1, dict(), 1.0),
    (1000, 2, 9, 2, dict(width=200, height=150), 0.7),
    (3000, 3, 16, 3, dict(), 1.0),
    (2048, 1, 16, 4, dict(extent=6.0), 1.2),                       # many culled; M > (deg+1)^2
    (5000, 3, 16, 5, dict(layout="mix", extent=10.0, dist=12.0, width=480, height=270, fov=50.0,
                          mu_scale=-5.0, sigma_scale=0.7), 1.0),  # headline-like distribution
    (700, 3, 16, 6, dict(mu_scale=-1.5, width=96, height=64), 1.0),  # large footprints
]


def _cam_settings(cam, deg, mod, dev):
    import volume_integration.gaussians as vg
    return vg.GaussianCamera(image_height=cam["image_height"], image_width=cam["image_width"],
                             tanfovx=cam["tanfovx"], tanfovy=cam["tanfovy"],
                             viewmatrix=cam["viewmatrix"].to(dev), projmatrix=cam["projmatrix"].to(dev),
                             campos=cam["cam_pos"].to(dev), sh_degree=deg, scale_modifier=mod)


def _oracle(means, scales, q, opac, shs, cam, deg, mod):
    return go.preprocess(means.numpy(), scales.numpy(), q.numpy(), opac.numpy(), shs.numpy(), deg, mod,
                         cam["viewmatrix"].numpy(), cam["projmatrix"].numpy(), cam["cam_pos"].numpy(),
                         cam["image_width"], cam["image_height"], cam["tanfovx"], cam["tanfovy"], 0.2)


@pytest.mark.parametrize("P,deg,M,seed,kw,mod", CASES)
def test_preprocess_bit_exact(P, deg, M, seed, kw, mod):
    import volume_integration.gaussians as vg
    dev = torch.device("cuda")
    means, scales, q, opac, shs, cam = gl.scene(P, deg, seed=seed, M=M, **kw)
    out = vg.preprocess_gaussians(means.to(dev), scales.to(dev), q.to(dev), opac.to(dev), shs.to(dev),
                                  _cam_settings(cam, deg, mod, dev))
    ref = _oracle(means, scales, q, opac, shs, cam, deg, mod)
    for k in ("radii", "means2D", "depths", "cov3D", "conic_opacity", "rgb", "tiles_touched"):
        got = getattr(out, k).cpu().numpy()
        np.testing.assert_array_equal(got, ref[k], err_msg=k)
    assert (ref["radii"] > 0).any()


@pytest.mark.parametrize("P,deg,M,seed,kw,mod", CASES)
def test_backward_matches_float64_autograd(P, deg, M, seed, kw, mod):
    import volume_integration.gaussians as vg
    dev = torch.device("cuda")
    means, scales, q, opac, shs, cam = gl.scene(P, deg, seed=seed, M=M, **kw)
    leaves = [x.to(dev).requires_grad_(True) for x in (means, scales, q, opac, shs)]
    out = vg.preprocess_gaussians(*leaves, _cam_settings(cam, deg, mod, dev))
    g = torch.Generator().manual_seed(100 + seed)
    gm2, gd, gcov = torch.randn(P, 2, generator=g), torch.randn(P, generator=g), torch.randn(P, 6, generator=g) * 1e2
    gco, grgb = torch.randn(P, 4, generator=g) * 1e-2, torch.randn(P, 3, generator=g)
    outs = (out.means2D, out.depths, out.cov3D, out.conic_opacity, out.rgb)
    grads = torch.autograd.grad(outs, leaves, [x.to(dev) for x in (gm2, gd, gcov, gco, grgb)])
    live = out.radii.cpu() > 0
    clamped = torch.from_numpy(_oracle(means, scales, q, opac, shs, cam, deg, mod)["clamped"].astype(bool))
    ref = gl.autograd_grads(means, scales, q, shs, cam, deg, mod, live, clamped, gm2, gd, gcov, gco[:, :3], grgb)
    for name, got, want in zip(("means3D", "scales", "rotations", "shs"), (grads[0], grads[1], grads[2], grads[4]),
                               ref):
        ok, worst = gl.rel_close(got.cpu().numpy(), want.numpy(), rtol=2e-3, atol_frac=2e-4)
        assert ok, (name, worst)
    want_op = torch.where(live, gco[:, 3], torch.zeros(P)).reshape(P, 1)
    torch.testing.assert_close(grads[3].cpu(), want_op)


@pytest.mark.parametrize("P,deg,M,seed,kw,mod", CASES)
def test_binning_bit_exact(P, deg, M, seed, kw, mod):
    import volume_integration.gaussians as vg
    dev = torch.device("cuda")
    means, scales, q, opac, shs, cam = gl.scene(P, deg, seed=seed, M=M, **kw)
    out = vg.preprocess_gaussians(means.to(dev), scales.to(dev), q.to(dev), opac.to(dev), shs.to(dev),
                                  _cam_settings(cam, deg, mod, dev))
    W, H = cam["image_width"], cam["image_height"]
    bins = vg.bin_gaussians(out, W, H)
    ref = _oracle(means, scales, q, opac, shs, cam, deg, mod)
    pl, tid, ranges = go.binning(ref["radii"], ref["means2D"], ref["depths"], ref["tiles_touched"], W, H)
    np.testing.assert_array_equal(bins.point_list.cpu().numpy(), pl)
    np.testing.assert_array_equal(bins.tile_ids.cpu().numpy(), tid)
    np.testing.assert_array_equal(bins.ranges.cpu().numpy(), ranges)


def test_empty_and_all_culled():
    import volume_integration.gaussians as vg
    dev = torch.device("cuda")
    means, scales, q, opac, shs, cam = gl.scene(50, 1, seed=9)
    cs = _cam_settings(cam, 1, 1.0, dev)
    e = vg.preprocess_gaussians(means[:0].to(dev), scales[:0].to(dev), q[:0].to(dev), opac[:0].to(dev),
                                shs[:0].to(dev), cs)
    assert e.radii.numel() == 0
    b = vg.bin_gaussians(e, cam["image_width"], cam["image_height"])
    assert b.point_list.numel() == 0 and int(b.ranges.abs().sum()) == 0
    behind = means.clone()
    behind[:, 2] = -10.0  # behind the camera at z = -4 looking at +z
    out = vg.preprocess_gaussians(behind.to(dev), scales.to(dev), q.to(dev), opac.to(dev), shs.to(dev), cs)
    assert int(out.radii.abs().sum()) == 0 and int(out.tiles_touched.sum()) == 0
    b = vg.bin_gaussians(out, cam["image_width"], cam["image_height"])
    assert b.point_list.numel() == 0


def test_binning_rejects_wrong_overlap_count():
    import volume_integration.gaussians as vg
    dev = torch.device("cuda")
    means, scales, q, opac, shs, cam = gl.scene(200, 0, seed=11)
    out = vg.preprocess_gaussians(means.to(dev), scales.to(dev), q.to(dev), opac.to(dev), shs.to(dev),
                                  _cam_settings(cam, 0, 1.0, dev))
    W, H = cam["image_width"], cam["image_height"]
    R = int(out.tiles_touched.sum())
    lib = ctypes.CDLL(LIB)
    lib.vi_bin_gaussians_scratch_bytes.restype = ctypes.c_uint64
    lib.vi_bin_gaussians_scratch_bytes.argtypes = [ctypes.c_int, ctypes.c_uint64, ctypes.c_int, ctypes.c_int]
    lib.vi_last_error.restype = ctypes.c_char_p
    wrong = R - 1
    nbytes = lib.vi_bin_gaussians_scratch_bytes(200, wrong, W, H)
    scratch = torch.empty(nbytes + 256, dtype=torch.uint8, device=dev)
    base = (scratch.data_ptr() + 255) // 256 * 256
    pl = torch.empty(max(wrong, 1), dtype=torch.int32, device=dev)
    ranges = torch.empty(((W + 15) // 16) * ((H + 15) // 16) * 2, dtype=torch.int32, device=dev)
    P_ = ctypes.c_void_p
    rc = lib.vi_bin_gaussians(ctypes.c_int(200), ctypes.c_int(W), ctypes.c_int(H), P_(out.radii.data_ptr()),
                              P_(out.means2D.data_ptr()), P_(out.depths.data_ptr()), P_(out.tiles_touched.data_ptr()),
                              ctypes.c_uint64(wrong), P_(base), ctypes.c_uint64(nbytes), P_(pl.data_ptr()), P_(None),
                              P_(ranges.data_ptr()), P_(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert rc != 0 and b"tiles touched sum" in lib.vi_last_error()
