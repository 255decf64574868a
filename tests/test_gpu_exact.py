"""Exact-gradient mode (an extension; IntegrationSettings.exact_gradients) on
the GPU against the float64 autograd of the forward on the oracle's discrete
structure (tests/exact_lib.py): images within 1e-4, every gradient, dL/dmeans3D
included, within the parity tolerance (1e-3 relative)."""
import dataclasses
import zlib

import numpy as np
import pytest
import torch

import exact_lib as ex
import vi_testlib as tl

pytestmark = pytest.mark.gpu

CASES = {
    "default": dict(P=60, W=48, H=32),
    "bg_and_features": dict(P=60, W=48, H=32, bg=(0.2, 0.5, 0.9), Fout=2),
    "no_features": dict(P=60, W=48, H=32, Fout=0),
    "dense_overlap": dict(P=150, W=64, H=48, scale=0.15, extent=0.7),
    "K3": dict(P=80, W=48, H=32, K=3),
    "dense_levels": dict(P=60, W=48, H=32, L=4, base=4, growth=1.5, log2_T=16),
}


def _gpu(means, conf, s, dc, df, dv):
    import volume_integration as vi
    m = means.clone().requires_grad_(True)
    c = conf.clone().requires_grad_(True)
    t = s.feature_table.clone().requires_grad_(True)
    w = s.linear_weights.clone().requires_grad_(True)
    b = s.linear_bias.clone().requires_grad_(True)
    oc, of, vis = vi.integrate_primitives(m, c, t, w, b, s)
    ((oc * dc).sum() + (of * df).sum() + (vis * dv).sum()).backward()
    torch.cuda.synchronize()
    img = dict(out_color=oc.detach().cpu().numpy(), out_features=of.detach().cpu().numpy(),
               visibility=vis.detach().cpu().numpy())
    grads = dict(dL_dmeans3D=m.grad.cpu().numpy(), dL_dconfidences=c.grad.cpu().numpy(),
                 dL_dfeature_table=t.grad.cpu().numpy(), dL_dlinear_weights=w.grad.cpu().numpy(),
                 dL_dlinear_bias=b.grad.cpu().numpy())
    return img, grads


@pytest.mark.parametrize("name", sorted(CASES))
def test_exact_gradients(name):
    means, conf, s = tl.custom_scene(seed=zlib.crc32(name.encode()) % 1000, **CASES[name])
    s = dataclasses.replace(s, exact_gradients=True)
    dc, df = tl.random_grads(s, seed=4)
    dv = torch.randn(s.image_height, s.image_width, generator=torch.Generator().manual_seed(9)).cuda()
    img, grads = _gpu(means, conf, s, dc, df, dv)
    rimg, rgrads, _ = ex.exact_grads(means, conf, s, dc, df, dv)
    for k in img:
        np.testing.assert_allclose(img[k], rimg[k], atol=1e-4, err_msg=k)
    assert np.abs(rgrads["dL_dmeans3D"]).max() > 0
    tl.assert_grads(grads, rgrads)


def test_exact_gradients_with_hash_bounds():
    means, conf, s = tl.custom_scene(seed=31, P=60, W=48, H=32, extent=2.0, dist=6.0)
    s = dataclasses.replace(s, exact_gradients=True, hash_bounds=(-2.2, -2.2, -2.2, 2.2, 2.2, 2.2))
    dc, df = tl.random_grads(s, seed=5)
    dv = torch.zeros(s.image_height, s.image_width).cuda()
    img, grads = _gpu(means, conf, s, dc, df, dv)
    rimg, rgrads, _ = ex.exact_grads(means, conf, s, dc, df, dv)
    for k in img:
        np.testing.assert_allclose(img[k], rimg[k], atol=1e-4, err_msg=k)
    tl.assert_grads(grads, rgrads)


def test_exact_mode_keeps_the_forward():
    """The flag changes the backward only: images are bit-identical."""
    means, conf, s = tl.custom_scene(seed=32, P=80, W=48, H=32)
    a = tl.run_gpu(means, conf, s, state=False)
    b = tl.run_gpu(means, conf, dataclasses.replace(s, exact_gradients=True), state=False)
    for k in ("out_color", "out_features", "visibility"):
        np.testing.assert_array_equal(a[k], b[k])
