"""CUDA path vs the CPU oracle on the benchmarked configurations (needs a B200).

The parity cases in test_gpu_parity.py are small scenes.  These run the
workloads the benchmark times -- the mid scene (one of its 8 cameras), the
headline scene and the stress scene -- at their full sizes, with the
reference's fixed hashgrid box and with the scene's own bounds (where no grid
point clamps and the hashgrid kernels do the most work).  The feature table is
drawn from U(-1, 1) so that images and gradients are not bias-dominated.

* The whole frame's integer state is compared bit for bit: radii, tiles
  touched, depths, screen means, sorted keys, point list and tile ranges.
* The oracle renders a subset of tiles (the longest lists plus a seeded random
  sample): images, final transmittance, contributor counts, contributor list
  indices and delta t of those tiles' pixels must match (images within 1e-4,
  the rest bit-exact).
* dL/dimage is zeroed outside the subset on both sides, so the CUDA path's
  full-frame gradients must equal the oracle's gradients over the subset
  (1e-3 relative).
"""
import numpy as np
import pytest
import torch

import vi_testlib as tl

pytestmark = pytest.mark.gpu

# (scene, view, scene bounds?) -- the stress scene is 6M primitives at 3840x2160
# with 4 features per level (D = 64) and T = 2^21.
CASES = [
    ("mid", 3, False), ("mid", 3, True),
    ("headline", 0, False), ("headline", 0, True),
    ("stress", 0, False),
]
EXTENT = {"mid": 3.0, "headline": 10.0, "stress": 10.0}


def _subset(ranges, n_long, n_random, seed):
    lens = ranges[:, 1].astype(np.int64) - ranges[:, 0].astype(np.int64)
    nonempty = np.flatnonzero(lens > 0)
    longest = nonempty[np.argsort(-lens[nonempty], kind="stable")[:n_long]]
    rest = np.setdiff1d(nonempty, longest)
    rng = np.random.default_rng(seed)
    pick = rng.choice(rest, size=min(n_random, rest.size), replace=False) if rest.size else rest
    mask = np.zeros(ranges.shape[0], np.uint8)
    mask[longest] = 1
    mask[pick] = 1
    return mask


def _pixel_mask(tile_mask, W, H):
    gx = (W + 15) // 16
    ty, tx = np.divmod(np.arange(tile_mask.size), gx)
    m = np.zeros((H, W), bool)
    for t in np.flatnonzero(tile_mask):
        m[ty[t] * 16:(ty[t] + 1) * 16, tx[t] * 16:(tx[t] + 1) * 16] = True
    return m


@pytest.mark.parametrize("name,view,own_bounds", CASES,
                         ids=[f"{n}-v{v}-{'scenebox' if b else 'refbox'}" for n, v, b in CASES])
def test_benchmarked_config_parity(name, view, own_bounds):
    over = {}
    if own_bounds:
        e = EXTENT[name]
        over["hash_bounds"] = (-e, -e, -e, e, e, e)
    means, conf, s = tl.scene(name, view=view, table_range=1.0)
    if own_bounds:
        s.hash_bounds = over["hash_bounds"]
    W, H, K = s.image_width, s.image_height, s.max_primitives_per_ray

    # whole-frame integer state of the CUDA path, and the tile subset from it
    g = tl.gpu_state(means, conf, s)
    o_sc = tl.oracle_scene(means, conf, s)
    import oracle as orc
    pre = orc.preprocess(o_sc)
    b = orc.binning(o_sc, pre)
    assert g["num_rendered"] == b["num_rendered"] > 0
    np.testing.assert_array_equal(g["radii"], pre["radii"])
    np.testing.assert_array_equal(g["tiles_touched"].view(np.uint32), pre["tiles_touched"])
    vis = pre["radii"] > 0
    np.testing.assert_array_equal(g["depths"][vis].view(np.uint32), pre["depths"][vis].view(np.uint32))
    np.testing.assert_array_equal(g["means2D"][vis].view(np.uint32), pre["means2D"][vis].view(np.uint32))
    np.testing.assert_array_equal(g["keys"], b["keys"])
    np.testing.assert_array_equal(g["point_list"].view(np.uint32), b["point_list"])
    np.testing.assert_array_equal(g["ranges"].view(np.uint32), b["ranges"])
    tmask = _subset(b["ranges"], n_long=6, n_random=26, seed=view + 17)
    pm = _pixel_mask(tmask, W, H)
    del g

    # images, contributor lists and gradients on the subset
    dc, df = tl.random_grads(s, seed=5, device="cpu")
    pmt = torch.from_numpy(pm)
    dc, df = dc * pmt, df * pmt
    gg = tl.run_gpu(means, conf, s, dc.cuda(), df.cuda(), state=True)
    o = orc.render(o_sc, b, tile_mask=tmask)
    pix = pm.reshape(-1)
    for k in ("out_color", "out_features"):
        err = float(np.abs(gg[k][:, pm] - o[k][:, pm]).max())
        assert err <= tl.IMG_TOL, (k, err)
    assert float(np.abs(gg["visibility"][pm] - o["visibility"][pm]).max()) <= tl.IMG_TOL
    assert float(np.abs(gg["final_T"][pix] - o["final_T"][pix]).max()) <= tl.IMG_TOL
    np.testing.assert_array_equal(gg["n_contrib"][pix], o["n_contrib"][pix])
    used = (np.arange(K)[None, :] < o["n_contrib"][:, None]) & pix[:, None]
    np.testing.assert_array_equal(gg["contrib_idx"].reshape(-1, K)[used], o["contrib_idx"].reshape(-1, K)[used])
    np.testing.assert_array_equal(gg["delta_t"].reshape(-1, K)[used].view(np.uint32),
                                  o["delta_t"].reshape(-1, K)[used].view(np.uint32))
    assert int(o["n_contrib"][pix].sum()) > 1000  # the subset really composites
    og = orc.backward(o_sc, b, o, dc.numpy(), df.numpy(), tile_mask=tmask)
    tl.assert_grads(gg["grads"], og)
