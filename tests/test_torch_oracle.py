"""The vectorised PyTorch-CPU restatement (oracle/torch_oracle.py, the timed CPU
baseline) against the scalar C oracle on the same seeded scenes (CPU only).

Integer state (radii, sorted keys, point list, tile ranges, contributor counts
and lists) and delta t must be identical; images within 1e-4 and gradients
within 1e-3 relative, because the restatement forms the linear layer with a
matrix product and sums the table gradient per grid point before scattering.
"""
import numpy as np
import pytest
import torch

import oracle as orc
import torch_oracle as tor
import vi_testlib as tl

CASES = {
    "default": {},
    "genus2": dict(genus=2),
    "grid2": dict(G=2),
    "grid4": dict(G=4, P=150),
    "fout0": dict(Fout=0),
    "K3": dict(K=3),
    "bg_ragged": dict(bg=(0.2, 0.5, 0.9), W=70, H=45),
    "dense_levels": dict(L=4, base=4, growth=1.5, log2_T=16),
    "T_not_pow2": dict(T=3001, log2_T=11),
    "near_camera": dict(dist=1.2, extent=0.8, scale=0.3),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_torch_restatement_matches_c_oracle(name):
    means, conf, s = tl.custom_scene(seed=7, device="cpu", **CASES[name])
    dc, df = tl.random_grads(s, seed=2, device="cpu")
    sc, o = tl.oracle_run(means, conf, s, dc, df, threads=4)
    t, tg = tor.run(sc, dc.numpy(), df.numpy())
    assert t["num_rendered"] == o["num_rendered"]
    np.testing.assert_array_equal(t["radii"], o["radii"])
    np.testing.assert_array_equal(t["keys"].astype(np.uint64), o["keys"])
    np.testing.assert_array_equal(t["point_list"].astype(np.uint32), o["point_list"])
    np.testing.assert_array_equal(t["ranges"].astype(np.uint32), o["ranges"])
    np.testing.assert_array_equal(t["n_contrib"], o["n_contrib"])
    K = s.max_primitives_per_ray
    used = (np.arange(K)[None, :] < o["n_contrib"][:, None]).reshape(-1)
    np.testing.assert_array_equal(t["contrib_idx"][used], o["contrib_idx"][used])
    np.testing.assert_array_equal(t["delta_t"][used].view(np.uint32), o["delta_t"][used].view(np.uint32))
    tl.assert_images(t, o)
    tl.assert_grads(tg, o["grads"])


def test_torch_restatement_on_a_tile_subset():
    means, conf, s = tl.custom_scene(seed=11, device="cpu", P=600, W=96, H=64)
    dc, df = tl.random_grads(s, seed=3, device="cpu")
    sco = orc.Scene.from_settings(means, conf, s)
    mask = np.zeros(sco.tiles, np.uint8)
    mask[::3] = 1
    _, o = tl.oracle_run(means, conf, s, dc, df, threads=4, tile_mask=mask)
    t, tg = tor.run(sco, dc.numpy(), df.numpy(), tile_mask=mask)
    np.testing.assert_array_equal(t["n_contrib"], o["n_contrib"])
    tl.assert_images(t, o)
    tl.assert_grads(tg, o["grads"])
    assert int(o["n_contrib"].sum()) > 100
