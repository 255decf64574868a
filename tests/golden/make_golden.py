"""Generates tests/golden/*.npz: the reference extension's own outputs on fixed
inputs, used to pin the CPU oracle (tests/test_golden.py) and to check the
CUDA path (tests/test_gpu_golden.py).

Run on a machine with a GPU, from the repository root, after
`make -C oracle/ref REF=<reference checkout>` has built
oracle/_ref/libviref_{G,O3}.so from the reference sources:

    python tests/golden/make_golden.py [--out DIR] [binning] [full] [<full case name> ...]

Two kinds of fixtures:

* binning (b_*.npz): preprocess, scan, duplicateWithKeys, CUB radix sort and
  identifyTileRanges of the reference (no render kernel) on any scene; radii,
  tiles touched, depths, screen means, sorted keys, point list, tile ranges.
* full (f_*.npz): the reference's whole Integrator::forward and ::backward on
  scenes with a 1x1 or 2x1 image in which every primitive covers every active
  pixel.  The reference render kernel skips a CTA barrier for pixels that no
  grid point covers (forward.cu:629-631 vs :715); on these scenes the CPU oracle
  counts zero such events, so every reference thread takes every barrier.
  A scene is only handed to the reference after that check passes.

Each file stores the inputs next to the outputs of both reference builds
(`-G` as shipped, and `-O3`).
"""
import ctypes
import math
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
for p in (os.path.join(ROOT, "volume-integration_b200"), os.path.join(ROOT, "oracle")):
    sys.path.insert(0, p)
import oracle as orc  # noqa: E402
import vi_workloads as wl  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
REF = {k: os.path.join(ROOT, "oracle", "_ref", f"libviref_{k}.so") for k in ("G", "O3")}


def load(kind):
    lib = ctypes.CDLL(REF[kind])
    vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    lib.ref_binning_run.argtypes = [i, vp, f, vp, vp, i, i, f, f, ctypes.POINTER(ctypes.c_longlong)]
    lib.ref_binning_fetch.argtypes = [vp] * 7
    lib.ref_mark_visible.argtypes = [i, vp, vp, vp, vp]
    lib.ref_forward_run.argtypes = [i, i, i, vp, f, vp, vp, vp, f, f, f, f, vp, vp, vp, vp, vp, i, vp, vp, i, i, i, f,
                                    vp, vp, vp, vp, ctypes.c_uint, ctypes.c_uint, ctypes.c_uint, ctypes.c_uint,
                                    ctypes.POINTER(ctypes.c_int)]
    lib.ref_forward_fetch.argtypes = [vp] * 8
    lib.ref_backward_run.argtypes = [vp, vp, vp, f, vp, vp, vp, f, f, f, f, vp, vp, vp, vp, vp, i, vp, vp, i, i, i, f,
                                     vp, ctypes.c_uint, ctypes.c_uint, ctypes.c_uint, ctypes.c_uint, vp, vp, vp, vp, vp]
    return lib


def dev(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=dtype)).cuda()


def p(t):
    return ctypes.c_void_p(t.data_ptr())


# ---------------------------------------------------------------------------
# binning fixtures
# ---------------------------------------------------------------------------
def binning_case(libs, name, means, cam, scale):
    out = dict(means=means.astype(np.float32), viewmatrix=cam["viewmatrix"].numpy(),
               projmatrix=cam["projmatrix"].numpy(), tanfovx=cam["tanfovx"], tanfovy=cam["tanfovy"],
               width=cam["image_width"], height=cam["image_height"], scale=scale)
    P = means.shape[0]
    W, H = cam["image_width"], cam["image_height"]
    tiles = ((W + 15) // 16) * ((H + 15) // 16)
    m, v, pr = dev(means, np.float32), dev(out["viewmatrix"], np.float32), dev(out["projmatrix"], np.float32)
    for kind, lib in libs.items():
        R = ctypes.c_longlong(0)
        torch.cuda.synchronize()
        assert lib.ref_binning_run(P, p(m), scale, p(v), p(pr), W, H, cam["tanfovx"], cam["tanfovy"],
                                   ctypes.byref(R)) == 0
        R = R.value
        radii = np.zeros(P, np.int32)
        m2 = np.zeros((P, 2), np.float32)
        dep = np.zeros(P, np.float32)
        tt = np.zeros(P, np.uint32)
        keys = np.zeros(max(R, 1), np.uint64)
        pl = np.zeros(max(R, 1), np.uint32)
        rng = np.zeros((tiles, 2), np.uint32)
        assert lib.ref_binning_fetch(*[x.ctypes.data for x in (radii, m2, dep, tt, keys, pl, rng)]) == 0
        vis = radii > 0
        out.update({f"{kind}_num_rendered": R, f"{kind}_radii": radii, f"{kind}_tiles_touched": tt,
                    f"{kind}_depths": np.where(vis, dep, 0).astype(np.float32),
                    f"{kind}_means2D": np.where(vis[:, None], m2, 0).astype(np.float32),
                    f"{kind}_keys": keys[:R], f"{kind}_point_list": pl[:R], f"{kind}_ranges": rng})
        present = torch.zeros(P, dtype=torch.bool, device="cuda")
        assert lib.ref_mark_visible(P, p(m), p(v), p(pr), p(present)) == 0
        out[f"{kind}_present"] = present.cpu().numpy()
    np.savez_compressed(os.path.join(OUT, f"b_{name}.npz"), **out)
    print("binning", name, "P", P, "R", out["G_num_rendered"], out["O3_num_rendered"])


def binning_fixtures(libs):
    means, conf, kw, cams = wl.make("tiny")
    binning_case(libs, "tiny", means.numpy(), cams[0], kw["primitive_scale"])
    g = torch.Generator().manual_seed(11)
    m = (torch.rand(300, 3, generator=g) * 2 - 1).numpy()
    binning_case(libs, "ragged", m, wl.camera((0.3, -0.4, -3.0), 70, 45, 50.0), 0.25)
    m = (torch.rand(400, 3, generator=g) * 2 - 1).numpy()
    m[:, 2] = 0.25  # equal depths: ties must keep primitive order
    binning_case(libs, "ties", m, wl.camera((0.0, 0.0, -3.0), 64, 48, 50.0), 0.2)
    m = (torch.rand(120, 3, generator=g) * 2 - 1).numpy()
    binning_case(libs, "big", m, wl.camera((0.3, -0.4, -3.0), 96, 64, 50.0), 0.9)
    m = (torch.rand(500, 3, generator=g) * 2 - 1).numpy() * 0.8
    binning_case(libs, "near", m, wl.camera((0.0, 0.2, -1.0), 80, 60, 60.0), 0.3)
    m = wl.mixture(20000, 64, 10.0, g).numpy()
    binning_case(libs, "hd", m, wl.camera((0.0, 0.0, -12.0), 1920, 1080, 50.0), 6.0 * math.exp(-5.0))


# ---------------------------------------------------------------------------
# full forward/backward fixtures on race-free scenes
# ---------------------------------------------------------------------------
def full_scene(seed, P=24, W=1, H=1, G=3, genus=1, K=64, bg=(0.0, 0.0, 0.0), ties=False, table_range=0.3):
    gen = np.random.default_rng(seed)
    cam = wl.camera((0.0, 0.0, -3.0), W, H, 50.0)
    tx, ty = cam["tanfovx"], cam["tanfovy"]
    zc = gen.uniform(2.0, 6.0, P)  # camera-space depth of each centre
    if ties:
        zc[1] = zc[0]
        zc[3] = zc[2]
    if W == 1:
        u = gen.uniform(0.4, 1.6, P)  # ndc x in [0, 2) -> pixel 0
    scale = 0.1 if W == 1 else 0.6
    if W != 1:
        # ndc x = 0.5 is the boundary of pixels 0 and 1.  Centre half a column
        # spacing to its right: the left column lies in pixel 0, the other two in
        # pixel 1, and no grid point comes within a quarter spacing of the
        # boundary, so a last-bit difference in projection cannot move a point.
        delta = (scale / 2) / (zc * tx)
        u = 0.5 + delta / 2
    v = gen.uniform(0.4, 1.6, P)
    means = np.stack([u * zc * tx, v * zc * ty, zc - 3.0], 1).astype(np.float32)
    L, F, log2_T, Fout = 16, 2, 8, 4
    hg = wl.hashgrid(L, F, log2_T, 4, 1.5)
    T = hg["feature_offset"]
    table = gen.uniform(-table_range, table_range, T * L * F).astype(np.float32)
    D, O = L * F, Fout + 4
    Wl = gen.uniform(-1 / math.sqrt(D), 1 / math.sqrt(D), O * D).astype(np.float32)
    bl = gen.uniform(-0.5, 0.5, O).astype(np.float32)
    bl[-1] = -2.0  # low density so several primitives composite before the pixel saturates
    conf = gen.normal(1.0, 1.0, (P, G ** 3)).astype(np.float32)
    return dict(means=means, conf=conf, scale=scale, viewmatrix=cam["viewmatrix"].numpy(),
                projmatrix=cam["projmatrix"].numpy(), cam_pos=cam["cam_pos"].numpy(), tanfovx=tx, tanfovy=ty,
                width=W, height=H, near_plane=0.01, max_distance=100.0, table=table,
                resolution=hg["resolution"].numpy(), do_hash=hg["do_hash"].numpy(), primes=hg["primes"].numpy(),
                T=T, Wl=Wl, bl=bl, genus=genus, G=G, K=K, bg=np.array(bg, np.float32), F=F, Fout=Fout, L=L)


def oracle_scene(d):
    return orc.Scene(d["means"], d["conf"], d["scale"], d["viewmatrix"], d["projmatrix"], d["tanfovx"],
                     d["tanfovy"], d["height"], d["width"], d["near_plane"], d["max_distance"], d["table"],
                     d["resolution"], d["do_hash"], d["primes"], d["T"], d["Wl"], d["bl"], d["genus"], d["G"],
                     d["K"], d["bg"], d["F"], d["Fout"], d["L"])


def race_free(d):
    f = orc.forward(oracle_scene(d))
    return int(f["skips"].sum()) == 0 and f["num_rendered"] > 0, f


def full_case(libs, name, **kw):
    for seed in range(100, 400):
        d = full_scene(seed, **kw)
        ok, f = race_free(d)
        if ok:
            break
    else:
        raise RuntimeError(f"no race-free scene for {name}")
    W, H, P, K = d["width"], d["height"], d["means"].shape[0], d["K"]
    N = W * H
    tiles = ((W + 15) // 16) * ((H + 15) // 16)
    gen = np.random.default_rng(seed + 1)
    dc = gen.standard_normal((3, H, W)).astype(np.float32)
    df = gen.standard_normal((d["Fout"], H, W)).astype(np.float32)
    d.update(dL_dcolor=dc, dL_dfeatures=df, seed=seed)
    t = {k: dev(d[k], np.float32) for k in ("means", "conf", "viewmatrix", "projmatrix", "cam_pos", "table", "Wl",
                                            "bl", "bg")}
    t.update({k: dev(d[k], np.int32) for k in ("resolution", "do_hash", "primes")})
    gdc, gdf = dev(dc, np.float32), dev(df, np.float32)
    for kind, lib in libs.items():
        oc = torch.zeros(3, H, W, device="cuda")
        of = torch.zeros(d["Fout"], H, W, device="cuda")
        vis = torch.zeros(H, W, device="cuda")
        R = ctypes.c_int(0)
        torch.cuda.synchronize()
        rc = lib.ref_forward_run(P, W, H, p(t["means"]), d["scale"], p(t["viewmatrix"]), p(t["projmatrix"]),
                                 p(t["cam_pos"]), d["near_plane"], d["max_distance"], d["tanfovx"], d["tanfovy"],
                                 p(t["conf"]), p(t["table"]), p(t["resolution"]), p(t["do_hash"]), p(t["primes"]),
                                 d["T"], p(t["Wl"]), p(t["bl"]), d["genus"], d["G"], K, 0.5, p(t["bg"]), p(oc), p(of),
                                 p(vis), d["F"], d["Fout"], d["L"] * d["F"], d["L"], ctypes.byref(R))
        assert rc == 0
        R = R.value
        fT = np.zeros(N, np.float32)
        nc = np.zeros(N, np.int32)
        ci = np.zeros(N * K, np.int32)
        dt = np.zeros(N * K, np.float32)
        rng = np.zeros((tiles, 2), np.uint32)
        keys = np.zeros(max(R, 1), np.uint64)
        pl = np.zeros(max(R, 1), np.uint32)
        radii = np.zeros(P, np.int32)
        assert lib.ref_forward_fetch(*[x.ctypes.data for x in (fT, nc, ci, dt, rng, keys, pl, radii)]) == 0
        grads = [torch.zeros(P, 3, device="cuda"), torch.zeros(P, d["G"] ** 3, device="cuda"),
                 torch.zeros(d["table"].size, device="cuda"), torch.zeros(d["Wl"].size, device="cuda"),
                 torch.zeros(d["bl"].size, device="cuda")]
        rc = lib.ref_backward_run(p(gdc), p(gdf), p(t["means"]), d["scale"], p(t["viewmatrix"]), p(t["projmatrix"]),
                                  p(t["cam_pos"]), d["near_plane"], d["max_distance"], d["tanfovx"], d["tanfovy"],
                                  p(t["conf"]), p(t["table"]), p(t["resolution"]), p(t["do_hash"]), p(t["primes"]),
                                  d["T"], p(t["Wl"]), p(t["bl"]), d["genus"], d["G"], K, 0.5, p(t["bg"]), d["F"],
                                  d["Fout"], d["L"], d["table"].size, *[p(g) for g in grads])
        assert rc == 0
        torch.cuda.synchronize()
        mask = (np.arange(K)[None, :] < nc[:, None]).reshape(-1)
        d.update({f"{kind}_num_rendered": R, f"{kind}_out_color": oc.cpu().numpy(),
                  f"{kind}_out_features": of.cpu().numpy(), f"{kind}_visibility": vis.cpu().numpy(),
                  f"{kind}_final_T": fT, f"{kind}_n_contrib": nc, f"{kind}_contrib_idx": np.where(mask, ci, -1),
                  f"{kind}_delta_t": np.where(mask, dt, 0).astype(np.float32), f"{kind}_ranges": rng,
                  f"{kind}_keys": keys[:R], f"{kind}_point_list": pl[:R], f"{kind}_radii": radii,
                  f"{kind}_dL_dconfidences": grads[1].cpu().numpy(), f"{kind}_dL_dfeature_table": grads[2].cpu().numpy(),
                  f"{kind}_dL_dlinear_weights": grads[3].cpu().numpy(),
                  f"{kind}_dL_dlinear_bias": grads[4].cpu().numpy(), f"{kind}_dL_dmeans3D": grads[0].cpu().numpy()})
    np.savez_compressed(os.path.join(OUT, f"f_{name}.npz"), **d)
    print("full", name, "seed", seed, "R", d["G_num_rendered"], "contrib", d["G_n_contrib"].tolist())


FULL_CASES = {
    "px1": {},
    "px1_k3": dict(K=3),
    "px1_genus2": dict(genus=2),
    "px1_bg": dict(bg=(0.2, 0.4, 0.6), table_range=0.5),
    "px1_ties": dict(ties=True),
    "px1_grid2": dict(G=2),
    "px2": dict(W=2, P=16),
    # 4^3 and 5^3 grids (the reference's MAX_GRID_SIZE is 5, forward.cu:204-205)
    "px1_grid4": dict(G=4, P=12),
    "px1_grid5": dict(G=5, P=8),
}


def full_fixtures(libs, names=None):
    for name, kw in FULL_CASES.items():
        if names is None or name in names:
            full_case(libs, name, **kw)


if __name__ == "__main__":
    assert torch.cuda.is_available(), "the reference extension needs a GPU"
    args = sys.argv[1:]
    if "--out" in args:
        i = args.index("--out")
        OUT = args[i + 1]
        os.makedirs(OUT, exist_ok=True)
        del args[i:i + 2]
    libs = {k: load(k) for k in ("G", "O3")}
    which = args or ["binning", "full"]
    if "binning" in which:
        binning_fixtures(libs)
    if "full" in which:
        full_fixtures(libs)
    picked = [a for a in which if a in FULL_CASES]  # single full cases by name
    if picked:
        full_fixtures(libs, picked)
