"""Times the reference's own CUDA kernels on a B200 -- the GPU baseline of the
renderer (test infrastructure; it never times the product).

On the headline workload (1M primitives, 1920x1080, 16-level hashgrid; the
seeded synthetic scene of vi_workloads) it measures, per reference build:

* the binning stages (preprocess, CUB scan with the 4-byte read of R,
  duplicateWithKeys, CUB radix sort, identifyTileRanges; integrator_impl.cu:
  277-365) with CUDA events, and the CUB sort alone (keys/s);
* Integrator::forward and Integrator::backward as whole calls (the reference
  synchronises the device inside them), after one untimed call that sizes the
  reference's state buffers.

The render runs only in its barrier-fixed form (libviref_*_bf.so, see
barrier_fix.py): the shipped kernel skips a CTA barrier on ordinary scenes.
The binning and backward kernels are the shipped ones.

Usage (on a GPU machine, after `make -C oracle/ref REF=...` here):
    python oracle/ref/time_reference.py [--kinds O3_bf,G_bf] [--reps 3] [--out FILE.json]
"""
import argparse
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (HERE, os.path.join(ROOT, "volume-integration_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

import torch  # noqa: E402

import reflib  # noqa: E402


def headline_inputs(name="headline", view=0):
    """The seeded scene and camera `view` of vi_workloads as CUDA tensors, with the
    settings as a plain namespace (the reference's IntegrationSettings fields;
    nothing of this build's library is loaded)."""
    import types
    import vi_workloads as wl
    means, conf, kw, cams = wl.make(name)
    d = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in list(kw.items()) + list(cams[view].items())}
    s = types.SimpleNamespace(**d)
    means, conf = means.cuda(), conf.cuda()
    gen = torch.Generator().manual_seed(7)
    dc = torch.randn(3, s.image_height, s.image_width, generator=gen).cuda()
    df = torch.randn(s.output_feature_dim, s.image_height, s.image_width, generator=gen).cuda()
    return means, conf, s, dc, df


def measure(kinds=("O3_bf", "G_bf"), reps=3, name="headline", deadline_s=600.0):
    """Returns {kind: {...}} for every built kind; a kind whose library is missing
    is reported as unavailable.  Stops timing a build early (fewer repetitions)
    once deadline_s of wall time has passed, and says so."""
    means, conf, s, dc, df = headline_inputs(name)
    sc = reflib.Scene(means, conf, s)
    t_start = time.time()
    out = {}
    for kind in kinds:
        if not reflib.available(kind):
            out[kind] = {"unavailable": "oracle/_ref/libviref_%s.so not built" % kind}
            continue
        lib = reflib.load(kind)
        r = {}
        nb = reps if kind.startswith("O3") else 1
        ms, R = reflib.time_binning(lib, sc, reps=nb)
        r["binning_ms"] = dict(zip(("preprocess", "scan", "duplicate", "sort", "ranges"), ms[:5]))
        r["num_rendered"] = R
        r["cub_sort_ms"] = ms[5]
        r["cub_sort_gkeys_per_s"] = R / (ms[5] * 1e-3) / 1e9 if ms[5] > 0 else None
        reflib.forward(lib, sc, timed=True, fetch=False)  # sizes the state buffers
        reflib.backward(lib, sc, dc, df, timed=True)
        fw, bw = [], []
        n = reps if kind.startswith("O3") else 1
        for _ in range(n):
            fw.append(reflib.forward(lib, sc, timed=True, fetch=False)["ms"])
            bw.append(reflib.backward(lib, sc, dc, df, timed=True)["ms"])
            if time.time() - t_start > deadline_s:
                r["note"] = "stopped after %d repetitions at the time limit" % len(fw)
                break
        r["forward_ms"] = sum(fw) / len(fw)
        r["backward_ms"] = sum(bw) / len(bw)
        r["frames_per_s"] = 1000.0 / (r["forward_ms"] + r["backward_ms"])
        r["repetitions"] = len(fw)
        out[kind] = r
    out["workload"] = "%s: P=%d, %dx%d, L=%d F=%d T=%d, G=%d, K=%d" % (
        name, means.shape[0], s.image_width, s.image_height, s.hashgrid_levels, s.input_feature_dim,
        s.feature_offset, s.grid_size, s.max_primitives_per_ray)
    out["gpu"] = torch.cuda.get_device_name(0)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kinds", default="O3_bf,G_bf")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--scene", default="headline")
    ap.add_argument("--out", default=None)
    a = ap.parse_args()
    res = measure(tuple(a.kinds.split(",")), a.reps, a.scene)
    text = json.dumps(res, indent=1)
    print(text)
    if a.out:
        with open(a.out, "w") as f:
            f.write(text + "\n")


if __name__ == "__main__":
    main()
