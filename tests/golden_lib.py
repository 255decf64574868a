"""Loading of the reference fixtures in tests/golden/ (written by
tests/golden/make_golden.py from the reference extension's own kernels)."""
import glob
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
REF_BUILDS = ("G", "O3")


def files(prefix):
    return sorted(glob.glob(os.path.join(GOLDEN, prefix + "_*.npz")))


def load(path):
    with np.load(path) as z:
        return {k: z[k] for k in z.files}


def name(path):
    return os.path.basename(path)[:-4]


def full_scene_args(d):
    """Positional arguments of oracle.Scene for a full fixture."""
    return (d["means"], d["conf"], float(d["scale"]), d["viewmatrix"], d["projmatrix"], float(d["tanfovx"]),
            float(d["tanfovy"]), int(d["height"]), int(d["width"]), float(d["near_plane"]),
            float(d["max_distance"]), d["table"], d["resolution"], d["do_hash"], d["primes"], int(d["T"]), d["Wl"],
            d["bl"], int(d["genus"]), int(d["G"]), int(d["K"]), d["bg"], int(d["F"]), int(d["Fout"]), int(d["L"]))
