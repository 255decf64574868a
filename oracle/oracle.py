"""ctypes front end of the CPU oracle (oracle/vi_oracle.c) -- test infrastructure.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU baseline / reference
arm import this module; the product library never does.  Every function takes
and returns numpy arrays.  The stage functions mirror the reference pipeline
(``cuda_integrator/integrator_impl.cu:196-469`` forward, ``:474-756`` backward).
"""
import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libvi_oracle.so")
_lib = None


def build():
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


class Params(ctypes.Structure):
    _fields_ = [
        ("P", ctypes.c_int), ("W", ctypes.c_int), ("H", ctypes.c_int),
        ("means", ctypes.c_void_p), ("conf", ctypes.c_void_p),
        ("scale", ctypes.c_float),
        ("view", ctypes.c_void_p), ("proj", ctypes.c_void_p),
        ("near_plane", ctypes.c_float), ("max_distance", ctypes.c_float),
        ("table", ctypes.c_void_p),
        ("res", ctypes.c_void_p), ("do_hash", ctypes.c_void_p), ("primes", ctypes.c_void_p),
        ("T", ctypes.c_int),
        ("Wl", ctypes.c_void_p), ("bl", ctypes.c_void_p),
        ("genus", ctypes.c_int), ("G", ctypes.c_int), ("K", ctypes.c_int),
        ("bg", ctypes.c_void_p),
        ("F", ctypes.c_int), ("Fout", ctypes.c_int), ("L", ctypes.c_int),
        ("table_size", ctypes.c_uint64),
        ("hlo", ctypes.c_float * 3), ("hext", ctypes.c_float * 3),
    ]


def _declare(l):
    vp, i, f, u64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_uint64
    l.vio_higher_msb.restype = ctypes.c_uint
    l.vio_higher_msb.argtypes = [ctypes.c_uint]
    l.vio_preprocess.argtypes = [i, vp, f, vp, vp, i, i, f, f, vp, vp, vp, vp]
    l.vio_scan.restype = u64
    l.vio_scan.argtypes = [i, vp, vp]
    l.vio_duplicate.argtypes = [i, vp, vp, vp, vp, i, i, vp, vp]
    l.vio_sort.argtypes = [u64, vp, vp, vp, vp, i]
    l.vio_ranges.argtypes = [u64, vp, vp]
    l.vio_mark_visible.argtypes = [i, vp, vp, vp]
    l.vio_render.argtypes = [ctypes.POINTER(Params), vp, vp, vp, i, vp, vp, vp, vp, vp, vp, vp, vp]
    l.vio_backward.argtypes = [ctypes.POINTER(Params), vp, vp, u64, vp, i, vp, vp, vp, vp, vp,
                               vp, vp, vp, vp]
    l.vio_record_lanes.restype = i
    l.vio_record_lanes.argtypes = [ctypes.POINTER(Params), ctypes.c_uint32, ctypes.c_uint, ctypes.c_uint, vp, vp]


def _p(a):
    return None if a is None else a.ctypes.data


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def higher_msb(n):
    return int(lib().vio_higher_msb(int(n)))


class Scene:
    """All inputs of one forward/backward call, as contiguous numpy arrays.

    Field names follow the reference's ``IntegrationSettings``
    (``volume_integration/__init__.py:27-64``).
    """

    def __init__(self, means3D, confidences, primitive_scale, viewmatrix, projmatrix,
                 tanfovx, tanfovy, image_height, image_width, near_plane, max_distance,
                 feature_table, resolution, do_hash, primes, feature_offset,
                 linear_weights, linear_bias, stencil_genus, grid_size, max_primitives_per_ray,
                 bg_color, input_feature_dim, output_feature_dim, hashgrid_levels, hash_bounds=None):
        self.means = _c(means3D, np.float32).reshape(-1, 3)
        self.P = self.means.shape[0]
        self.G = int(grid_size)
        self.conf = _c(confidences, np.float32).reshape(self.P, self.G ** 3)
        self.scale = float(primitive_scale)
        self.view = _c(viewmatrix, np.float32).reshape(16)
        self.proj = _c(projmatrix, np.float32).reshape(16)
        self.tanfovx, self.tanfovy = float(tanfovx), float(tanfovy)
        self.H, self.W = int(image_height), int(image_width)
        self.near_plane, self.max_distance = float(near_plane), float(max_distance)
        self.table = _c(feature_table, np.float32).reshape(-1)
        self.res = _c(resolution, np.int32)
        self.do_hash = _c(do_hash, np.int32)
        self.primes = _c(primes, np.int32)
        self.T = int(feature_offset)
        self.Wl = _c(linear_weights, np.float32).reshape(-1)
        self.bl = _c(linear_bias, np.float32).reshape(-1)
        self.genus, self.K = int(stencil_genus), int(max_primitives_per_ray)
        self.bg = _c(bg_color, np.float32).reshape(-1)
        self.F, self.Fout, self.L = int(input_feature_dim), int(output_feature_dim), int(hashgrid_levels)
        # hashgrid box (lo, extent) per axis; the reference's is fixed (hashgrid.h:23-24)
        if hash_bounds is None:
            self.hlo, self.hext = [np.float32(-1.3)] * 3, [np.float32(2.6)] * 3
        else:
            hb = np.asarray(hash_bounds, np.float32).reshape(6)
            self.hlo = [hb[a] for a in range(3)]
            self.hext = [np.float32(hb[3 + a] - hb[a]) for a in range(3)]

    @staticmethod
    def from_settings(means3D, confidences, settings):
        """Build from torch tensors + an ``IntegrationSettings`` instance."""
        def n(t):
            return t.detach().cpu().numpy() if hasattr(t, "detach") else np.asarray(t)
        s = settings
        return Scene(n(means3D), n(confidences), s.primitive_scale, n(s.viewmatrix), n(s.projmatrix),
                     s.tanfovx, s.tanfovy, s.image_height, s.image_width, s.near_plane, s.max_distance,
                     n(s.feature_table), n(s.resolution), n(s.do_hash), n(s.primes), s.feature_offset,
                     n(s.linear_weights), n(s.linear_bias), s.stencil_genus, s.grid_size,
                     s.max_primitives_per_ray, n(s.bg_color), s.input_feature_dim,
                     s.output_feature_dim, s.hashgrid_levels, getattr(s, "hash_bounds", None))

    @property
    def tiles(self):
        return ((self.W + 15) // 16) * ((self.H + 15) // 16)

    def params(self):
        p = Params()
        p.P, p.W, p.H = self.P, self.W, self.H
        p.means, p.conf = _p(self.means), _p(self.conf)
        p.scale = self.scale
        p.view, p.proj = _p(self.view), _p(self.proj)
        p.near_plane, p.max_distance = self.near_plane, self.max_distance
        p.table = _p(self.table)
        p.res, p.do_hash, p.primes = _p(self.res), _p(self.do_hash), _p(self.primes)
        p.T = self.T
        p.Wl, p.bl = _p(self.Wl), _p(self.bl)
        p.genus, p.G, p.K = self.genus, self.G, self.K
        p.bg = _p(self.bg)
        p.F, p.Fout, p.L = self.F, self.Fout, self.L
        p.table_size = self.table.size
        for a in range(3):
            p.hlo[a], p.hext[a] = float(self.hlo[a]), float(self.hext[a])
        return p


def preprocess(s):
    P = s.P
    radii = np.zeros(P, np.int32)
    means2D = np.zeros((P, 2), np.float32)
    depths = np.zeros(P, np.float32)
    tt = np.zeros(P, np.uint32)
    lib().vio_preprocess(P, _p(s.means), s.scale, _p(s.view), _p(s.proj), s.W, s.H,
                         s.tanfovx, s.tanfovy, _p(radii), _p(means2D), _p(depths), _p(tt))
    return dict(radii=radii, means2D=means2D, depths=depths, tiles_touched=tt)


def binning(s, pre):
    """Scan, duplicate, stable sort, tile ranges (integrator_impl.cu:306-365)."""
    P = s.P
    offsets = np.zeros(P, np.uint32)
    R = int(lib().vio_scan(P, _p(pre["tiles_touched"]), _p(offsets)))
    ku = np.zeros(R, np.uint64)
    vu = np.zeros(R, np.uint32)
    lib().vio_duplicate(P, _p(pre["means2D"]), _p(pre["depths"]), _p(offsets), _p(pre["radii"]),
                        s.W, s.H, _p(ku), _p(vu))
    bit = higher_msb(s.tiles)
    ks = np.zeros(R, np.uint64)
    vs = np.zeros(R, np.uint32)
    lib().vio_sort(R, _p(ku), _p(vu), _p(ks), _p(vs), 32 + bit)
    ranges = np.zeros((s.tiles, 2), np.uint32)
    lib().vio_ranges(R, _p(ks), _p(ranges))
    return dict(num_rendered=R, point_offsets=offsets, keys_unsorted=ku, vals_unsorted=vu,
                keys=ks, point_list=vs, ranges=ranges, end_bit=32 + bit)


def render(s, binned, tile_mask=None, threads=0):
    H, W, K, N = s.H, s.W, s.K, s.H * s.W
    out = dict(
        out_color=np.zeros((3, H, W), np.float32),
        out_features=np.zeros((s.Fout, H, W), np.float32),
        visibility=np.zeros((H, W), np.float32),
        final_T=np.zeros(N, np.float32),
        n_contrib=np.zeros(N, np.int32),
        contrib_idx=np.full(N * K, -1, np.int32),
        delta_t=np.zeros(N * K, np.float32),
        skips=np.zeros(N, np.int32),
    )
    tm = None if tile_mask is None else _c(tile_mask, np.uint8)
    p = s.params()
    lib().vio_render(ctypes.byref(p), _p(binned["ranges"]), _p(binned["point_list"]), _p(tm), int(threads),
                     _p(out["out_color"]), _p(out["out_features"]), _p(out["visibility"]),
                     _p(out["final_T"]), _p(out["n_contrib"]), _p(out["contrib_idx"]), _p(out["delta_t"]),
                     _p(out["skips"]))
    return out


def backward(s, binned, fwd, dL_dcolor, dL_dfeat, tile_mask=None, threads=0):
    D = s.L * s.F
    O = 3 + s.Fout + 1
    g = dict(
        dL_dmeans3D=np.zeros((s.P, 3), np.float32),
        dL_dconfidences=np.zeros((s.P, s.G ** 3), np.float32),
        dL_dfeature_table=np.zeros(s.table.size, np.float32),
        dL_dlinear_weights=np.zeros(O * D, np.float32),
        dL_dlinear_bias=np.zeros(O, np.float32),
    )
    if binned["num_rendered"] == 0:
        return g
    tm = None if tile_mask is None else _c(tile_mask, np.uint8)
    dc = _c(dL_dcolor, np.float32)
    df = _c(dL_dfeat, np.float32) if s.Fout > 0 else None
    p = s.params()
    lib().vio_backward(ctypes.byref(p), _p(binned["ranges"]), _p(binned["point_list"]), binned["num_rendered"],
                       _p(tm), int(threads), _p(dc), _p(df), _p(fwd["n_contrib"]), _p(fwd["contrib_idx"]),
                       _p(fwd["delta_t"]), _p(g["dL_dconfidences"]), _p(g["dL_dfeature_table"]),
                       _p(g["dL_dlinear_weights"]), _p(g["dL_dlinear_bias"]))
    return g


def mark_visible(means, view):
    means = _c(means, np.float32).reshape(-1, 3)
    out = np.zeros(means.shape[0], np.uint8)
    lib().vio_mark_visible(means.shape[0], _p(means), _p(_c(view, np.float32)), _p(out))
    return out.astype(bool)


def forward(s, tile_mask=None, threads=0):
    """Full forward: preprocess + binning + render.  Returns one dict of all state.

    P == 0 or an empty image returns zero images and no state, as the reference
    skips the whole forward then (integrate_primitives.cu:153-190).
    """
    if s.P == 0 or s.W * s.H == 0:
        N, K = s.H * s.W, s.K
        return dict(radii=np.zeros(0, np.int32), means2D=np.zeros((0, 2), np.float32),
                    depths=np.zeros(0, np.float32), tiles_touched=np.zeros(0, np.uint32), num_rendered=0,
                    keys=np.zeros(0, np.uint64), point_list=np.zeros(0, np.uint32),
                    ranges=np.zeros((s.tiles, 2), np.uint32),
                    out_color=np.zeros((3, s.H, s.W), np.float32),
                    out_features=np.zeros((s.Fout, s.H, s.W), np.float32),
                    visibility=np.zeros((s.H, s.W), np.float32), final_T=np.zeros(N, np.float32),
                    n_contrib=np.zeros(N, np.int32), contrib_idx=np.full(N * K, -1, np.int32),
                    delta_t=np.zeros(N * K, np.float32))
    pre = preprocess(s)
    b = binning(s, pre)
    out = render(s, b, tile_mask=tile_mask, threads=threads)
    res = dict(pre)
    res.update(b)
    res.update(out)
    return res


def record_lanes(s, q, px, py):
    """Grid points of primitive q forming its record at pixel (px, py) in the
    forward, with their stencil magnitudes (test helper for the exact-gradient
    mode; vio_record_lanes)."""
    V = s.G ** 3
    lanes = np.zeros(V, np.int32)
    mags = np.zeros(V, np.float32)
    p = s.params()
    n = lib().vio_record_lanes(ctypes.byref(p), int(q), int(px), int(py), _p(lanes), _p(mags))
    return lanes[:n].copy(), mags[:n].copy()
