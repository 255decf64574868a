"""ctypes front end of the reference's own CUDA kernels (oracle/_ref/libviref_*.so,
built by oracle/ref/Makefile from the reference checkout) -- test infrastructure.

Used by tests/golden/make_golden.py, tests/test_gpu_reference.py and
oracle/ref/time_reference.py; the product never loads it.  Builds:

  G, O3        the reference as shipped (-G, setup.py:16, :39) and at -O3;
  G_bf, O3_bf  the same with the barrier-fixed render kernel (barrier_fix.py),
               the only form of the reference render that is safe to run on an
               ordinary scene.

All tensors passed in are CUDA tensors; the reference kernels run on the legacy
default stream and the harness synchronises the device after every call.
"""
import ctypes
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(os.path.dirname(HERE), "_ref")
KINDS = ("G", "O3", "G_bf", "O3_bf")


def path(kind):
    return os.path.join(REF_DIR, f"libviref_{kind}.so")


def available(kind):
    return os.path.exists(path(kind))


def load(kind):
    lib = ctypes.CDLL(path(kind))
    vp, i, f, u = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_uint
    lib.ref_binning_run.argtypes = [i, vp, f, vp, vp, i, i, f, f, ctypes.POINTER(ctypes.c_longlong)]
    lib.ref_binning_fetch.argtypes = [vp] * 7
    lib.ref_mark_visible.argtypes = [i, vp, vp, vp, vp]
    fwd = [i, i, i, vp, f, vp, vp, vp, f, f, f, f, vp, vp, vp, vp, vp, i, vp, vp, i, i, i, f, vp, vp, vp, vp,
           u, u, u, u, ctypes.POINTER(ctypes.c_int)]
    bwd = [vp, vp, vp, f, vp, vp, vp, f, f, f, f, vp, vp, vp, vp, vp, i, vp, vp, i, i, i, f, vp, u, u, u, u,
           vp, vp, vp, vp, vp]
    lib.ref_forward_run.argtypes = fwd
    lib.ref_forward_fetch.argtypes = [vp] * 8
    lib.ref_backward_run.argtypes = bwd
    if hasattr(lib, "ref_time_binning"):
        lib.ref_time_binning.argtypes = [i, vp, f, vp, vp, i, i, f, f, i, ctypes.POINTER(ctypes.c_double),
                                         ctypes.POINTER(ctypes.c_longlong)]
        lib.ref_timed_forward.argtypes = fwd
        lib.ref_timed_backward.argtypes = bwd
        lib.ref_last_call_ms.restype = ctypes.c_double
    return lib


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


class Scene:
    """Inputs of one reference call as CUDA tensors, from (means, conf, settings)
    of the drop-in API (volume_integration.IntegrationSettings)."""

    def __init__(self, means, conf, s):
        f32 = torch.float32
        self.s = s
        self.P = means.shape[0]
        self.G = s.grid_size
        self.means = means.detach().to("cuda", f32).contiguous()
        self.conf = conf.detach().to("cuda", f32).reshape(self.P, self.G ** 3).contiguous()
        self.view = s.viewmatrix.to("cuda", f32).contiguous()
        self.proj = s.projmatrix.to("cuda", f32).contiguous()
        self.cam_pos = s.cam_pos.to("cuda", f32).contiguous()
        self.table = s.feature_table.detach().to("cuda", f32).contiguous()
        self.res = s.resolution.to("cuda", torch.int32).contiguous()
        self.do_hash = s.do_hash.to("cuda", torch.int32).contiguous()
        self.primes = s.primes.to("cuda", torch.int32).contiguous()
        self.Wl = s.linear_weights.detach().to("cuda", f32).contiguous()
        self.bl = s.linear_bias.detach().to("cuda", f32).contiguous()
        self.bg = s.bg_color.to("cuda", f32).contiguous()
        self.W, self.H, self.K = s.image_width, s.image_height, s.max_primitives_per_ray
        self.Fout = s.output_feature_dim

    def fwd_args(self, oc, of, vis, R):
        s = self.s
        return [self.P, self.W, self.H, _p(self.means), s.primitive_scale, _p(self.view), _p(self.proj),
                _p(self.cam_pos), s.near_plane, s.max_distance, s.tanfovx, s.tanfovy, _p(self.conf), _p(self.table),
                _p(self.res), _p(self.do_hash), _p(self.primes), s.feature_offset, _p(self.Wl), _p(self.bl),
                s.stencil_genus, s.grid_size, self.K, s.occupancy_threshold, _p(self.bg), _p(oc), _p(of), _p(vis),
                s.input_feature_dim, s.output_feature_dim, s.intermediate_feature_dim, s.hashgrid_levels,
                ctypes.byref(R)]

    def bwd_args(self, dc, df, grads):
        s = self.s
        return [_p(dc), _p(df), _p(self.means), s.primitive_scale, _p(self.view), _p(self.proj), _p(self.cam_pos),
                s.near_plane, s.max_distance, s.tanfovx, s.tanfovy, _p(self.conf), _p(self.table), _p(self.res),
                _p(self.do_hash), _p(self.primes), s.feature_offset, _p(self.Wl), _p(self.bl), s.stencil_genus,
                s.grid_size, self.K, s.occupancy_threshold, _p(self.bg), s.input_feature_dim, s.output_feature_dim,
                s.hashgrid_levels, self.table.numel()] + [_p(g) for g in grads]


def forward(lib, sc, timed=False, fetch=True):
    """Integrator::forward of the reference.  Returns images, R, and (fetch) the
    integer state in the reference's own layouts; `ms` when timed."""
    oc = torch.zeros(3, sc.H, sc.W, device="cuda")
    of = torch.zeros(sc.Fout, sc.H, sc.W, device="cuda")
    vis = torch.zeros(sc.H, sc.W, device="cuda")
    R = ctypes.c_int(0)
    torch.cuda.synchronize()
    fn = lib.ref_timed_forward if timed else lib.ref_forward_run
    rc = fn(*sc.fwd_args(oc, of, vis, R))
    if rc != 0:
        raise RuntimeError("reference forward failed")
    out = dict(num_rendered=R.value, out_color=oc.cpu().numpy(), out_features=of.cpu().numpy(),
               visibility=vis.cpu().numpy())
    if timed:
        out["ms"] = float(lib.ref_last_call_ms())
    if fetch:
        N, K, R = sc.W * sc.H, sc.K, R.value
        tiles = ((sc.W + 15) // 16) * ((sc.H + 15) // 16)
        fT = np.zeros(N, np.float32)
        nc = np.zeros(N, np.int32)
        ci = np.zeros(N * K, np.int32)
        dt = np.zeros(N * K, np.float32)
        rng = np.zeros((tiles, 2), np.uint32)
        keys = np.zeros(max(R, 1), np.uint64)
        pl = np.zeros(max(R, 1), np.uint32)
        radii = np.zeros(sc.P, np.int32)
        if lib.ref_forward_fetch(*[x.ctypes.data for x in (fT, nc, ci, dt, rng, keys, pl, radii)]) != 0:
            raise RuntimeError("reference forward fetch failed")
        used = (np.arange(K)[None, :] < nc[:, None]).reshape(-1)
        out.update(final_T=fT, n_contrib=nc, contrib_idx=np.where(used, ci, -1),
                   delta_t=np.where(used, dt, 0).astype(np.float32), ranges=rng, keys=keys[:R], point_list=pl[:R],
                   radii=radii)
    return out


def backward(lib, sc, dcolor, dfeat, timed=False):
    """Integrator::backward on the state of the last forward of this library."""
    grads = [torch.zeros(sc.P, 3, device="cuda"), torch.zeros(sc.P, sc.G ** 3, device="cuda"),
             torch.zeros(sc.table.numel(), device="cuda"), torch.zeros(sc.Wl.numel(), device="cuda"),
             torch.zeros(sc.bl.numel(), device="cuda")]
    dc = dcolor.to("cuda", torch.float32).contiguous()
    df = dfeat.to("cuda", torch.float32).contiguous()
    torch.cuda.synchronize()
    fn = lib.ref_timed_backward if timed else lib.ref_backward_run
    if fn(*sc.bwd_args(dc, df, grads)) != 0:
        raise RuntimeError("reference backward failed")
    out = dict(zip(("dL_dmeans3D", "dL_dconfidences", "dL_dfeature_table", "dL_dlinear_weights", "dL_dlinear_bias"),
                   [g.cpu().numpy() for g in grads]))
    if timed:
        out["ms"] = float(lib.ref_last_call_ms())
    return out


def time_binning(lib, sc, reps=5):
    """Per-stage ms of the reference binning (preprocess, scan + R read-back,
    duplicateWithKeys, CUB radix sort, identifyTileRanges) and of the CUB sort
    alone, averaged over reps; returns (ms[6], R)."""
    s = sc.s
    ms = (ctypes.c_double * 6)()
    R = ctypes.c_longlong(0)
    torch.cuda.synchronize()
    rc = lib.ref_time_binning(sc.P, _p(sc.means), s.primitive_scale, _p(sc.view), _p(sc.proj), sc.W, sc.H,
                              s.tanfovx, s.tanfovy, reps, ms, ctypes.byref(R))
    if rc != 0:
        raise RuntimeError("reference binning timing failed")
    return list(ms), R.value
