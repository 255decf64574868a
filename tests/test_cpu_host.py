"""CPU-only tests: the C ABI library loads and exports what its header declares,
the drop-in Python surface matches the reference's, and the host-side checks
raise before any device work."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "volume-integration_b200")
HEADER = os.path.join(ROOT, "include", "volume_integration_b200.h")
LIB = os.path.join(ROOT, "volume-integration_b200", "volume_integration", "libvi_b200.so")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(vi_[a-z0-9_]+)\s*\(", text)) - {"vi_resize_fn"})


def test_c_abi_exports_every_declared_symbol():
    lib = ctypes.CDLL(LIB)
    names = declared_functions()
    assert "vi_integrate_primitives" in names and "vi_integrate_primitives_backward" in names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_c_abi_host_checks_without_gpu():
    lib = ctypes.CDLL(LIB)
    lib.vi_sort_end_bit.restype = ctypes.c_int
    # getHigherMsb of the tile counts of the benchmark images (integrator_impl.cu:47-62)
    assert [lib.vi_sort_end_bit(t) for t in (64, 2500, 8160, 32400)] == [39, 44, 45, 47]
    lib.vi_last_error.restype = ctypes.c_char_p
    rc = lib.vi_get_state_layout(-1, 0, 1, 1, 1, 3, 4, None)
    assert rc == 1 and b"layout" in lib.vi_last_error()


def test_noalloc_sort_scratch_holds_its_largest_sort():
    # VI_SORT_NOALLOC_MAX_KEYS keys over all 64 bits must fit the fixed scratch
    # array; vi_sort_pairs_temp_bytes covers the same carving plus 512 bytes of
    # alignment and status word, so it bounds the no-allocation sort's need.
    text = open(HEADER).read()
    max_keys = eval(re.search(r"#define VI_SORT_NOALLOC_MAX_KEYS \((.*?)\)", text).group(1).replace("u", ""))
    scratch = eval(re.search(r"#define VI_SORT_NOALLOC_SCRATCH_BYTES \((.*?)\)", text).group(1).replace("u", ""))
    lib = ctypes.CDLL(LIB)
    lib.vi_sort_pairs_temp_bytes.restype = ctypes.c_size_t
    lib.vi_sort_pairs_temp_bytes.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_int]
    assert max_keys == 1 << 20 and scratch == 3 << 20
    for begin, end in ((0, 64), (0, 32), (7, 64)):
        assert lib.vi_sort_pairs_temp_bytes(max_keys, begin, end) <= scratch


def test_settings_fields_and_defaults_match_reference():
    import volume_integration as vi
    s = vi.IntegrationSettings()
    expected = dict(tanfovx=1.0, tanfovy=1.0, image_height=512, image_width=512, near_plane=0.1,
                    max_distance=100.0, primitive_scale=0.01, feature_offset=0, stencil_genus=1, grid_size=3,
                    max_primitives_per_ray=64, occupancy_threshold=0.5, input_feature_dim=2,
                    output_feature_dim=8, intermediate_feature_dim=32, hashgrid_levels=16,
                    num_output_channels=3, debug=False)
    for k, v in expected.items():
        assert getattr(s, k) == v, k
    assert torch.equal(s.viewmatrix, torch.eye(4)) and torch.equal(s.cam_pos, torch.zeros(3))
    assert s.resolution.dtype == torch.int32 and s.feature_table.numel() == 0
    names = [f for f in vi.IntegrationSettings.__dataclass_fields__]
    assert names[:6] == ["viewmatrix", "projmatrix", "cam_pos", "tanfovx", "tanfovy", "image_height"]
    assert hasattr(vi.VolumeIntegrator, "markVisible")


def test_confidence_shape_checks():
    import volume_integration as vi
    s = vi.IntegrationSettings(grid_size=3, cam_pos=torch.zeros(3))
    m = torch.zeros(4, 3)
    with pytest.raises(ValueError):
        vi.integrate_primitives(m, torch.zeros(4, 3, 9), torch.zeros(1), torch.zeros(1), torch.zeros(1), s)
    with pytest.raises(AssertionError):
        vi.integrate_primitives(m, torch.zeros(5, 27), torch.zeros(1), torch.zeros(1), torch.zeros(1), s)
    with pytest.raises(AssertionError):
        vi.integrate_primitives(m, torch.zeros(4, 2, 2, 2), torch.zeros(1), torch.zeros(1), torch.zeros(1), s)


def test_cam_pos_must_be_cuda():
    import volume_integration as vi
    s = vi.IntegrationSettings(cam_pos=torch.zeros(3))
    with pytest.raises(TypeError):
        vi.integrate_primitives(torch.zeros(2, 3), torch.zeros(2, 27), torch.zeros(1), torch.zeros(1),
                                torch.zeros(1), s)


def test_oracle_reference_box_is_the_default():
    """The oracle with the reference's hashgrid box given explicitly is bit-identical to the default."""
    import dataclasses
    import vi_testlib as tl
    means, conf, s = tl.custom_scene(P=60, W=32, H=24, seed=4, device="cpu")
    _, a = tl.oracle_run(means, conf, s)
    _, b = tl.oracle_run(means, conf, dataclasses.replace(s, hash_bounds=(-1.3, -1.3, -1.3, 1.3, 1.3, 1.3)))
    for k in ("out_color", "out_features", "visibility"):
        np.testing.assert_array_equal(a[k], b[k])
    _, c = tl.oracle_run(means, conf, dataclasses.replace(s, hash_bounds=(-1.0, -1.0, -1.0, 1.0, 1.0, 1.0)))
    assert not np.array_equal(a["out_color"], c["out_color"])


def test_binding_raises_runtime_error_on_a_c_abi_error():
    """A status code from the C ABI becomes a RuntimeError carrying vi_last_error()
    (run in a child process: a binding built against a mismatched C++ runtime
    crashes here instead of raising)."""
    import subprocess
    import sys
    code = ("import sys; sys.path.insert(0, %r)\n"
            "import torch\n"
            "from volume_integration import _C\n"
            "e = torch.empty(0, dtype=torch.uint8)\n"
            "try:\n"
            "    _C.state_views(e, e, e, -5, 0, 16, 16, 8, 3, 4)\n"
            "except RuntimeError as ex:\n"
            "    print('raised:', ex)\n") % PKG
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "raised: volume_integration: bad layout query (status 1)" in r.stdout


def test_exact_restatement_reproduces_the_forward():
    """The float64 restatement behind the exact-gradient tests computes the
    oracle's forward images (it is the forward, on the same discrete structure)."""
    import vi_testlib as tl
    import exact_lib as ex
    means, conf, s = tl.custom_scene(P=50, W=48, H=32, seed=5, device="cpu", bg=(0.3, 0.1, 0.6))
    dc, df = tl.random_grads(s, seed=1, device="cpu")
    dv = torch.zeros(s.image_height, s.image_width)
    img, grads, f = ex.exact_grads(means, conf, s, dc, df, dv)
    np.testing.assert_allclose(img["out_color"], f["out_color"], atol=1e-4)
    np.testing.assert_allclose(img["out_features"], f["out_features"], atol=1e-4)
    np.testing.assert_allclose(img["visibility"], f["visibility"], atol=1e-4)
    assert np.abs(grads["dL_dmeans3D"]).max() > 0 and np.abs(grads["dL_dfeature_table"]).max() > 0


def _lib():
    import ctypes
    lib = ctypes.CDLL(os.path.join(PKG, "volume_integration", "libvi_b200.so"))
    lib.vi_last_error.restype = ctypes.c_char_p
    return lib


def _forward_ex_args(flags, bounds):
    """Arguments of vi_integrate_primitives_ex for an empty scene (P = 0): the
    call validates its settings and returns before touching the device."""
    import ctypes
    RESIZE = ctypes.CFUNCTYPE(ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t)
    cb = RESIZE(lambda u, n: 0)
    vp, f, i, u, u64 = ctypes.c_void_p, ctypes.c_float, ctypes.c_int, ctypes.c_uint, ctypes.c_uint64
    hb = (ctypes.c_float * 6)(*bounds) if bounds is not None else None
    R = ctypes.c_int(0)
    args = [cb, None, cb, None, cb, None, vp(0), vp(0), vp(0), ctypes.byref(R), i(0), vp(0), vp(0), f(0.1), vp(0),
            vp(0), vp(0), f(1.0), f(1.0), i(0), i(0), f(0.01), f(100.0), vp(0), u64(0), vp(0), vp(0), vp(0), i(64),
            vp(0), u64(0), vp(0), u64(0), i(1), i(3), i(8), f(0.5), vp(0), u(2), u(4), u(8), u(4), u(3), i(0), vp(0),
            hb, u(flags)]
    return args, cb


@pytest.mark.parametrize("G,flags,rc,msg", [(6, 0, 2, b"grid_size=6"), (4, 1, 2, b"exact_gradients needs grid_size"),
                                            (5, 1, 2, b"exact_gradients needs grid_size")])
def test_c_abi_grid_size_limits(G, flags, rc, msg):
    # grid sizes 1..5 are supported (the reference's MAX_GRID_SIZE); the
    # exact-gradient extension only up to 3
    lib = _lib()
    args, _keep = _forward_ex_args(flags, None)
    args[34] = ctypes.c_int(G)
    assert lib.vi_integrate_primitives_ex(*args) == rc
    assert msg in lib.vi_last_error()


@pytest.mark.parametrize("flags,bounds,msg", [
    (2, None, b"unknown flags"),
    (0, (0.0, 0.0, 0.0, 1.0, -1.0, 1.0), b"hash_bounds axis 1"),
    (0, (0.0, 0.0, 0.0, 1.0, 1.0, float("nan")), b"hash_bounds axis 2"),
])
def test_c_abi_rejects_bad_flags_and_bounds(flags, bounds, msg):
    lib = _lib()
    args, _keep = _forward_ex_args(flags, bounds)
    assert lib.vi_integrate_primitives_ex(*args) == 1
    assert msg in lib.vi_last_error()

