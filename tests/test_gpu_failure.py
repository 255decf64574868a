"""Failure detection without a GPU fault: the onesweep sort's bounded look-back
wait.  A CTA waits for its predecessor tile's digit counts; if they never come,
it gives up after a spin limit, latches VI_DEVICE_LOOKBACK_TIMEOUT in the
status word and returns, and the entry point reports VI_ERR_DEVICE instead of
handing back unsorted keys as a success.

vi_sort_pairs_withheld_tile withholds tile 0 of every digit pass (one CTA fewer
runs; the tile counter starts at 1), so tile 1 waits for a predecessor that
never publishes.  Every launched CTA still works on an existing tile and writes
only inside the outputs, and the wait is limited to a few polls.  The context
must stay usable: a normal sort afterwards on the same stream is exact."""
import ctypes
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "volume-integration_b200",
                   "volume_integration", "libvi_b200.so")
VI_ERR_DEVICE = 6
VI_DEVICE_LOOKBACK_TIMEOUT = 0x1


def _lib():
    lib = ctypes.CDLL(LIB)
    vp, u64, i = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int
    lib.vi_sort_pairs.argtypes = [vp, vp, vp, vp, u64, i, i, vp, ctypes.c_size_t, vp]
    lib.vi_sort_pairs_temp_bytes.restype = ctypes.c_size_t
    lib.vi_sort_pairs_temp_bytes.argtypes = [u64, i, i]
    lib.vi_sort_pairs_withheld_tile.argtypes = [vp, vp, vp, vp, u64, i, i, vp, ctypes.c_size_t, i,
                                                ctypes.POINTER(ctypes.c_uint32), vp]
    lib.vi_last_error.restype = ctypes.c_char_p
    return lib


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("n,begin,end", [(4 * 3072, 0, 64), (5 * 3072 + 17, 0, 45)])
def test_lookback_wait_gives_up_and_is_reported(n, begin, end):
    lib = _lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    g = torch.Generator().manual_seed(n)
    keys = torch.randint(0, 2 ** 62, (n,), generator=g, dtype=torch.int64).cuda()
    vals = torch.arange(n, dtype=torch.int32).cuda()
    tb = lib.vi_sort_pairs_temp_bytes(n, begin, end)
    temp = torch.empty(tb, dtype=torch.uint8, device="cuda")
    k, v = keys.clone(), vals.clone()
    ko, vo = torch.empty_like(k), torch.empty_like(v)
    st = ctypes.c_uint32(0)
    rc = lib.vi_sort_pairs_withheld_tile(_p(k), _p(v), _p(ko), _p(vo), n, begin, end, _p(temp), tb, 64,
                                         ctypes.byref(st), stream)
    assert rc == VI_ERR_DEVICE, (rc, lib.vi_last_error())
    assert st.value & VI_DEVICE_LOOKBACK_TIMEOUT
    assert b"look-back" in lib.vi_last_error()
    # the context is intact: the same sort without the withheld tile is exact
    k, v = keys.clone(), vals.clone()
    assert lib.vi_sort_pairs(_p(k), _p(v), _p(ko), _p(vo), n, begin, end, _p(temp), tb, stream) == 0, \
        lib.vi_last_error()
    kk = keys.cpu().numpy().view(np.uint64)
    digit = (kk >> np.uint64(begin)) & np.uint64(2 ** 64 - 1 if end - begin == 64 else (1 << (end - begin)) - 1)
    np.testing.assert_array_equal(vo.cpu().numpy(), np.argsort(digit, kind="stable").astype(np.int32))


def test_withheld_tile_hook_rejects_single_tile_and_bad_limits():
    lib = _lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    n = 3072
    keys = torch.zeros(n, dtype=torch.int64, device="cuda")
    vals = torch.zeros(n, dtype=torch.int32, device="cuda")
    tb = lib.vi_sort_pairs_temp_bytes(n, 0, 64)
    temp = torch.empty(tb, dtype=torch.uint8, device="cuda")
    st = ctypes.c_uint32(0)
    assert lib.vi_sort_pairs_withheld_tile(_p(keys), _p(vals), _p(keys), _p(vals), n, 0, 64, _p(temp), tb, 64,
                                           ctypes.byref(st), stream) == 1
    assert lib.vi_sort_pairs_withheld_tile(_p(keys), _p(vals), _p(keys), _p(vals), n, 0, 64, _p(temp), tb, 0,
                                           ctypes.byref(st), stream) == 1


def test_render_staging_wait_gives_up_and_is_reported(monkeypatch):
    # The render's bulk copies complete on an mbarrier that every pixel waits
    # for, at most a bounded number of polls.  The testing hook withholds each
    # batch's barrier arrival and copies, so nothing completes the wait (and
    # nothing is in flight): every tile must give up, latch
    # VI_DEVICE_STAGE_TIMEOUT, read the records
    # from global memory instead, and produce exactly the images of a normal
    # run.  With debug on, the forward reports the bit as an error.
    import vi_testlib as tl
    VI_DEVICE_STAGE_TIMEOUT = 0x4
    means, conf, s = tl.custom_scene(seed=21, P=400)
    s.debug = False
    monkeypatch.setenv("VI_RENDER_TMA", "1")  # the staged render, without the hook
    ok = tl.gpu_state(means, conf, s)
    assert not ok["status"][0] & VI_DEVICE_STAGE_TIMEOUT
    monkeypatch.setenv("VI_RENDER_TMA_TEST_TIMEOUT", "1")
    to = tl.gpu_state(means, conf, s)
    assert to["status"][0] & VI_DEVICE_STAGE_TIMEOUT
    for k in ("n_contrib", "final_T", "contrib_idx", "delta_t", "contrib_rec"):
        np.testing.assert_array_equal(to[k], ok[k])
    g_to = tl.run_gpu(means, conf, s, state=False)
    monkeypatch.delenv("VI_RENDER_TMA_TEST_TIMEOUT")
    g_ok = tl.run_gpu(means, conf, s, state=False)
    for k in ("out_color", "out_features", "visibility"):
        np.testing.assert_array_equal(g_to[k], g_ok[k])
    # debug: the status word is read after the render and raises
    monkeypatch.setenv("VI_RENDER_TMA_TEST_TIMEOUT", "1")
    s.debug = True
    with pytest.raises(RuntimeError, match="0x4"):
        tl.run_gpu(means, conf, s, state=False)
    monkeypatch.delenv("VI_RENDER_TMA_TEST_TIMEOUT")
    torch.cuda.synchronize()
