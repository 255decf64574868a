"""vi_sort_pairs_noalloc, the sort for callers that must not allocate device
memory (hosts that own all device memory, or cannot take the device-wide
synchronisation of cudaMalloc/cudaFree mid-frame), against the allocating
vi_sort_pairs.  Both are called through the C ABI of libvi_b200.so; the sorted
keys and values must agree exactly on two calls in a row with different sizes
and bit ranges, so the second call also shows that the shared scratch array is
reset between calls.  Collected last on purpose (file name)."""
import ctypes
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "volume-integration_b200",
                   "volume_integration", "libvi_b200.so")


def _lib():
    lib = ctypes.CDLL(LIB)
    vp, u64, i = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int
    lib.vi_sort_pairs.argtypes = [vp, vp, vp, vp, u64, i, i, vp, ctypes.c_size_t, vp]
    lib.vi_sort_pairs_temp_bytes.restype = ctypes.c_size_t
    lib.vi_sort_pairs_temp_bytes.argtypes = [u64, i, i]
    lib.vi_sort_pairs_noalloc.argtypes = [vp, vp, vp, vp, u64, i, i, vp]
    lib.vi_last_error.restype = ctypes.c_char_p
    return lib


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _inputs(n, seed):
    g = torch.Generator().manual_seed(seed)
    keys = torch.randint(-(2 ** 62), 2 ** 62, (n,), generator=g, dtype=torch.int64)
    keys[: n // 4] = keys[0]  # repeated keys: the order of their values checks stability
    return keys.cuda(), torch.arange(n, dtype=torch.int32).cuda()


def test_noalloc_sort_matches_allocating_sort_on_two_calls():
    lib = _lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # the largest n the scratch array allows, over all 64 key bits (where its
    # look-back words fill it most), then a smaller, offset bit range
    for n, begin, end, seed in ((1 << 20, 0, 64, 1), (300_001, 4, 45, 2)):
        keys, vals = _inputs(n, seed)
        # allocating entry point, caller-provided temp buffer
        k1, v1 = keys.clone(), vals.clone()
        ko1, vo1 = torch.empty_like(k1), torch.empty_like(v1)
        tb = lib.vi_sort_pairs_temp_bytes(n, begin, end)
        temp = torch.empty(tb, dtype=torch.uint8, device="cuda")
        assert lib.vi_sort_pairs(_ptr(k1), _ptr(v1), _ptr(ko1), _ptr(vo1), n, begin, end, _ptr(temp), tb,
                                 stream) == 0, lib.vi_last_error()
        # non-allocating entry point
        k2, v2 = keys.clone(), vals.clone()
        ko2, vo2 = torch.empty_like(k2), torch.empty_like(v2)
        assert lib.vi_sort_pairs_noalloc(_ptr(k2), _ptr(v2), _ptr(ko2), _ptr(vo2), n, begin, end, stream) == 0, \
            lib.vi_last_error()
        torch.cuda.synchronize()
        assert torch.equal(ko1, ko2) and torch.equal(vo1, vo2)
        # and both are the stable order of the selected bits
        k = keys.cpu().numpy().view(np.uint64)
        digit = (k >> np.uint64(begin)) & np.uint64((1 << (end - begin)) - 1 if end - begin < 64 else 2 ** 64 - 1)
        np.testing.assert_array_equal(vo2.cpu().numpy(), np.argsort(digit, kind="stable").astype(np.int32))


def test_noalloc_sort_rejects_sizes_beyond_its_scratch():
    lib = _lib()
    n = (1 << 20) + 1
    keys, vals = _inputs(16, 3)
    rc = lib.vi_sort_pairs_noalloc(_ptr(keys), _ptr(vals), _ptr(keys), _ptr(vals), n, 0, 64,
                                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 1 and b"VI_SORT_NOALLOC_MAX_KEYS" in lib.vi_last_error()
