"""The allocation-free linear entry point (eii_linear_noalloc) gives the same integers as eii_linear.

eii_linear_noalloc is for callers that must not allocate device memory (their device memory is owned
by another allocator, or they cannot afford cudaMalloc's implicit synchronisation); it keeps its
scratch in fixed device arrays of the library.  This file is named to be collected last, so a run
that stops at the first failure has already run every other test."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _noalloc_fn():
    import _eii
    f = _eii.lib().eii_linear_noalloc
    P = ctypes.c_void_p
    f.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                  ctypes.c_int, P, P, P]
    f.restype = ctypes.c_int
    return f


def _case(seed, M, K, N, bits_in):
    rng = np.random.default_rng(seed)
    lo, hi = -(1 << (bits_in - 1)), 1 << (bits_in - 1)
    a = rng.integers(lo, hi, size=(M, K), dtype=np.int64)
    a[0] = lo
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int64).astype(np.int8)
    m = rng.integers(1 << 13, (1 << 14) + 1, size=N, dtype=np.int64)
    n = rng.integers(18, 30, size=N, dtype=np.int64)
    return a, W, m, n


def _dev(*arrays):
    import torch
    return [torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in arrays]


def test_noalloc_linear_matches_eii_linear_twice(base_model_path):
    import torch
    import _eii
    eng = _eii.Engine(base_model_path, 0)
    fn = _noalloc_fn()
    torch.cuda.set_device(0)
    try:
        # two calls in a row with different shapes and formats; the second reuses the scratch
        for seed, (M, K, N, bits_in, f_in, f_out, bits_out) in enumerate(
                [(300, 576, 192, 16, 12, 10, 16), (129, 1536, 576, 32, 23, 15, 64)]):
            a, W, m, n = _case(seed, M, K, N, bits_in)
            want_out, want_acc = eng.linear(a, bits_in, W, m, n, f_in, f_out, bits_out)
            ad, Wd, md, nd = _dev(a, W, m, n)
            out = torch.empty((M, N), dtype=torch.int64, device="cuda")
            acc = torch.empty((M, N), dtype=torch.int64, device="cuda")
            torch.cuda.synchronize()
            rc = fn(ad.data_ptr(), M, K, bits_in, Wd.data_ptr(), md.data_ptr(), nd.data_ptr(), N, f_in, f_out,
                    bits_out, out.data_ptr(), acc.data_ptr(), None)
            assert rc == _eii.EII_OK, _eii.lib().eii_last_error()
            assert np.array_equal(acc.cpu().numpy(), want_acc)
            assert np.array_equal(out.cpu().numpy(), want_out)
        # sizes beyond the static scratch are rejected before any GPU work
        big = torch.empty(8, dtype=torch.int64, device="cuda")
        rc = fn(big.data_ptr(), 16384, 1536, 32, big.data_ptr(), big.data_ptr(), big.data_ptr(), 64, 0, 0, 16,
                big.data_ptr(), None, None)
        assert rc == _eii.EII_ERR_ARG
        assert b"exceeds the static scratch" in _eii.lib().eii_last_error()
    finally:
        eng.close()


def test_noalloc_allocates_nothing_and_runs_on_a_side_stream(base_model_path):
    """After the first call on the device, further calls leave the device's free memory unchanged
    (cudaMemGetInfo), and a call without acc on a non-default stream equals eii_linear."""
    import torch
    import _eii
    eng = _eii.Engine(base_model_path, 0)
    fn = _noalloc_fn()
    try:
        M, K, N, bits_in, f_in, f_out, bits_out = 257, 576, 576, 16, 13, 10, 16
        a, W, m, n = _case(7, M, K, N, bits_in)
        want_out, _ = eng.linear(a, bits_in, W, m, n, f_in, f_out, bits_out)
        ad, Wd, md, nd = _dev(a, W, m, n)
        out = torch.empty((M, N), dtype=torch.int64, device="cuda")
        side = torch.cuda.Stream()
        torch.cuda.synchronize()
        args = (ad.data_ptr(), M, K, bits_in, Wd.data_ptr(), md.data_ptr(), nd.data_ptr(), N, f_in, f_out, bits_out,
                out.data_ptr(), None, side.cuda_stream)
        assert fn(*args) == _eii.EII_OK, _eii.lib().eii_last_error()  # first call: resolves the scratch
        out.zero_()  # torch's own kernels load lazily (device memory of their modules): use them once first
        torch.cuda.synchronize()
        out.cpu()
        free0, _ = torch.cuda.mem_get_info()
        got = []
        for _ in range(2):
            out.zero_()
            torch.cuda.synchronize()
            assert fn(*args) == _eii.EII_OK, _eii.lib().eii_last_error()
            got.append(out.cpu().numpy())
        free1, _ = torch.cuda.mem_get_info()
        assert free1 == free0, f"free device memory changed by {free0 - free1} bytes"
        for g in got:
            assert np.array_equal(g, want_out)
    finally:
        eng.close()


def test_noalloc_argument_errors(base_model_path):
    """A column shift n + f_in - f_out outside [1, 62], N above EII_NOALLOC_MAX_N and an activation
    outside the signed bits_in range are argument errors; a good call afterwards is exact."""
    import torch
    import _eii
    eng = _eii.Engine(base_model_path, 0)
    fn = _noalloc_fn()
    try:
        M, K, N = 64, 576, 64
        a, W, m, n = _case(3, M, K, N, 16)
        ad, Wd, md, nd = _dev(a, W, m, n)
        out = torch.empty((M, N), dtype=torch.int64, device="cuda")
        torch.cuda.synchronize()
        # n in [18, 30): f_in - f_out = -40 gives shifts below 1
        rc = fn(ad.data_ptr(), M, K, 16, Wd.data_ptr(), md.data_ptr(), nd.data_ptr(), N, 0, 40, 16, out.data_ptr(),
                None, None)
        assert rc == _eii.EII_ERR_ARG and b"[1, 62]" in _eii.lib().eii_last_error()
        rc = fn(ad.data_ptr(), M, K, 16, Wd.data_ptr(), md.data_ptr(), nd.data_ptr(), 49168, 12, 10, 16,
                out.data_ptr(), None, None)
        assert rc == _eii.EII_ERR_ARG and b"exceeds the maximum" in _eii.lib().eii_last_error()
        bad = ad.clone()
        bad[5, 9] = 1 << 15
        rc = fn(bad.data_ptr(), M, K, 16, Wd.data_ptr(), md.data_ptr(), nd.data_ptr(), N, 12, 10, 16, out.data_ptr(),
                None, None)
        assert rc == _eii.EII_ERR_ARG and b"outside the signed 16-bit range" in _eii.lib().eii_last_error()
        rc = fn(ad.data_ptr(), M, K, 16, Wd.data_ptr(), md.data_ptr(), nd.data_ptr(), N, 12, 10, 16, out.data_ptr(),
                None, None)
        assert rc == _eii.EII_OK, _eii.lib().eii_last_error()
        want_out, _ = eng.linear(a, 16, W, m, n, 12, 10, 16)
        assert np.array_equal(out.cpu().numpy(), want_out)
    finally:
        eng.close()
