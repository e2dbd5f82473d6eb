"""The cross-entropy forward that allocates nothing, for callers that cannot
let the library allocate device memory during a call.

It is checked through the C ABI against the allocating entry point
(dc_ce_fwd with no row-loss buffer, which takes its scratch from the
stream-ordered allocator) on two calls in a row, within the 1e-5 relative
tolerance of the other cross-entropy tests.  The file sorts last so that a run
stopping at the first failure has already run every other test; it also
passes on its own in a fresh process, where its first call is the one that
resolves the library's scratch array on the device.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_ROWS = 65536


def _bind():
    from dart_cuda_b200 import _lib

    L = _lib.lib()
    f = L.dc_ce_fwd_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                  ctypes.c_float, ctypes.c_void_p]
    return L, f


def test_ce_fwd_noalloc_matches_allocating_entry_point():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    L, noalloc = _bind()
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(5)
    # two calls in a row; the second uses fewer rows than the first, so the
    # shared scratch still holds stale rows beyond T that must not leak in
    for T, V in ((4096, 65), (300, 8192)):
        x = torch.from_numpy((2 * rng.standard_normal((T, V))).astype(np.float32)).cuda()
        y = torch.from_numpy(rng.integers(0, V, T).astype(np.int32)).cuda()
        got = torch.empty(1, device="cuda")
        ref = torch.empty(1, device="cuda")
        assert noalloc(x.data_ptr(), y.data_ptr(), got.data_ptr(), T, V, 0.1, stream) == 0
        assert L.dc_ce_fwd(x.data_ptr(), y.data_ptr(), ref.data_ptr(), None, T, V, 0.1, stream) == 0
        torch.cuda.synchronize()
        g, r = float(got), float(ref)
        assert abs(g - r) <= 1e-5 * abs(r), (T, V, g, r)


def test_ce_fwd_noalloc_queued_calls_and_max_rows():
    """Three calls queued back to back on one stream with no synchronisation
    between them (each call's row-loss kernel must wait until the previous
    call's mean has read the shared array), the first at the maximum row
    count so the array's last entries are used, then compared one by one."""
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    L, noalloc = _bind()
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(6)
    cases = []
    for T, V in ((MAX_ROWS, 8), (1000, 512), (MAX_ROWS - 3, 16)):
        x = torch.from_numpy((3 * rng.standard_normal((T, V))).astype(np.float32)).cuda()
        y = torch.from_numpy(rng.integers(0, V, T).astype(np.int32)).cuda()
        cases.append((T, V, x, y, torch.empty(1, device="cuda")))
    torch.cuda.synchronize()
    for T, V, x, y, out in cases:
        assert noalloc(x.data_ptr(), y.data_ptr(), out.data_ptr(), T, V, 0.1, stream) == 0
    torch.cuda.synchronize()
    for T, V, x, y, out in cases:
        ref = torch.empty(1, device="cuda")
        assert L.dc_ce_fwd(x.data_ptr(), y.data_ptr(), ref.data_ptr(), None, T, V, 0.1, stream) == 0
        torch.cuda.synchronize()
        g, r = float(out), float(ref)
        assert abs(g - r) <= 1e-5 * abs(r), (T, V, g, r)


def test_ce_fwd_noalloc_rejects_too_many_rows():
    L, noalloc = _bind()
    stream = torch.cuda.current_stream().cuda_stream
    dummy = torch.empty(1, device="cuda")
    rc = noalloc(dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), MAX_ROWS + 1, 8, 0.1, stream)
    assert rc == 1  # DC_ERR_INVALID
    assert b"exceeds" in L.dc_last_error()
