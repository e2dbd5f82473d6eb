"""A bounded mbarrier wait of the tensor-core kernels running out, on a GPU,
without a fault: the test-only library (lib/libmat_mul_waittest.so, built by
dart_cuda_b200/build.py with DC_TEST_WITHHOLD and a 50 ms wait limit) lets the
next launch's CTA 0 withhold the TMA load and the arrival of its first
pipeline stage.  The MMA issuer's wait for that stage runs out: it raises the
CTA's abort flag and a status bit, the epilogue and producer see the flag and
stop, the producer's drain of its in-flight copies gives up on the withheld
stage after the limit, issued MMAs are drained by a commit, TMEM is freed and
the kernel returns.  The host then reads DC_ERR_DEVICE with the timeout bits,
and the same context runs a normal call correctly afterwards.

The product library (lib/libmat_mul.so) contains none of this code."""
import ctypes
from ctypes import POINTER, byref, c_int, c_size_t, c_void_p
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LIB = Path(__file__).resolve().parents[1] / "dart_cuda_b200" / "lib" / "libmat_mul_waittest.so"
DC_BF16, DC_AFT_CAUSAL, DC_ERR_DEVICE = 1, 1, 5
TIMEOUT_FULL, TIMEOUT_ACC, TIMEOUT_DRAIN = 0x1, 0x4, 0x8


def _lib():
    L = ctypes.CDLL(str(LIB))
    L.dc_test_withhold_next.argtypes = [c_int]
    L.dc_aft_fwd.argtypes = [c_void_p] * 4 + [c_int, c_void_p] + [c_int] * 6 + [c_void_p, c_size_t, c_void_p]
    L.dc_aft_workspace_size.argtypes = [c_int] * 6 + [POINTER(c_size_t)]
    L.dc_device_status.argtypes = [c_void_p, POINTER(c_int)]
    L.dc_last_error.restype = ctypes.c_char_p
    return L


def test_withheld_stage_times_out_and_context_survives():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    assert LIB.exists(), "build the test library: python -m dart_cuda_b200.build"
    L = _lib()
    dev = torch.device("cuda:0")
    B, T, D = 2, 256, 128  # single-CTA tiles (no CTA pairs below T = 1024)
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    Q, K, V = (torch.randn(B, T, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(3))
    w = 0.02 * torch.randn(T, T, device=dev, generator=g)
    n = c_size_t(0)
    assert L.dc_aft_workspace_size(B, T, T, D, DC_BF16, DC_AFT_CAUSAL, byref(n)) == 0
    ws = torch.empty(n.value + 1024, dtype=torch.uint8, device=dev)
    wsp = (ws.data_ptr() + 1023) // 1024 * 1024
    stream = torch.cuda.current_stream().cuda_stream

    def fwd(Z):
        return L.dc_aft_fwd(Q.data_ptr(), K.data_ptr(), V.data_ptr(), w.data_ptr(), T, Z.data_ptr(), B, T, T, D,
                            DC_BF16, DC_AFT_CAUSAL, wsp, n.value, stream)

    bits = c_int(0)
    assert L.dc_device_status(stream, byref(bits)) == 0 and bits.value == 0
    Z_bad = torch.zeros_like(Q)
    assert L.dc_test_withhold_next(1) == 0
    assert fwd(Z_bad) == 0  # the launch itself is fine; the kernel reports on the device
    rc = L.dc_device_status(stream, byref(bits))
    assert rc == DC_ERR_DEVICE, (rc, L.dc_last_error())
    assert bits.value & (TIMEOUT_FULL | TIMEOUT_ACC), hex(bits.value)
    assert not bits.value & ~(TIMEOUT_FULL | TIMEOUT_ACC | 0x2 | TIMEOUT_DRAIN), hex(bits.value)
    assert b"bounded wait" in L.dc_last_error()
    # the status word was cleared and the context still works: a normal call
    # gives the product library's result bit for bit
    Z_ok = torch.zeros_like(Q)
    assert fwd(Z_ok) == 0
    assert L.dc_device_status(stream, byref(bits)) == 0 and bits.value == 0
    from dart_cuda_b200 import ops

    Z_ref = ops.aft_fwd(Q, K, V, w, causal=True)
    assert torch.equal(Z_ok, Z_ref)
    torch.cuda.synchronize()
