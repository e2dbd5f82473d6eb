"""The reference's handle ABI, driven exactly as the reference's Python front end
drives it (python/dart_cuda/core/tensor/gpu_tensor.py): create_tensor,
aft_forward / layernorm_forward / add_tensor_row_broadcast /
cross_entropy_loss, backward, get_tensor_data / get_tensor_grad."""
import ctypes

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from dart_cuda_b200 import lib

    return lib()


FP = ctypes.POINTER(ctypes.c_float)


def relerr(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30))


class H:
    """Minimal handle helper (rows = shape[0], cols = product of the rest)."""

    def __init__(self, L, arr):
        arr = np.ascontiguousarray(arr, np.float32)
        self.shape = arr.shape
        r = arr.shape[0]
        c = int(np.prod(arr.shape[1:])) if arr.ndim > 1 else 1
        self.L = L
        self.h = L.create_tensor(r, c, arr.ctypes.data_as(FP))

    @classmethod
    def wrap(cls, L, h, shape):
        o = cls.__new__(cls)
        o.L, o.h, o.shape = L, h, shape
        return o

    def data(self):
        out = np.empty(self.shape, np.float32)
        self.L.get_tensor_data(self.h, out.ctypes.data_as(FP))
        return out

    def grad(self):
        out = np.empty(self.shape, np.float32)
        self.L.get_tensor_grad(self.h, out.ctypes.data_as(FP))
        return out

    def free(self):
        self.L.destroy_tensor(self.h)


def seed_grad(L, out: H, dOut):
    """Scalar loss sum(out * dOut): backward seeds out.grad = dOut."""
    g = H(L, dOut)
    prod = H.wrap(L, L.mul_tensors(out.h, g.h), out.shape)
    s = H.wrap(L, L.sum_tensor(prod.h), (1, 1))
    return s, [g, prod, s]


@pytest.mark.parametrize("masked", [True, False])
def test_aft_forward_backward_handles(L, masked):
    rng = np.random.default_rng(21)
    T_, D = 64, 128
    Q, K, V, dZ = (rng.standard_normal((T_, D)).astype(np.float32) for _ in range(4))
    W = (0.02 * rng.standard_normal((T_, T_))).astype(np.float32)
    hq, hk, hv, hw = (H(L, a) for a in (Q, K, V, W))
    z = H.wrap(L, L.aft_forward(hq.h, hk.h, hv.h, hw.h, masked), (T_, D))
    s, extra = seed_grad(L, z, dZ)
    L.backward(s.h)
    Zr = oracle.aft_full_fwd(Q, K, V, W, masked)
    gr = oracle.aft_full_bwd(Q, K, V, W, dZ, masked)
    assert relerr(z.data(), Zr) < 1e-3
    for h, r in zip((hq, hk, hv, hw), gr):
        assert relerr(h.grad(), r) < 1e-3
    # A second backward on the same graph follows the reference's rule
    # (engine.cu:145-195): only the root's grad is re-seeded, every other grad
    # keeps accumulating.  z.grad becomes 1*dZ + 2*dZ = 3*dZ, so K's grad
    # grows from g1 to g1 + 3*g1.
    g1 = hk.grad()
    L.backward(s.h)
    np.testing.assert_allclose(hk.grad(), 4 * g1, rtol=1e-4, atol=1e-5)
    for h in (*extra, z, hq, hk, hv, hw):
        h.free()


def test_aft_posbias_wider_than_T(L):
    """posBias allocated [maxSeqLen, maxSeqLen] is read with row stride T."""
    rng = np.random.default_rng(22)
    T_, D, Tmax = 20, 16, 32
    Q, K, V, dZ = (rng.standard_normal((T_, D)).astype(np.float32) for _ in range(4))
    Wbig = (0.3 * rng.standard_normal((Tmax, Tmax))).astype(np.float32)
    hq, hk, hv, hw = H(L, Q), H(L, K), H(L, V), H(L, Wbig)
    z = H.wrap(L, L.aft_forward(hq.h, hk.h, hv.h, hw.h, True), (T_, D))
    s, extra = seed_grad(L, z, dZ)
    L.backward(s.h)
    flat = Wbig.reshape(-1)
    Zr = oracle.aft_full_fwd(Q, K, V, flat, True, ldw=T_)
    dWr = np.zeros(T_ * T_, np.float32)
    gr = oracle.aft_full_bwd(Q, K, V, flat, dZ, True, ldw=T_,
                             grads=(np.zeros((1, T_, D), np.float32), np.zeros((1, T_, D), np.float32),
                                    np.zeros((1, T_, D), np.float32), dWr))
    assert relerr(z.data(), Zr) < 1e-3
    got = hw.grad().reshape(-1)
    assert relerr(got[: T_ * T_], dWr) < 1e-3
    assert np.all(got[T_ * T_:] == 0)


def test_aft_cross_handles(L):
    rng = np.random.default_rng(23)
    TDec, TEnc, D = 12, 5, 8
    Q, dZ = (rng.standard_normal((TDec, D)).astype(np.float32) for _ in range(2))
    K, V = (rng.standard_normal((TEnc, D)).astype(np.float32) for _ in range(2))
    W = (0.3 * rng.standard_normal((TDec, TEnc))).astype(np.float32)
    hq, hk, hv, hw = (H(L, a) for a in (Q, K, V, W))
    z = H.wrap(L, L.aft_cross_forward(hq.h, hk.h, hv.h, hw.h), (TDec, D))
    s, extra = seed_grad(L, z, dZ)
    L.backward(s.h)
    assert relerr(z.data(), oracle.aft_cross_fwd(Q, K, V, W)) < 1e-3
    for h, r in zip((hq, hk, hv, hw), oracle.aft_cross_bwd(Q, K, V, W, dZ)):
        assert relerr(h.grad(), r) < 1e-3


def test_layernorm_bias_ce_handles(L):
    rng = np.random.default_rng(24)
    R, C, V = 64, 256, 65
    x = rng.standard_normal((R, C)).astype(np.float32)
    gamma = np.ones((1, C), np.float32)
    beta = np.zeros((1, C), np.float32)
    wout = (0.02 * rng.standard_normal((1, V))).astype(np.float32)
    hx, hg, hb = H(L, x), H(L, gamma), H(L, beta)
    y = H.wrap(L, L.layernorm_forward(hx.h, hg.h, hb.h, 1e-5), (R, C))
    np.testing.assert_allclose(y.data().mean(1), 0, atol=1e-5)
    # bias add on [R, V] logits, then CE
    logits_np = rng.standard_normal((R, V)).astype(np.float32)
    hl, hbias = H(L, logits_np), H(L, wout)
    lg = H.wrap(L, L.add_tensor_row_broadcast(hl.h, hbias.h), (R, V))
    tg = rng.integers(0, V, R).astype(np.int32)
    loss = H.wrap(L, L.cross_entropy_loss(lg.h, tg.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), R, V), (1, 1))
    L.backward(loss.h)
    ref_loss, _ = oracle.ce_fwd(logits_np + wout, tg)
    assert abs(float(loss.data()[0, 0]) - ref_loss) < 1e-5 * abs(ref_loss)
    g = oracle.ce_bwd(logits_np + wout, tg)
    assert relerr(hl.grad(), g) < 1e-5
    assert relerr(hbias.grad()[0], g.sum(0)) < 1e-4
