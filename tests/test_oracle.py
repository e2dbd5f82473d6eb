"""The fp32 C restatement of the reference kernels (oracle/aft_oracle.c)
against independent float64 formulations and finite differences.  CPU only."""
import numpy as np
import pytest

import oracle


def _inputs(rng, B, T, D, wscale=0.02, seed_shift=0):
    Q = rng.standard_normal((B, T, D)).astype(np.float32)
    K = rng.standard_normal((B, T, D)).astype(np.float32)
    V = rng.standard_normal((B, T, D)).astype(np.float32)
    W = (wscale * rng.standard_normal((T, T))).astype(np.float32)
    dZ = rng.standard_normal((B, T, D)).astype(np.float32)
    return Q, K, V, W, dZ


def relerr(a, b):
    """Normwise relative error: max|a-b| / max|b|."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


@pytest.mark.parametrize("masked", [True, False])
@pytest.mark.parametrize("B,T,D", [(1, 1, 1), (2, 7, 5), (4, 64, 128)])
def test_aft_fwd_matches_f64(rng, masked, B, T, D):
    Q, K, V, W, _ = _inputs(rng, B, T, D)
    Z = oracle.aft_full_fwd(Q, K, V, W, masked)
    Zr = oracle.aft_f64(Q, K, V, W, masked)
    assert relerr(Z, Zr) < 1e-5


@pytest.mark.parametrize("masked", [True, False])
@pytest.mark.parametrize("B,T,D", [(1, 1, 1), (3, 9, 6), (2, 33, 16)])
def test_aft_bwd_matches_f64(rng, masked, B, T, D):
    Q, K, V, W, dZ = _inputs(rng, B, T, D, wscale=0.5)
    got = oracle.aft_full_bwd(Q, K, V, W, dZ, masked)
    ref = oracle.aft_grads_f64(Q, K, V, W, dZ, masked)
    for g, r in zip(got, ref):
        assert relerr(g, r) < 1e-4


def test_aft_bwd_finite_difference(rng):
    """Central differences of L = sum(Z * dZ) in float64 against the
    closed-form float64 gradients used above."""
    B, T, D = 1, 5, 3
    Q, K, V, W, dZ = (x.astype(np.float64) for x in _inputs(rng, B, T, D, wscale=0.7))
    dQ, dK, dV, dW = oracle.aft_grads_f64(Q, K, V, W, dZ, True)
    h = 1e-6

    def L(Q_, K_, V_, W_):
        return float((oracle.aft_f64(Q_, K_, V_, W_, True) * dZ).sum())

    for name, arr, grad in (("Q", Q, dQ), ("K", K, dK), ("V", V, dV), ("W", W, dW)):
        num = np.zeros_like(arr)
        it = np.nditer(arr, flags=["multi_index"])
        for _ in it:
            idx = it.multi_index
            ap = arr.copy(); ap[idx] += h
            am = arr.copy(); am[idx] -= h
            args_p = [Q, K, V, W]; args_m = [Q, K, V, W]
            k = "QKVW".index(name)
            args_p[k] = ap; args_m[k] = am
            num[idx] = (L(*args_p) - L(*args_m)) / (2 * h)
        if name == "W":
            num = np.tril(num)  # entries above the diagonal never enter Z
        assert np.max(np.abs(num - grad)) < 1e-6, name


def test_aft_bwd_accumulates(rng):
    Q, K, V, W, dZ = _inputs(rng, 2, 8, 4)
    g1 = oracle.aft_full_bwd(Q, K, V, W, dZ)
    g2 = oracle.aft_full_bwd(Q, K, V, W, dZ, grads=tuple(x.copy() for x in g1))
    for a, b in zip(g1, g2):
        np.testing.assert_allclose(b, 2 * a, rtol=1e-6, atol=1e-7)


def test_aft_ldw_quirk(rng):
    """The reference indexes WB with row stride T even when the bias was
    allocated wider ([maxSeqLen, maxSeqLen]); ldw reproduces that."""
    T, D, Tmax = 6, 4, 10
    Q, K, V, _, _ = _inputs(rng, 1, T, D)
    Wbig = rng.standard_normal((Tmax, Tmax)).astype(np.float32)
    flat = Wbig.reshape(-1)
    Z_legacy = oracle.aft_full_fwd(Q, K, V, flat, True, ldw=T)
    Wview = flat[: T * T].reshape(T, T)
    np.testing.assert_array_equal(Z_legacy, oracle.aft_full_fwd(Q, K, V, Wview, True))


def test_aft_cross_matches_full_unmasked(rng):
    Q, K, V, W, dZ = _inputs(rng, 1, 12, 8, wscale=0.3)
    Zc = oracle.aft_cross_fwd(Q[0], K[0], V[0], W)
    Zf = oracle.aft_full_fwd(Q[0], K[0], V[0], W, False)
    np.testing.assert_allclose(Zc, Zf, rtol=1e-6, atol=1e-7)
    gc = oracle.aft_cross_bwd(Q[0], K[0], V[0], W, dZ[0])
    gf = oracle.aft_grads_f64(Q[0], K[0], V[0], W, dZ[0], False)
    for a, b in zip(gc, gf):
        assert relerr(a, b) < 1e-4


def test_ce_known_answer():
    """x=[0,0], target 1 -> grad [+0.45, -0.45]
    (reference test/core/tensor_autograd_test.dart:154-166)."""
    g = oracle.ce_bwd(np.zeros((1, 2), np.float32), np.array([1], np.int32))
    np.testing.assert_allclose(g, [[0.45, -0.45]], atol=1e-6)


def test_ce_finite_difference(rng):
    T, V = 4, 7
    x = rng.standard_normal((T, V)).astype(np.float32)
    y = rng.integers(0, V, T).astype(np.int32)
    g = oracle.ce_bwd(x, y)
    h = 1e-2
    for t in range(T):
        for v in range(V):
            xp = x.copy(); xp[t, v] += h
            xm = x.copy(); xm[t, v] -= h
            num = (oracle.ce_fwd(xp, y)[0] - oracle.ce_fwd(xm, y)[0]) / (2 * h)
            assert abs(num - g[t, v]) < 1e-3


def test_layernorm_stats_and_grad(rng):
    R, C = 5, 16
    x = rng.standard_normal((R, C)).astype(np.float32) * 3 + 1
    gamma = np.ones(C, np.float32)
    beta = np.zeros(C, np.float32)
    y = oracle.layernorm_fwd(x, gamma, beta)
    np.testing.assert_allclose(y.mean(1), 0, atol=1e-5)
    np.testing.assert_allclose(y.var(1), 1, atol=1e-3)
    go = rng.standard_normal((R, C)).astype(np.float32)
    gamma = rng.standard_normal(C).astype(np.float32)
    beta = rng.standard_normal(C).astype(np.float32)
    gx, gg, gb = oracle.layernorm_bwd(x, gamma, go)
    # float64 closed form
    xd = x.astype(np.float64)
    mu = xd.mean(1, keepdims=True)
    var = ((xd - mu) ** 2).mean(1, keepdims=True)
    xh = (xd - mu) / np.sqrt(var + 1e-5)
    dxh = go * gamma
    gx_ref = (dxh - dxh.mean(1, keepdims=True) - xh * (dxh * xh).mean(1, keepdims=True)) / np.sqrt(var + 1e-5)
    assert relerr(gx, gx_ref) < 1e-5
    assert relerr(gg, (go * xh).sum(0)) < 1e-5
    assert relerr(gb, go.sum(0)) < 1e-6


def test_bias_known_answer():
    """Row-broadcast add values and bias grad = row count
    (reference test/core/tensor/gpu_tensor_test.dart:522-576)."""
    a = np.arange(6, dtype=np.float32).reshape(3, 2)
    b = np.array([10, 20], np.float32)
    np.testing.assert_array_equal(oracle.bias_fwd(a, b), a + b)
    ga, gb = oracle.bias_bwd(np.ones((3, 2), np.float32))
    np.testing.assert_array_equal(gb, [3, 3])
    np.testing.assert_array_equal(ga, np.ones((3, 2)))


def test_adam_matches_formula(rng):
    n = 10
    p = rng.standard_normal(n).astype(np.float32)
    g = rng.standard_normal(n).astype(np.float32)
    m = np.zeros(n, np.float32); v = np.zeros(n, np.float32)
    p0 = p.copy()
    oracle.adam(p, g, m, v, t=1, lr=3e-4)
    step = 2.0
    mr = 0.1 * g.astype(np.float64); vr = 0.001 * g.astype(np.float64) ** 2
    upd = 3e-4 * (mr / (1 - 0.9 ** step)) / (np.sqrt(vr / (1 - 0.999 ** step)) + 1e-8)
    np.testing.assert_allclose(p, p0 - upd - 3e-4 * 0.001 * p0, rtol=1e-5, atol=1e-7)
