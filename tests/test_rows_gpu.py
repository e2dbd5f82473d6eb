"""LayerNorm, row-broadcast bias, cross-entropy and AdamW on the GPU against the
CPU oracle (fp32 everywhere; tolerance 1e-5 normwise unless stated)."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")


@pytest.fixture(scope="module")
def ops():
    from dart_cuda_b200 import ops as _ops

    return _ops


def relerr(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30))


def T(dev, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.mark.parametrize("R,C", [(16384, 256), (64, 1024), (7, 3), (33, 1500), (5, 130)])
def test_layernorm(ops, dev, R, C):
    rng = np.random.default_rng(R + C)
    x = (2 * rng.standard_normal((R, C)) + 0.5).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    b = (0.1 * rng.standard_normal(C)).astype(np.float32)
    dy = rng.standard_normal((R, C)).astype(np.float32)
    y = ops.layernorm_fwd(T(dev, x), T(dev, g), T(dev, b))
    assert relerr(y.cpu().numpy(), oracle.layernorm_fwd(x, g, b)) < 1e-5
    dx, dg, db = ops.layernorm_bwd(T(dev, x), T(dev, g), T(dev, dy))
    rx, rg, rb = oracle.layernorm_bwd(x, g, dy)
    assert relerr(dx.cpu().numpy(), rx) < 1e-4
    assert relerr(dg.cpu().numpy(), rg) < 1e-4
    assert relerr(db.cpu().numpy(), rb) < 1e-5
    # accumulate semantics (the reference's += into x.grad, gamma.grad, beta.grad)
    grads = (dx.clone(), dg.clone(), db.clone())
    ops.layernorm_bwd(T(dev, x), T(dev, g), T(dev, dy), grads=grads, accumulate=True)
    torch.testing.assert_close(grads[0], 2 * dx, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(grads[2], 2 * db, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("M,N", [(16384, 1024), (64, 96), (5, 3), (1000, 65), (37, 260)])
def test_bias(ops, dev, M, N):
    rng = np.random.default_rng(M * N)
    a = rng.standard_normal((M, N)).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    dy = rng.standard_normal((M, N)).astype(np.float32)
    y = ops.bias_fwd(T(dev, a), T(dev, b))
    assert np.array_equal(y.cpu().numpy(), oracle.bias_fwd(a, b))
    da, db = ops.bias_bwd(T(dev, dy))
    ra, rb = oracle.bias_bwd(dy)
    assert np.array_equal(da.cpu().numpy(), ra)
    assert relerr(db.cpu().numpy(), rb) < 1e-5


@pytest.mark.parametrize("M,N", [(16384, 256), (3000, 768), (9, 160)])
def test_bias_grad_only(ops, dev, M, N):
    """db alone (no da), overwritten and then accumulated: the one-launch
    cluster reduction, deterministic from call to call."""
    rng = np.random.default_rng(M + N)
    dy = rng.standard_normal((M, N)).astype(np.float32)
    rb = oracle.bias_bwd(dy)[1]
    tdy = T(dev, dy)
    db = torch.full((N,), 3.0, device=dev)
    ops.bias_bwd(tdy, grads=(None, db))
    assert relerr(db.cpu().numpy(), rb) < 1e-5
    db2 = torch.zeros(N, device=dev)
    ops.bias_bwd(tdy, grads=(None, db2))
    assert torch.equal(db, db2)
    ops.bias_bwd(tdy, grads=(None, db), accumulate=True)
    assert relerr(db.cpu().numpy(), 2 * rb) < 1e-5


@pytest.mark.parametrize("M,N", [(262144, 256), (131072, 1024), (140001, 12)])
def test_bias_bwd_tall(ops, dev, M, N):
    """Tall matrices take the row-contiguous form: whole rows a CTA, then the
    last CTA adds the CTAs' partial column sums (several threads a column,
    in a fixed order: the same bits on every call)."""
    rng = np.random.default_rng(M + N)
    dy = rng.standard_normal((M, N)).astype(np.float32)
    rb = dy.astype(np.float64).sum(0)
    tdy = T(dev, dy)
    da, db = ops.bias_bwd(tdy)
    assert np.array_equal(da.cpu().numpy(), dy)
    assert relerr(db.cpu().numpy(), rb) < 1e-5
    db2 = torch.zeros(N, device=dev)
    ops.bias_bwd(tdy, grads=(None, db2))
    assert torch.equal(db, db2)
    ops.bias_bwd(tdy, grads=(None, db2), accumulate=True)
    assert relerr(db2.cpu().numpy(), 2 * rb) < 1e-5


@pytest.mark.parametrize("M,N,ld", [(16384, 256, 256), (300, 96, 100), (7, 6, 6)])
def test_gate(ops, dev, M, N, ld):
    """z = sigmoid(q) * v0 and its backward (dq, dv0 accumulated) against
    float64 on the host, row strides wider than N included."""
    from dart_cuda_b200._lib import lib

    rng = np.random.default_rng(M * N)
    q = rng.standard_normal((M, ld)).astype(np.float32)
    v0 = rng.standard_normal(N).astype(np.float32)
    dz = rng.standard_normal((M, ld)).astype(np.float32)
    tq, tv, tdz = T(dev, q), T(dev, v0), T(dev, dz)
    z = torch.zeros(M, ld, device=dev)
    dq = torch.zeros(M, ld, device=dev)
    dv = torch.ones(N, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    assert lib().dc_gate_fwd(tq.data_ptr(), ld, tv.data_ptr(), z.data_ptr(), ld, M, N, st) == 0
    assert lib().dc_gate_bwd(tq.data_ptr(), ld, tv.data_ptr(), tdz.data_ptr(), ld, dq.data_ptr(), ld,
                             dv.data_ptr(), M, N, st) == 0
    s = 1.0 / (1.0 + np.exp(-q[:, :N].astype(np.float64)))
    g = dz[:, :N].astype(np.float64)
    assert relerr(z[:, :N].cpu().numpy(), s * v0) < 1e-5
    assert relerr(dq[:, :N].cpu().numpy(), g * v0 * s * (1 - s)) < 1e-5
    assert relerr(dv.cpu().numpy(), 1.0 + (g * s).sum(0)) < 1e-5
    assert float(z[:, N:].abs().sum()) == 0.0 and float(dq[:, N:].abs().sum()) == 0.0


@pytest.mark.parametrize("Tn,V", [(16384, 65), (64, 8192), (4, 2), (3, 50257), (33, 2052), (17, 16384),
                                  (9, 1028)])
def test_cross_entropy(ops, dev, Tn, V):
    rng = np.random.default_rng(Tn + V)
    x = (2 * rng.standard_normal((Tn, V))).astype(np.float32)
    y = rng.integers(0, V, Tn).astype(np.int32)
    tx, ty = T(dev, x), T(dev, y)
    rows = torch.empty(Tn, device=dev)
    loss = ops.ce_fwd(tx, ty, row_loss=rows)
    rl, rrows = oracle.ce_fwd(x, y)
    assert abs(float(loss) - rl) / abs(rl) < 1e-5
    assert relerr(rows.cpu().numpy(), rrows) < 1e-5
    gs = torch.tensor([0.7], device=dev)
    g = ops.ce_bwd(tx, ty, grad_scale=gs)
    assert relerr(g.cpu().numpy(), oracle.ce_bwd(x, y, 0.7)) < 1e-5


def test_cross_entropy_known_answer(ops, dev):
    g = ops.ce_bwd(torch.zeros(1, 2, device=dev), torch.tensor([1], dtype=torch.int32, device=dev))
    np.testing.assert_allclose(g.cpu().numpy(), [[0.45, -0.45]], atol=1e-6)


def test_adam(ops, dev):
    rng = np.random.default_rng(3)
    n = 100003
    p = rng.standard_normal(n).astype(np.float32)
    g = rng.standard_normal(n).astype(np.float32)
    m = (0.1 * rng.standard_normal(n)).astype(np.float32)
    v = np.abs(0.1 * rng.standard_normal(n)).astype(np.float32)
    tp, tg, tm, tv = (T(dev, a.copy()) for a in (p, g, m, v))
    for step in range(3):
        ops.adam_step(tp, tg, tm, tv, step, 3e-4)
        oracle.adam(p, g, m, v, step, 3e-4)
    assert relerr(tp.cpu().numpy(), p) < 1e-6
    assert relerr(tm.cpu().numpy(), m) < 1e-6
    assert relerr(tv.cpu().numpy(), v) < 1e-6
