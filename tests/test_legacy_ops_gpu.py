"""The non-AFT ops of the reference handle ABI (kept for drop-in loading)
against float64 numpy on the same inputs.  Forward and backward, with the
reference's accumulate-into-grad semantics."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
FP = ctypes.POINTER(ctypes.c_float)


@pytest.fixture(scope="module")
def L():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from dart_cuda_b200 import lib

    lib_ = lib()
    VP = ctypes.c_void_p
    for n in ("sub_tensors", "div_tensors", "add_tensor_scalar", "sub_tensor_scalar", "mul_tensor_scalar",
              "div_tensor_scalar", "matmul_tensors"):
        getattr(lib_, n).restype = VP
        getattr(lib_, n).argtypes = [VP, VP]
    for n in ("relu_tensor", "gelu_tensor", "tanh_tensor", "sigmoid_tensor", "log_tensor", "abs_tensor",
              "softmax_forward", "transpose_tensor"):
        getattr(lib_, n).restype = VP
        getattr(lib_, n).argtypes = [VP]
    lib_.pow_tensor.restype = VP
    lib_.pow_tensor.argtypes = [VP, ctypes.c_float]
    lib_.concat_tensors_gpu.restype = VP
    lib_.concat_tensors_gpu.argtypes = [ctypes.POINTER(VP), ctypes.c_int]
    lib_.concat_tensors_axis0_gpu.restype = VP
    lib_.concat_tensors_axis0_gpu.argtypes = [ctypes.POINTER(VP), ctypes.c_int]
    lib_.embedding_forward.restype = VP
    lib_.embedding_forward.argtypes = [ctypes.POINTER(ctypes.c_int32), VP, VP, ctypes.c_int, ctypes.c_int]
    lib_.slice_tensor.restype = VP
    lib_.slice_tensor.argtypes = [VP, ctypes.c_int, ctypes.c_int]
    lib_.layer_norm_tensor.restype = VP
    lib_.layer_norm_tensor.argtypes = [VP, ctypes.c_float]
    return lib_


def mk(L, a):
    a = np.ascontiguousarray(a, np.float32)
    return L.create_tensor(a.shape[0], int(np.prod(a.shape[1:])) if a.ndim > 1 else 1, a.ctypes.data_as(FP))


def get(L, h, shape, grad=False):
    out = np.empty(shape, np.float32)
    (L.get_tensor_grad if grad else L.get_tensor_data)(h, out.ctypes.data_as(FP))
    return out


def backprop(L, h, shape, g):
    """Run backward of L = sum(out * g)."""
    hg = mk(L, g)
    prod = L.mul_tensors(h, hg)
    s = L.sum_tensor(prod)
    L.backward(s)
    return [hg, prod, s]


def close(a, b, tol=1e-5):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    assert np.max(np.abs(a - b)) <= tol * max(1.0, np.max(np.abs(b))), (np.max(np.abs(a - b)), np.max(np.abs(b)))


def test_matmul(L):
    rng = np.random.default_rng(0)
    A = rng.standard_normal((37, 50)).astype(np.float32)
    B = rng.standard_normal((50, 29)).astype(np.float32)
    G = rng.standard_normal((37, 29)).astype(np.float32)
    ha, hb = mk(L, A), mk(L, B)
    hc = L.matmul_tensors(ha, hb)
    close(get(L, hc, (37, 29)), A.astype(np.float64) @ B, 1e-5)
    backprop(L, hc, (37, 29), G)
    close(get(L, ha, A.shape, True), G.astype(np.float64) @ B.T, 1e-5)
    close(get(L, hb, B.shape, True), A.T.astype(np.float64) @ G, 1e-5)


@pytest.mark.parametrize("name,f,df", [
    ("relu_tensor", lambda x: np.maximum(x, 0), lambda x: (x > 0).astype(float)),
    ("tanh_tensor", np.tanh, lambda x: 1 - np.tanh(x) ** 2),
    ("sigmoid_tensor", lambda x: 1 / (1 + np.exp(-x)), lambda x: np.exp(-x) / (1 + np.exp(-x)) ** 2),
    ("abs_tensor", np.abs, np.sign),
    ("gelu_tensor", lambda x: 0.5 * x * (1 + np.tanh(0.7978845608 * (x + 0.044715 * x ** 3))), None),
])
def test_unary(L, name, f, df):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((9, 33)).astype(np.float32)
    g = rng.standard_normal((9, 33)).astype(np.float32)
    hx = mk(L, x)
    hy = getattr(L, name)(hx)
    close(get(L, hy, x.shape), f(x.astype(np.float64)), 1e-5)
    backprop(L, hy, x.shape, g)
    if df is None:  # numeric derivative in float64
        h = 1e-6
        xd = x.astype(np.float64)
        df_ = lambda z: (f(z + h) - f(z - h)) / (2 * h)  # noqa: E731
        close(get(L, hx, x.shape, True), g * df_(xd), 1e-4)
    else:
        close(get(L, hx, x.shape, True), g * df(x.astype(np.float64)), 1e-5)


def test_binary_scalar_pow_log(L):
    rng = np.random.default_rng(2)
    a = rng.standard_normal((6, 10)).astype(np.float32)
    b = (rng.random((6, 10)) + 0.5).astype(np.float32)
    s = np.array([[1.7]], np.float32)
    ha, hb, hs = mk(L, a), mk(L, b), mk(L, s)
    close(get(L, L.sub_tensors(ha, hb), a.shape), a - b)
    close(get(L, L.div_tensors(ha, hb), a.shape), a / b)
    close(get(L, L.mul_tensor_scalar(ha, hs), a.shape), a * 1.7)
    close(get(L, L.div_tensor_scalar(ha, hs), a.shape), a / 1.7)
    close(get(L, L.add_tensor_scalar(ha, hs), a.shape), a + 1.7)
    close(get(L, L.sub_tensor_scalar(ha, hs), a.shape), a - 1.7)
    close(get(L, L.pow_tensor(hb, 3.0), b.shape), b.astype(np.float64) ** 3)
    close(get(L, L.log_tensor(hb), b.shape), np.log(b.astype(np.float64) + 1e-7))
    hm = L.mul_tensor_scalar(ha, hs)
    g = rng.standard_normal(a.shape).astype(np.float32)
    backprop(L, hm, a.shape, g)
    close(get(L, hs, (1, 1), True)[0, 0], float((g.astype(np.float64) * a).sum()), 1e-5)


def test_softmax_transpose_concat_slice_embed(L):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5, 12)).astype(np.float32)
    hx = mk(L, x)
    sm = np.exp(x - x.max(1, keepdims=True))
    sm = sm / (sm.sum(1, keepdims=True) + 1e-9)
    close(get(L, L.softmax_forward(hx), x.shape), sm)
    close(get(L, L.transpose_tensor(hx), (12, 5)), x.T)
    z = rng.standard_normal((5, 12)).astype(np.float32)
    hz = mk(L, z)
    arr = (ctypes.c_void_p * 2)(hx, hz)
    hc = L.concat_tensors_gpu(ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p)), 2)
    close(get(L, hc, (5, 24)), np.concatenate([x, z], 1))
    g = rng.standard_normal((5, 24)).astype(np.float32)
    backprop(L, hc, (5, 24), g)
    close(get(L, hz, z.shape, True), g[:, 12:])
    h0 = L.concat_tensors_axis0_gpu(ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p)), 2)
    close(get(L, h0, (10, 12)), np.concatenate([x, z], 0))
    close(get(L, L.slice_tensor(hz, 1, 3), (3, 12)), z[1:4])
    wte = rng.standard_normal((65, 8)).astype(np.float32)
    wpe = rng.standard_normal((6, 8)).astype(np.float32)
    idx = np.array([3, 64, 0, 3, 5, 7], np.int32)
    he = L.embedding_forward(idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), mk(L, wte), mk(L, wpe), 6, 8)
    close(get(L, he, (6, 8)), wte[idx] + wpe)


def test_layer_norm_nonaffine(L):
    rng = np.random.default_rng(4)
    x = (3 * rng.standard_normal((4, 20)) + 1).astype(np.float32)
    hy = L.layer_norm_tensor(mk(L, x), 1e-5)
    xd = x.astype(np.float64)
    ref = (xd - xd.mean(1, keepdims=True)) / np.sqrt(xd.var(1, keepdims=True) + 1e-5)
    close(get(L, hy, x.shape), ref, 1e-5)
