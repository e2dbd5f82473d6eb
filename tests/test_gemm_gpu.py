"""dc_gemm (tcgen05 dense layers) against float64 products on the host.

tf32 operands keep 10 mantissa bits, so fp32 inputs are checked normwise to
2e-3; bf16 inputs are exact in the MMA and only the fp32 accumulation order
differs (1e-5)."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from dart_cuda_b200 import ops as _ops
    return _ops


def rel(got, ref):
    got = got.double().cpu()
    return float((got - ref).norm() / max(ref.norm(), 1e-30))


def gelu64(x):
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608 * (x + 0.044715 * x ** 3)))


def gelu_d64(x):
    t = torch.tanh(0.7978845608 * (x + 0.044715 * x ** 3))
    return 0.5 * (1 + t) + 0.5 * x * (1 - t * t) * 0.7978845608 * (1 + 3 * 0.044715 * x * x)


def operands(M, N, K, ta, tb, dtype, seed=0):
    g = torch.Generator().manual_seed(seed)
    A = torch.randn((K, M) if ta else (M, K), generator=g)
    B = torch.randn((N, K) if tb else (K, N), generator=g)
    A64, B64 = A.to(dtype).double(), B.to(dtype).double()
    ref = (A64.T if ta else A64) @ (B64.T if tb else B64)
    return A.to(dtype).cuda(), B.to(dtype).cuda(), ref


TOL = {torch.float32: 2e-3, torch.bfloat16: 1e-5}


@pytest.mark.parametrize("ta,tb", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (300, 200, 72), (1000, 384, 256)])
def test_layouts(ops, ta, tb, dtype, M, N, K):
    if dtype == torch.bfloat16 and (M % 8 or N % 8 or K % 8):
        pytest.skip("bf16 rows must be 16-byte multiples")
    A, B, ref = operands(M, N, K, ta, tb, dtype)
    C = ops.gemm(A, B, trans_a=ta, trans_b=tb)
    torch.cuda.synchronize()
    assert rel(C, ref) < TOL[dtype]


@pytest.mark.parametrize("ta,tb", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("M,N,K", [(4736, 512, 256), (4700, 300, 72)])
def test_wide_tiles(ops, ta, tb, dtype, M, N, K):
    """Enough rows for 128 x 256 tiles (one N = 256 MMA a K slice): the
    K-major B operand in two 128-row boxes, the MN-major one in eight or
    four 128-byte blocks; N = 300 leaves a partly empty last tile."""
    if dtype == torch.bfloat16 and (M % 8 or N % 8 or K % 8):
        pytest.skip("bf16 rows must be 16-byte multiples")
    A, B, ref = operands(M, N, K, ta, tb, dtype, seed=5)
    C = ops.gemm(A, B, trans_a=ta, trans_b=tb)
    torch.cuda.synchronize()
    assert rel(C, ref) < TOL[dtype]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("M,N,K", [(256, 768, 8192), (200, 300, 8200)])
def test_long_k_split(ops, dtype, M, N, K):
    """Weight-gradient shapes (X^T dY over a long K): 128 x 256 tiles split
    along K, partial sums added by 16-byte atomics from the staged epilogue;
    M = 200 leaves half-empty row quadrants, N = 300 a ragged last tile."""
    if dtype == torch.bfloat16 and (M % 8 or N % 8 or K % 8):
        pytest.skip("bf16 rows must be 16-byte multiples")
    A, B, ref = operands(M, N, K, True, False, dtype, seed=9)
    C = ops.gemm(A, B, trans_a=True)
    torch.cuda.synchronize()
    assert rel(C, ref) < TOL[dtype] * (4 if dtype == torch.bfloat16 else 1)


def test_wide_tiles_fused_epilogues(ops):
    """Bias, GELU with the pre-activation kept, and a residual on 128 x 256
    tiles (the decoder's feed-forward shapes)."""
    M, N, K = 4736, 1024, 256
    A, B, ref = operands(M, N, K, False, False, torch.float32, seed=6)
    A, ref = A * 0.2, ref * 0.2
    bias = torch.randn(N).cuda()
    pre = torch.empty(M, N, device="cuda")
    H = ops.gemm(A, B, bias=bias, gelu=True, gelu_aux=pre)
    pre_ref = ref + bias.double().cpu()
    assert rel(pre, pre_ref) < TOL[torch.float32]
    assert rel(H, gelu64(pre_ref)) < TOL[torch.float32]
    W = torch.randn(N, 256).cuda() * 0.05
    R = torch.randn(M, 256).cuda()
    Y = ops.gemm(H, W, residual=R)
    yref = H.double().cpu() @ W.double().cpu() + R.double().cpu()
    assert rel(Y, yref) < TOL[torch.float32]


@pytest.mark.parametrize("M,N,K", [(64, 512, 512), (64, 2048, 512), (64, 512, 2048), (7, 65, 256)])
def test_skinny_split_k(ops, M, N, K):
    """Few output tiles: K is split across CTAs (bias once, residual kept)."""
    if N % 4:  # row stride padded to 16 bytes, as the LM head of a 65-token vocabulary
        Bfull = torch.randn(K, N + (4 - N % 4)).cuda()
        B = Bfull[:, :N]
        ref_B = B.double().cpu()
    else:
        B = torch.randn(K, N).cuda()
        ref_B = B.double().cpu()
    A = torch.randn(M, K).cuda()
    bias = torch.randn(N).cuda()
    R = torch.randn(M, N).cuda()
    C = ops.gemm(A, B, bias=bias, residual=R)
    ref = A.double().cpu() @ ref_B + bias.double().cpu() + R.double().cpu()
    assert rel(C, ref) < TOL[torch.float32]
    acc = R.clone()
    ops.gemm(A, B, out=acc, accumulate=True)
    assert rel(acc, A.double().cpu() @ ref_B + R.double().cpu()) < TOL[torch.float32]


@pytest.mark.parametrize("M,N,K", [(64, 2048, 512), (1, 100, 40), (3, 36, 1000)])
def test_skinny_gelu_alpha(ops, M, N, K):
    """Few rows (the decode step's layers): GELU with the pre-activation
    kept, a bias and alpha (K split over a cluster of CTAs where the tiles
    are few: the partial tiles are added before the GELU)."""
    A = torch.randn(M, K).cuda()
    B = torch.randn(K, N).cuda()
    bias = torch.randn(N).cuda()
    aux = torch.empty(M, N).cuda()
    C = ops.gemm(A, B, bias=bias, gelu=True, gelu_aux=aux, alpha=0.5)
    pre = 0.5 * (A.double().cpu() @ B.double().cpu()) + bias.double().cpu()
    assert rel(aux, pre) < TOL[torch.float32]
    assert rel(C, gelu64(pre)) < TOL[torch.float32]


def test_gelu_and_its_backward(ops):
    M, N, K = 512, 1024, 256
    A, B, ref = operands(M, N, K, False, False, torch.float32, seed=3)
    A = A * 0.2
    ref = ref * 0.2
    bias = torch.randn(N).cuda()
    pre = torch.empty(M, N, device="cuda")
    H = ops.gemm(A, B, bias=bias, gelu=True, gelu_aux=pre)
    pre_ref = ref + bias.double().cpu()
    assert rel(pre, pre_ref) < TOL[torch.float32]
    assert rel(H, gelu64(pre_ref)) < TOL[torch.float32]
    # backward of the following layer: dPre = (dY @ W^T) * gelu'(pre)
    dY = torch.randn(M, 384).cuda()
    W = torch.randn(N, 384).cuda()
    dP = ops.gemm(dY, W, trans_b=True, gelu_bwd_aux=pre)
    dref = (dY.double().cpu() @ W.double().cpu().T) * gelu_d64(pre.double().cpu())
    assert rel(dP, dref) < TOL[torch.float32]


def test_alpha_and_strided_views(ops):
    """Leading dimensions wider than the logical shape (column views)."""
    M, N, K = 200, 96, 128
    Abig = torch.randn(M, K + 32).cuda()
    Bbig = torch.randn(K, N + 64).cuda()
    Cbig = torch.zeros(M, N + 16, device="cuda")
    A, B, C = Abig[:, 8:8 + K], Bbig[:, 16:16 + N], Cbig[:, :N]
    ops.gemm(A, B, out=C, alpha=0.5)
    ref = 0.5 * (A.double().cpu() @ B.double().cpu())
    assert rel(C, ref) < TOL[torch.float32]
    assert torch.count_nonzero(Cbig[:, N:]) == 0


def test_rejects_unaligned(ops):
    A = torch.randn(64, 66).cuda()  # 264-byte rows: not a multiple of 16
    B = torch.randn(66, 64).cuda()
    with pytest.raises(ops.DcError):
        ops.gemm(A, B)
    assert ops.device_status() == 0


@pytest.mark.parametrize("M,N,K", [(64, 512, 512), (4736, 512, 256), (300, 200, 72), (1, 100, 40)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gate_epilogue(ops, M, N, K, dtype):
    """C = sigmoid(A B + bias) * v0 (the decoder's cross-attention query
    projection and gate in one launch): few tiles split K over a cluster,
    many run unsplit, through both epilogue forms; against dc_gate_fwd on the
    unfused product and against float64."""
    from dart_cuda_b200._lib import check, lib
    g = torch.Generator().manual_seed(M + N)
    if dtype == torch.bfloat16 and (K % 8 or N % 8):
        pytest.skip("bf16 rows must be 16-byte multiples")
    A = torch.randn(M, K, generator=g).to(dtype).cuda()
    B = (torch.randn(K, N, generator=g) / K ** 0.5).to(dtype).cuda()
    bias = torch.randn(N, generator=g).cuda()
    v0 = torch.randn(N, generator=g).cuda()
    Y = ops.gemm(A, B, bias=bias, gate=v0)
    Y2 = ops.gemm(A, B, bias=bias, gate=v0)
    q = ops.gemm(A, B, bias=bias)
    G = torch.empty_like(q)
    check(lib().dc_gate_fwd(q.data_ptr(), N, v0.data_ptr(), G.data_ptr(), N, M, N, ops._stream()),
          "dc_gate_fwd")
    torch.cuda.synchronize()
    pre = A.double().cpu() @ B.double().cpu() + bias.double().cpu()
    assert rel(Y, torch.sigmoid(pre) * v0.double().cpu()) < TOL[torch.float32]
    assert rel(Y, G.double().cpu()) < 1e-5
    assert torch.equal(Y, Y2)  # a cluster adds its partial tiles in a fixed order
    assert ops.device_status() == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("M,N,K", [(64, 2048, 512), (64, 512, 512), (128, 640, 1024), (3, 40, 1000)])
def test_cluster_split_k_gelu_residual(ops, M, N, K, dtype):
    """GELU with a separate residual and few tiles: K split over a cluster of
    CTAs whose partial tiles are added before the epilogue, the same bits on
    every run (tf32 and bf16 operands)."""
    g = torch.Generator().manual_seed(N + K)
    A = torch.randn(M, K, generator=g).to(dtype).cuda()
    B = (torch.randn(K, N, generator=g) / K ** 0.5).to(dtype).cuda()
    bias = torch.randn(N, generator=g).cuda()
    R = torch.randn(M, N, generator=g).cuda()
    aux = torch.empty(M, N, device="cuda")
    H = ops.gemm(A, B, bias=bias, residual=R, gelu=True, gelu_aux=aux)
    H2 = ops.gemm(A, B, bias=bias, residual=R, gelu=True)
    torch.cuda.synchronize()
    pre = A.double().cpu() @ B.double().cpu() + bias.double().cpu() + R.double().cpu()
    assert rel(aux, pre) < TOL[torch.float32]
    assert rel(H, gelu64(pre)) < TOL[torch.float32]
    assert torch.equal(H, H2)


def test_gate_rejects(ops):
    A = torch.randn(64, 64).cuda()
    B = torch.randn(64, 128).cuda()
    v0 = torch.randn(128).cuda()
    with pytest.raises(ops.DcError):
        ops.gemm(A, B, gelu=True, gelu_aux=torch.empty(64, 128, device="cuda"), gate=v0)
    from dart_cuda_b200._lib import lib
    C = torch.empty(64, 128, device="cuda")
    assert lib().dc_gemm_gate(A.data_ptr(), 64, B.data_ptr(), 128, C.data_ptr(), 128, 64, 128, 64, 0,
                              0x8, 1.0, None, None, 0, v0.data_ptr(), ops._stream()) != 0
    assert ops.device_status() == 0
