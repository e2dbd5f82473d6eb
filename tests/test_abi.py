"""The C ABI library loads and exports every symbol include/*.h declares.
CPU only: nothing here calls into CUDA."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_functions():
    names = []
    for h in HEADERS:
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        text = re.sub(r"#[^\n]*", "", text)
        for m in re.finditer(r"([A-Za-z_][A-Za-z0-9_]*)\s*\([^;{]*\)\s*;", text):
            names.append(m.group(1))
    return sorted(set(names))


def test_headers_declare_entry_points():
    names = declared_functions()
    assert "dc_aft_fwd" in names and "aft_forward" in names and len(names) > 20


def test_library_exports_every_declared_symbol():
    from dart_cuda_b200 import _lib

    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_matches_header():
    from dart_cuda_b200 import _lib

    assert set(_lib.SIGNATURES) <= set(declared_functions())
    _lib.lib()  # binds every signature; raises on a missing symbol


def test_library_is_sm100a_only():
    """The build passes exactly one -gencode, for sm_100a."""
    from dart_cuda_b200 import build

    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


# Every symbol the reference's loaders bind eagerly
# (python/dart_cuda/core/tensor/cuda_engine.py:99-199,
#  lib/core/tensor/cuda_engine.dart:320-420): a missing one fails their import.
REFERENCE_UNION = """
create_tensor destroy_tensor get_tensor_data get_tensor_grad tensor_to_host set_tensor_data
backward zero_grad tensor_step clip_gradients add_tensors sub_tensors mul_tensors div_tensors
add_tensor_scalar sub_tensor_scalar mul_tensor_scalar div_tensor_scalar add_tensor_row_broadcast
matmul_tensors pow_tensor relu_tensor gelu_tensor tanh_tensor sigmoid_tensor log_tensor abs_tensor
softmax_forward transpose_tensor sum_tensor mean_tensor aft_forward aft_cross_forward
concat_tensors_gpu concat_tensors_axis0_gpu layernorm_forward embedding_forward cross_entropy_loss
adam_step sdg_step slice_tensor tensor_xavier_init tensor_zero_init layer_norm_tensor
compute_cost_matrix im2col_cuda col2im_cuda
""".split()


def test_exports_reference_symbol_union():
    from dart_cuda_b200 import _lib

    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    assert len(REFERENCE_UNION) == 47
    missing = [n for n in REFERENCE_UNION if not hasattr(lib, n)]
    assert not missing, missing
    assert set(REFERENCE_UNION) <= set(declared_functions())


def test_split_backward_flags_are_validated_on_the_host():
    """The two-part backward's flag rules are checked before any CUDA call,
    so misuse fails the same way on a machine without a GPU."""
    from dart_cuda_b200 import _lib

    lib = _lib.lib()
    fake = 0x1000  # never dereferenced: validation returns first
    base = _lib.DC_AFT_CAUSAL

    def bwd(flags, dQ=fake, dK=fake, dV=fake, dW=fake):
        return lib.dc_aft_bwd(fake, fake, fake, fake, 128, fake, dQ, dK, dV, dW, 1, 128, 128, 64,
                              _lib.DC_BF16, flags, None, 0, None)

    both = base | _lib.DC_AFT_BWD_NO_DKDV | _lib.DC_AFT_BWD_DKDV | _lib.DC_AFT_WS_VALID
    assert bwd(both) == _lib.DC_ERR_INVALID
    assert b"together" in lib.dc_last_error()
    assert bwd(base | _lib.DC_AFT_BWD_DKDV) == _lib.DC_ERR_INVALID  # needs the first part's workspace
    assert b"WS_VALID" in lib.dc_last_error()
    dkdv = base | _lib.DC_AFT_BWD_DKDV | _lib.DC_AFT_WS_VALID
    assert bwd(dkdv, dK=None) == _lib.DC_ERR_INVALID
    assert bwd(base | _lib.DC_AFT_BWD_NO_DKDV, dW=None) == _lib.DC_ERR_INVALID
    assert _lib.DC_AFT_SPARE_SMS(48) == 48 << 16 and _lib.DC_AFT_SPARE_SMS(300) == (300 & 0xFF) << 16


def test_packed_dw_size():
    """Block-packed causal dW: rows in blocks of 256, block k holding
    min(Tk rounded up to 8, 256 (k+1)) columns per row."""
    import ctypes

    from dart_cuda_b200 import lib

    def expect(T):
        tk8 = (T + 7) // 8 * 8
        return sum(min(tk8, 256 * (t // 256 + 1)) for t in range(T))

    for T in (0, 1, 7, 256, 257, 300, 1024, 1100, 4096):
        n = ctypes.c_size_t(0)
        assert lib().dc_aft_dw_packed_size(T, T, ctypes.byref(n)) == 0
        assert n.value == expect(T), T
    n = ctypes.c_size_t(0)
    lib().dc_aft_dw_packed_size(4096, 4096, ctypes.byref(n))
    assert abs(n.value / 4096 ** 2 - 0.53) < 0.005
