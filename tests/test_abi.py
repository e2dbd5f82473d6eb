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
