"""The reference's own Python front end (python/dart_cuda of the reference
project) loading this library as its engine.

The reference project is located through the environment variable
DART_CUDA_REF (its root directory); without it these tests skip.  Each test
runs the front end in a fresh interpreter with DART_CUDA_LIB pointing at
dart_cuda_b200/lib/libmat_mul.so, the way the front end's loader finds its
engine (python/dart_cuda/core/tensor/cuda_engine.py:30-61).

* Loading binds every symbol eagerly (cuda_engine.py:92-199), so importing
  the package proves the exported ABI is complete; no GPU is needed.
* Checkpoints written by AftDecoder.save are read by the front end's
  load_module_binary (python/dart_cuda/core/utils/persistence.py:20-59) into
  parameters of the reference's shapes, and files written by its
  save_module_binary are read by AftDecoder.load.  The front end's
  parameters here are stand-ins with the interface persistence.py uses
  (length, data, fetch_data), since real ones live in GPU memory.
* With a GPU, Tensor.aft(q, k, v, wb, True) and backward() run through this
  library on a golden fixture of the reference engine.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
LIB = ROOT / "dart_cuda_b200" / "lib" / "libmat_mul.so"
GOLDEN = ROOT / "tests" / "golden"


def _ref_python():
    root = os.environ.get("DART_CUDA_REF")
    if not root:
        pytest.skip("DART_CUDA_REF (the reference project's root) is not set")
    pkg = Path(root) / "python"
    if not (pkg / "dart_cuda" / "__init__.py").exists():
        pytest.skip(f"no python/dart_cuda under DART_CUDA_REF={root}")
    if not LIB.exists():
        pytest.skip("libmat_mul.so is not built")
    return pkg


def _run(script: str, tmp_path: Path, timeout=300):
    pkg = _ref_python()
    env = dict(os.environ, DART_CUDA_LIB=str(LIB), PYTHONPATH=str(pkg))
    f = tmp_path / "frontend_script.py"
    f.write_text(script)
    r = subprocess.run([sys.executable, str(f)], env=env, cwd=str(tmp_path), capture_output=True, text=True,
                       timeout=timeout)
    assert r.returncode == 0, f"front end script failed:\n{r.stdout}\n{r.stderr}"
    return r.stdout


def test_frontend_binds_this_library(tmp_path):
    out = _run("""
import ctypes, json
import dart_cuda
from dart_cuda.core.tensor import cuda_engine
e = dart_cuda.engine
bound = [n for n, v in vars(e).items() if isinstance(v, ctypes._CFuncPtr)]
e._lib.dc_version.restype = ctypes.c_char_p
print(json.dumps({"lib": e.lib_path, "bound": len(bound), "version": e._lib.dc_version().decode()}))
""", tmp_path)
    info = json.loads(out.strip().splitlines()[-1])
    assert Path(info["lib"]).resolve() == LIB.resolve()
    assert info["version"].startswith("dart_cuda_b200")
    # every binding of cuda_engine._bind_all succeeded
    src = (_ref_python() / "dart_cuda" / "core" / "tensor" / "cuda_engine.py").read_text()
    assert info["bound"] == src.count("self._b(")


def _decoder():
    from dart_cuda_b200.decoder import AftDecoder, DecoderConfig

    cfg = DecoderConfig(vocab=13, d_model=32, n_layers=2, n_heads=4, block_size=8)
    return AftDecoder(cfg, device="cpu", seed=5)


FAKE = """
import json, sys
import numpy as np
from dart_cuda.core.utils.persistence import load_module_binary, save_module_binary

class Param:  # the interface persistence.py uses of a front-end Tensor
    def __init__(self, shape):
        self.shape = shape
        self.length = int(np.prod(shape))
        self.data = [0.0] * self.length
    def fetch_data(self):
        return list(self.data)

class Module:
    def __init__(self, shapes):
        self.ps = [Param(s) for s in shapes]
    def parameters(self):
        return self.ps

shapes = json.load(open("shapes.json"))
"""


def test_checkpoint_read_by_frontend(tmp_path):
    m = _decoder()
    params = m.reference_parameters()
    (tmp_path / "shapes.json").write_text(json.dumps([list(v.shape) for _, v in params]))
    m.save(tmp_path / "ours.bin")
    _run(FAKE + """
mod = Module(shapes)
load_module_binary(mod, "ours.bin")
np.save("loaded.npy", np.concatenate([np.asarray(p.data, np.float32) for p in mod.parameters()]))
""", tmp_path)
    loaded = np.load(tmp_path / "loaded.npy")
    want = np.concatenate([v.detach().contiguous().view(-1).numpy() for _, v in params])
    assert np.array_equal(loaded, want)


def test_checkpoint_written_by_frontend(tmp_path):
    m = _decoder()
    params = m.reference_parameters()
    (tmp_path / "shapes.json").write_text(json.dumps([list(v.shape) for _, v in params]))
    _run(FAKE + """
mod = Module(shapes)
rng = np.random.default_rng(11)
for p in mod.parameters():
    p.data = [float(x) for x in rng.standard_normal(p.length).astype(np.float32)]
save_module_binary(mod, "theirs.bin")
np.save("written.npy", np.concatenate([np.asarray(p.data, np.float32) for p in mod.parameters()]))
""", tmp_path)
    m.load(tmp_path / "theirs.bin")
    got = np.concatenate([v.detach().contiguous().view(-1).numpy() for _, v in m.reference_parameters()])
    assert np.array_equal(got, np.load(tmp_path / "written.npy"))


@pytest.mark.gpu
def test_frontend_tensor_aft_on_gpu(tmp_path):
    """Tensor.aft(q, k, v, wb, True) + backward() of the front end, per
    sequence on a shared bias, against the reference engine's fixture."""
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    out = _run(f"""
import json
import numpy as np
from dart_cuda import Tensor
g = dict(np.load({str(GOLDEN / 'aft_full_b4_t64_d128_causal.npz')!r}))
B, T, D = g["Q"].shape
def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / np.abs(b).max())
wb = Tensor.from_list([T, T], g["W"].ravel().tolist())
errs = {{}}
for b in range(B):
    q, k, v = (Tensor.from_list([T, D], g[n][b].ravel().tolist()) for n in "QKV")
    z = Tensor.aft(q, k, v, wb, True)
    dz = Tensor.from_list([T, D], g["dZ"][b].ravel().tolist())
    (z * dz).sum().backward()
    errs[f"Z{{b}}"] = rel(np.array(z.data).reshape(T, D), g["Z"][b])
    for t, n in ((q, "dQ"), (k, "dK"), (v, "dV")):
        errs[f"{{n}}{{b}}"] = rel(np.array(t.grad).reshape(T, D), g[n][b])
errs["dW"] = rel(np.array(wb.grad).reshape(T, T), g["dW"])
print(json.dumps(errs))
""", tmp_path)
    errs = json.loads(out.strip().splitlines()[-1])
    bad = {k: v for k, v in errs.items() if not v < 1e-3}
    assert not bad, bad
