"""Pin the CPU oracle to the reference itself.

The fixtures under tests/golden/ were produced by running the reference engine
(native/src/engine.cu compiled from its own sources) on a B200 through its own
C ABI — see tests/golden/make_golden.py.  Here the fp32 C restatement in
oracle/ must reproduce them on the same inputs.  CPU only.

Tolerance: the reference runs CUDA's expf and atomicAdd (nondeterministic
summation order), the oracle glibc expf and a fixed order, so agreement is to
fp32 rounding, not bitwise: normwise relative error below 1e-5.
"""
from pathlib import Path

import numpy as np
import pytest

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"


def relerr(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = max(np.max(np.abs(ref)), 1e-30)
    return float(np.max(np.abs(got - ref)) / scale)


def load(name):
    path = GOLDEN / f"{name}.npz"
    assert path.exists(), f"missing golden fixture {path}"
    return dict(np.load(path))


AFT_FULL = sorted(p.stem for p in GOLDEN.glob("aft_full_*.npz"))


def test_fixtures_present():
    assert len(AFT_FULL) >= 5
    for stem in ("aft_cross_t9_te5_d12", "layernorm_r64_c256", "bias_m64_n96", "ce_t64_v65"):
        assert (GOLDEN / f"{stem}.npz").exists()


@pytest.mark.parametrize("name", AFT_FULL)
def test_aft_full_oracle_matches_reference(name):
    g = load(name)
    masked = bool(g["masked"])
    Z = oracle.aft_full_fwd(g["Q"], g["K"], g["V"], g["W"], masked)
    assert relerr(Z, g["Z"]) < 1e-5
    dQ, dK, dV, dW = oracle.aft_full_bwd(g["Q"], g["K"], g["V"], g["W"], g["dZ"], masked)
    for got, key in ((dQ, "dQ"), (dK, "dK"), (dV, "dV"), (dW, "dW")):
        assert relerr(got, g[key]) < 1e-5, key


@pytest.mark.parametrize("name", sorted(p.stem for p in GOLDEN.glob("aft_cross_*.npz")))
def test_aft_cross_oracle_matches_reference(name):
    g = load(name)
    assert relerr(oracle.aft_cross_fwd(g["Q"], g["K"], g["V"], g["W"]), g["Z"]) < 1e-5
    for got, key in zip(oracle.aft_cross_bwd(g["Q"], g["K"], g["V"], g["W"], g["dZ"]), ("dQ", "dK", "dV", "dW")):
        assert relerr(got, g[key]) < 1e-5, key


@pytest.mark.parametrize("name", ["layernorm_r64_c256", "layernorm_r3_c7"])
def test_layernorm_oracle_matches_reference(name):
    g = load(name)
    gamma, beta = g["gamma"][0], g["beta"][0]
    assert relerr(oracle.layernorm_fwd(g["x"], gamma, beta), g["y"]) < 1e-5
    dx, dg, db = oracle.layernorm_bwd(g["x"], gamma, g["dy"])
    assert relerr(dx, g["dx"]) < 1e-5
    assert relerr(dg, g["dgamma"][0]) < 1e-5
    assert relerr(db, g["dbeta"][0]) < 1e-5


@pytest.mark.parametrize("name", ["bias_m64_n96", "bias_m5_n3"])
def test_bias_oracle_matches_reference(name):
    g = load(name)
    assert np.array_equal(oracle.bias_fwd(g["a"], g["b"][0]), g["y"])
    da, db = oracle.bias_bwd(g["dy"])
    assert np.array_equal(da, g["da"])
    assert relerr(db, g["db"][0]) < 1e-6


@pytest.mark.parametrize("name", ["ce_t64_v65", "ce_t4_v8192"])
def test_ce_oracle_matches_reference(name):
    g = load(name)
    loss, _ = oracle.ce_fwd(g["logits"], g["targets"])
    assert abs(loss - float(g["loss"][0, 0])) <= 1e-5 * abs(loss)
    assert relerr(oracle.ce_bwd(g["logits"], g["targets"]), g["dlogits"]) < 1e-5
