"""Pin the CPU oracle to the reference's own outputs (tests/golden/, made by
tests/golden/make_golden.py from the reference's eval/baselines.py)."""
import json
import os

import numpy as np
import pytest
import torch

import oracle

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = np.load(os.path.join(HERE, "golden", "golden.npz"))
META = json.load(open(os.path.join(HERE, "golden", "golden_meta.json")))
NAMES = [c["name"] for c in META["cases"]]
FWD = [n for n in NAMES if n.startswith("fwd_")]
BWD = [n for n in NAMES if n.startswith("bwd_")]


def g(name, key):
    return GOLD[f"{name}/{key}"]


@pytest.mark.parametrize("name", FWD)
def test_c_oracle_forward_bit_exact(name):
    y = oracle.scan_f64(g(name, "gates"), g(name, "tokens"))
    np.testing.assert_array_equal(y, g(name, "y"))


@pytest.mark.parametrize("name", [n for n in FWD if f"{n}/y_rev" in GOLD.files])
def test_c_oracle_reverse_bit_exact(name):
    y = oracle.scan_f64(g(name, "gates"), g(name, "tokens"), reverse=True)
    np.testing.assert_array_equal(y, g(name, "y_rev"))


@pytest.mark.parametrize("name", FWD)
def test_numpy_oracle_forward_bit_exact(name):
    y = oracle.sequential_scan_np(g(name, "gates"), g(name, "tokens"))
    np.testing.assert_array_equal(y, g(name, "y"))


@pytest.mark.parametrize("name", [n for n in FWD if f"{n}/y_hs" in GOLD.files])
def test_hillis_steele_port_bit_exact(name):
    gt = torch.from_numpy(g(name, "gates")).double()
    xt = torch.from_numpy(g(name, "tokens")).double()
    y = oracle.parallel_scan_torch(gt, xt).numpy()
    np.testing.assert_array_equal(y, g(name, "y_hs"))


@pytest.mark.parametrize("name", BWD)
def test_c_oracle_backward_formula_matches_autograd(name):
    # The golden gradients are autograd through the serial loop; the oracle
    # evaluates the PScan.backward formula.  Both are float64: they agree to
    # rounding, not bit-for-bit (different summation order).
    y = oracle.scan_f64(g(name, "gates"), g(name, "tokens"))
    np.testing.assert_array_equal(y, g(name, "y"))
    dg, dt = oracle.scan_bwd_f64(g(name, "gates"), y, g(name, "grad_out"))
    assert oracle.normwise_error(dt, g(name, "dtokens")) < 1e-13
    assert oracle.normwise_error(dg, g(name, "dgates")) < 1e-13


def test_backward_formula_port_matches_c_oracle():
    name = BWD[0]
    gt = torch.from_numpy(g(name, "gates")).double()
    yt = torch.from_numpy(g(name, "y")).double()
    got = torch.from_numpy(g(name, "grad_out")).double()
    dg, dt = oracle.pscan_backward_formula(
        gt, yt, got, lambda a, b, rev: torch.from_numpy(oracle.scan_f64(a.numpy(), b.numpy(), rev)))
    dg_c, dt_c = oracle.scan_bwd_f64(gt.numpy(), yt.numpy(), got.numpy())
    np.testing.assert_array_equal(dt.numpy(), dt_c)
    np.testing.assert_array_equal(dg.numpy(), dg_c)


def test_fp32_baseline_close_to_f64():
    name = BWD[-1] if "float32" in BWD[-1] else [n for n in BWD if "float32" in n][-1]
    y, dg, dt = oracle.pscan_fwdbwd_f32(g(name, "gates"), g(name, "tokens"), g(name, "grad_out"))
    assert oracle.normwise_error(y, g(name, "y")) < 1e-5
    assert oracle.normwise_error(dt, g(name, "dtokens")) < 1e-5
    assert oracle.normwise_error(dg, g(name, "dgates")) < 1e-5
