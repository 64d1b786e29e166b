"""The reference's own, unmodified ``fpscan/ops.py`` bound to this library.

The reference's public module loads its extension through
``importlib.import_module("fpscan._C")`` (fpscan/ops.py:14, 29-38).  With
this repository's ``fpscan`` package on the path, that name is
``fpscan/_C.py`` here, backed by libfpscan_b200.so.  These tests load the
reference's ops.py file as it is -- from the reference installed into
``baseline/_ref`` (which travels with the repository snapshot), else from the
reference checkout -- under a private module name, and run its
``scan_forward`` and ``PScan`` through this library.
"""
import importlib.util
import os
import sys

import numpy as np
import pytest
import torch

import oracle

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _reference_ops_path():
    cand = [os.path.join(REPO, "baseline", "_ref", "fpscan", "ops.py")]
    from oracle.build_ref import reference_root

    root = reference_root()
    if root:
        cand.append(os.path.join(root, "fpscan", "ops.py"))
    return next((p for p in cand if os.path.exists(p)), None)


def _load_reference_ops():
    path = _reference_ops_path()
    if path is None:
        pytest.skip("the reference's fpscan/ops.py is not available here")
    spec = importlib.util.spec_from_file_location("_reference_fpscan_ops", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_drop_in_names_resolve():
    import fpscan
    import fpscan._C
    import fpscan_b200

    assert fpscan.pscan is fpscan_b200.pscan
    assert fpscan.scan_forward is fpscan_b200.scan_forward
    assert fpscan.PScan is fpscan_b200.PScan
    assert callable(fpscan._C.fullscan_forward)
    assert os.path.dirname(os.path.abspath(fpscan.__file__)) == os.path.join(REPO, "fpscan")


def test_unmodified_reference_loader_binds_this_library():
    ref_ops = _load_reference_ops()
    ext = ref_ops._load_extension()
    assert ext is sys.modules["fpscan._C"]
    assert os.path.abspath(ext.__file__) == os.path.join(REPO, "fpscan", "_C.py")
    assert ext.fullscan_forward.__module__ == "fpscan_b200.ops"


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,L", [(torch.float32, 4096), (torch.float32, 65536),
                                     (torch.bfloat16, 2048), (torch.float16, 8192)])
def test_unmodified_reference_api_runs_on_this_library(dtype, L):
    ref_ops = _load_reference_ops()
    gen = torch.Generator(device="cuda").manual_seed(L)
    b, d = 2, 4
    g = (0.99 + 0.01 * torch.rand(b, d, L, generator=gen, device="cuda")).to(dtype)
    x = (torch.randn(b, d, L, generator=gen, device="cuda") / L).to(dtype)
    go = torch.randn(b, d, L, generator=gen, device="cuda").to(dtype)
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    g64, x64 = g.double().cpu().numpy(), x.double().cpu().numpy()
    for rev in (False, True):
        y64 = oracle.scan_f64(g64, x64, reverse=rev)
        y = ref_ops.scan_forward(g, x, reverse=rev)
        assert oracle.normwise_error(y.double().cpu().numpy(), y64) <= tol
        out = torch.full_like(x, float("nan"))
        ret = ref_ops.scan_forward(g, x, reverse=rev, out=out)
        assert ret is out
        assert torch.equal(out, y)
    gr = g.clone().requires_grad_()
    xr = x.clone().requires_grad_()
    y = ref_ops.pscan(gr, xr)
    dg, dx = torch.autograd.grad(y, (gr, xr), go)
    y64 = oracle.scan_f64(g64, x64)
    dg64, dx64 = oracle.scan_bwd_f64(g64, y64, go.double().cpu().numpy())
    assert oracle.normwise_error(y.detach().double().cpu().numpy(), y64) <= tol
    assert oracle.normwise_error(dx.double().cpu().numpy(), dx64) <= tol
    assert oracle.normwise_error(dg.double().cpu().numpy(), dg64) <= tol
