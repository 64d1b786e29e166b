"""Generate tests/golden/*.npz from the REFERENCE's own Python code.

Run with the path of a checkout of the reference:
    python tests/golden/make_golden.py <reference checkout>
It imports the reference's eval/baselines.py (sequential_scan,
parallel_scan_torch) by path and evaluates, in float64 on the CPU:

* forward and reverse scans (sequential_scan, eval/baselines.py:20-37),
* the Hillis-Steele baseline (parallel_scan_torch, eval/baselines.py:40-61),
* gradients by autograd through sequential_scan, exactly as the reference's
  test_backward_matches_oracle does (tests/test_fpscan.py:69-87).

Inputs follow the reference tests' distribution (tests/test_fpscan.py:25-29):
gates = 0.99 + 0.01*U[0,1), tokens = N(0,1)/seqlen, drawn in fp32 from a
seeded CPU torch.Generator and rounded to the case's dtype; the float64
oracle consumes the rounded values (as tests/test_fpscan.py:48 does).
The reference's extension is not needed: only its pure-Python baselines run.
"""
from __future__ import annotations

import importlib.util
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
B, D = 2, 2


def _load_baselines(ref_root: str):
    path = os.path.join(ref_root, "eval", "baselines.py")
    spec = importlib.util.spec_from_file_location("ref_eval_baselines", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _inputs(seqlen: int, dtype: torch.dtype, seed: int):
    gen = torch.Generator().manual_seed(seed)
    gates = 0.99 + 0.01 * torch.rand(B, D, seqlen, generator=gen)
    tokens = torch.randn(B, D, seqlen, generator=gen) / seqlen
    return gates.to(dtype), tokens.to(dtype)


def main(ref_root: str) -> None:
    bl = _load_baselines(ref_root)
    seq, par = bl.sequential_scan, bl.parallel_scan_torch
    cases = {}
    meta = []

    def put(name, dtype, **arrays):
        meta.append({"name": name, "dtype": str(dtype).replace("torch.", "")})
        for k, v in arrays.items():
            # inputs keep their (rounded) values in float32; results in float64
            as_input = k in ("gates", "tokens", "grad_out")
            cases[f"{name}/{k}"] = v.detach().to(torch.float32 if as_input else torch.float64).numpy()

    # forward + reverse, fp32, every seqlen the fixtures can afford
    for L in [32, 64, 128, 256, 512, 1024]:
        g, x = _inputs(L, torch.float32, seed=L)
        put(f"fwd_float32_L{L}", torch.float32, gates=g, tokens=x,
            y=seq(g.double(), x.double()), y_rev=seq(g.double(), x.double(), reverse=True),
            y_hs=par(g.double(), x.double()))
    g, x = _inputs(4096, torch.float32, seed=4096)
    put("fwd_float32_L4096", torch.float32, gates=g, tokens=x, y=seq(g.double(), x.double()))
    # half types: rounded inputs, float64 oracle
    for dt in (torch.float16, torch.bfloat16):
        for L in [32, 256, 1024]:
            g, x = _inputs(L, dt, seed=L + 7)
            put(f"fwd_{str(dt).replace('torch.', '')}_L{L}", dt, gates=g, tokens=x,
                y=seq(g.double(), x.double()), y_rev=seq(g.double(), x.double(), reverse=True))
    # backward by autograd through the serial loop (tests/test_fpscan.py:69-87)
    for dt, Ls in ((torch.float32, [32, 128, 512, 1024]), (torch.float16, [256]),
                   (torch.bfloat16, [256])):
        for L in Ls:
            g, x = _inputs(L, dt, seed=L + 3)
            gen = torch.Generator().manual_seed(L + 4)
            w = torch.randn(B, D, L, generator=gen).to(dt)
            g64 = g.double().clone().requires_grad_()
            x64 = x.double().clone().requires_grad_()
            y64 = seq(g64, x64)
            (y64 * w.double()).sum().backward()
            put(f"bwd_{str(dt).replace('torch.', '')}_L{L}", dt, gates=g, tokens=x, grad_out=w,
                y=y64.detach(), dgates=g64.grad, dtokens=x64.grad)

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **cases)
    with open(os.path.join(HERE, "golden_meta.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py",
                   "source": "reference eval/baselines.py (sequential_scan, parallel_scan_torch)",
                   "torch": torch.__version__, "batch": B, "dim": D, "cases": meta}, f, indent=1)
    print(f"wrote {len(meta)} cases")


if __name__ == "__main__":
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from oracle.build_ref import reference_root

    root = sys.argv[1] if len(sys.argv) > 1 else reference_root()
    if root is None:
        sys.exit("reference checkout not found: pass it as the argument or set "
                 "FPSCAN_REFERENCE_ROOT")
    main(root)
