"""CPU stand-in for fpscan_b200.distributed.CudaOps, for gloo tests of the
sequence-sharded exchange logic.  float64 numpy loops with the semantics the
C ABI documents for each shard entry point (include/fpscan_b200.h).  Test
helper only."""
from __future__ import annotations

import numpy as np
import torch

import oracle


def _np(t):
    return t.detach().double().cpu().numpy()


def _t(a, like):
    return torch.from_numpy(np.ascontiguousarray(a)).to(like.dtype)


def _scan_init(g, x, init):
    y = np.empty_like(x)
    acc = init.reshape(x.shape[:-1]).copy()
    for t in range(x.shape[-1]):
        acc = g[..., t] * acc + x[..., t]
        y[..., t] = acc
    return y


def _bwd(g, y, go, addend, y_prev):
    L = go.shape[-1]
    dt = np.empty_like(go)
    acc = addend.reshape(go.shape[:-1]).copy()
    for t in range(L - 1, -1, -1):
        gs = 1.0 if t == L - 1 else g[..., t + 1]
        acc = gs * acc + go[..., t]
        dt[..., t] = acc
    yp = np.concatenate([y_prev.reshape(go.shape[:-1] + (1,)), y[..., :-1]], axis=-1)
    return yp * dt, dt


class CpuOps:
    def fwd_reduce(self, gates, tokens):
        g, x = _np(gates), _np(tokens)
        y = oracle.scan_f64(g, x)
        rows = x.size // x.shape[-1]
        a = np.prod(g, axis=-1).reshape(rows)
        return torch.from_numpy(np.stack([a, y[..., -1].reshape(rows)])).float()

    def fwd_scan(self, gates, tokens, y_init):
        return _t(_scan_init(_np(gates), _np(tokens), _np(y_init)), tokens)

    def fwd_scan_zero(self, gates, tokens):
        return _t(oracle.scan_f64(_np(gates), _np(tokens)), tokens)

    def bwd_reduce(self, gates, grad_out):
        g, go = _np(gates), _np(grad_out)
        rows = go.size // go.shape[-1]
        _, dt = _bwd(g, np.zeros_like(go), go, np.zeros(rows), np.zeros(rows))
        return torch.from_numpy((g[..., 0] * dt[..., 0]).reshape(rows)).float()

    def bwd_scan(self, gates, y, grad_out, addend, y_prev):
        dg, dt = _bwd(_np(gates), _np(y), _np(grad_out), _np(addend), _np(y_prev))
        return _t(dg, grad_out), _t(dt, grad_out)

    def bwd_scan_zero(self, gates, y, grad_out):
        dg, dt = oracle.scan_bwd_f64(_np(gates), _np(y), _np(grad_out))
        return _t(dg, grad_out), _t(dt, grad_out)

    def combine(self, gathered, world, rank, reverse):
        G = _np(gathered)
        rows = G.shape[-1]
        v = np.zeros(rows)
        qs = range(rank) if not reverse else range(world - 1, rank, -1)
        first = True
        for q in qs:
            v = G[q, 1] if first else G[q, 0] * v + G[q, 1]
            first = False
        return torch.from_numpy(np.asarray(v, dtype=np.float64)).float()
