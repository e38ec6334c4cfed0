"""Test-only engine: the ``opendm_b200.engine`` interface computed by the CPU
oracle on CPU tensors. Used by the CPU tests to exercise the optimizer's host
logic (grouping, shard plans, state, collectives over gloo) without a GPU. The
product never uses it: ``MuonAdamW`` reaches it only through the private
``_engine`` argument that these tests pass."""

import numpy as np
import torch

from oracle import muon_oracle as O


def _np(t):
    return t.detach().float().cpu().numpy().copy()


def _dtype_name(t):
    return "bfloat16" if t.dtype == torch.bfloat16 else "float32"


class OracleEngine:
    def __init__(self, device_semantics="cpu"):
        self.sem = device_semantics
        self.calls = {"muon": 0, "momentum_only": 0, "direction": 0, "orthogonalize": 0, "adamw": 0}
        self.matrices_seen = 0

    def muon_matrices(self, items, *, momentum, nesterov, weight_decay_factor, ns_steps):
        self.calls["muon"] += 1
        self.matrices_seen += len(items)
        for it in items:
            g = None if it.grad is None else _np(it.grad)
            m, d = O.momentum_direction(g, _np(it.exp_avg), momentum, nesterov)
            it.exp_avg.copy_(torch.from_numpy(m))
            u = O.zeropower_via_newtonschulz5(d, steps=ns_steps)
            p = O.apply_update_factor(_np(it.param), u, wd_factor=weight_decay_factor, eff=it.eff,
                                      param_dtype=_dtype_name(it.param), device_semantics=self.sem)
            it.param.copy_(torch.from_numpy(p).to(it.param.dtype))

    def momentum_only(self, items, *, momentum, nesterov):
        self.calls["momentum_only"] += 1
        for it in items:
            g = None if it.grad is None else _np(it.grad)
            m, _ = O.momentum_direction(g, _np(it.exp_avg), momentum, nesterov)
            it.exp_avg.copy_(torch.from_numpy(m))

    def direction(self, grad, exp_avg, *, momentum, nesterov):
        self.calls["direction"] += 1
        g = None if grad is None else _np(grad)
        m, d = O.momentum_direction(g, _np(exp_avg), momentum, nesterov)
        exp_avg.copy_(torch.from_numpy(m))
        return torch.from_numpy(d)

    def directions_into(self, items, out, offsets, *, momentum, nesterov):
        self.calls["direction"] += len(items)
        for (grad, exp_avg), off in zip(items, offsets):
            g = None if grad is None else _np(grad).reshape(-1)
            m, d = O.momentum_direction(g, _np(exp_avg).reshape(-1), momentum, nesterov)
            exp_avg.copy_(torch.from_numpy(m).view_as(exp_avg))
            out[off:off + d.size].copy_(torch.from_numpy(d))

    def orthogonalize_many(self, mats, out_dtypes, steps=5, eps=1e-7):
        self.calls["orthogonalize"] += len(mats)
        self.matrices_seen += len(mats)
        return [torch.from_numpy(O.zeropower_via_newtonschulz5(_np(m), steps=steps, eps=eps)).to(dt)
                for m, dt in zip(mats, out_dtypes)]

    def apply_update_flat(self, items, wd_factor):
        for param, u, eff in items:
            p = O.apply_update_factor(_np(param), _np(u), wd_factor=wd_factor, eff=eff,
                                      param_dtype=_dtype_name(param), device_semantics=self.sem)
            param.copy_(torch.from_numpy(p).to(param.dtype))

    def orthogonalize(self, matrix, steps=5, eps=1e-7):
        self.calls["orthogonalize"] += 1
        return torch.from_numpy(O.zeropower_via_newtonschulz5(_np(matrix), steps=steps, eps=eps))

    def adamw(self, items, *, lr, beta1, beta2, eps, weight_decay):
        self.calls["adamw"] += 1
        for it in items:
            p, m, v, _ = O.adamw_step(_np(it.param), _np(it.grad), _np(it.exp_avg), _np(it.exp_avg_sq),
                                      it.step - 1.0, lr=lr, beta1=beta1, beta2=beta2, eps=eps,
                                      weight_decay=weight_decay, param_dtype=_dtype_name(it.param))
            it.param.copy_(torch.from_numpy(p).to(it.param.dtype))
            it.exp_avg.copy_(torch.from_numpy(m))
            it.exp_avg_sq.copy_(torch.from_numpy(v))

    def check_errors(self, block=False):
        pass
