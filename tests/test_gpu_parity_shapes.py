"""GPU parity against the CPU oracle at every Muon shape class of the benchmark
configs 4 (~4B VLA: ViT, LM and action-expert matrices) and 5 (7B decoder,
gradients with 1% heavy-tail entries N(0, 1e-1) over an N(0, 1e-3) bulk).

Per configuration, one matrix of each class:

* the orthogonalised update alone (zeropower_via_newtonschulz5, reference
  opendm/optimizer/muon_adamw.py:101-128) for the first step's Nesterov
  direction, with both 11-bit operand types (fp16, the default, and tf32):
  relative Frobenius error below 5e-3 (the bar is 1e-2);
* one full MuonAdamW step with every class in one grouped plan (default fp16
  operands, bf16 parameters, fp32 momentum; reference :381-414) against the
  oracle step: momentum bit-exact, the parameter value before its final
  bf16 rounding within 1e-3, the parameter change within 1e-2 and the
  parameters within the bf16 rounding floor (tests/test_gpu_optimizer.py
  states it).

The oracle's fp32 Newton-Schulz of an input is computed once and shared by
both parts (keyed by the input's bytes). Each class's errors are printed
(`pytest -s`) as "parity <config> <shape> ..." lines.
"""

import hashlib

import numpy as np
import pytest
import torch

from oracle import muon_oracle as O
from tests.test_gpu_optimizer import BF16_PARAM_TOL, UPDATE_TOL, _check_params, precast_error

pytestmark = pytest.mark.gpu

C4 = [(2560, 2560), (512, 2560), (9728, 2560), (2560, 9728), (1152, 1152), (4304, 1152), (1152, 4304),
      (1024, 1024), (4096, 1024), (1024, 4096)]
C5 = [(4096, 4096), (11008, 4096), (4096, 11008)]
LR, WD = 0.02, 0.01


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _grad(shape, rng, heavy):
    g = rng.standard_normal(shape, dtype=np.float32) * np.float32(1e-3)
    if heavy:
        tail = rng.random(shape, dtype=np.float32) < 0.01
        g = np.where(tail, rng.standard_normal(shape, dtype=np.float32) * np.float32(1e-1), g)
    return O.cast_to(g.astype(np.float32), "bfloat16")


@pytest.mark.parametrize("config", ["c4", "c5"])
def test_config_shape_classes_match_oracle(config, monkeypatch):
    from opendm_b200.optimizer import MuonAdamW, mark_muon_parameters, zeropower_via_newtonschulz5

    dev = _dev()
    shapes = C4 if config == "c4" else C5
    heavy = config == "c5"
    rng = np.random.default_rng(4 if config == "c4" else 5)
    params = [O.cast_to(rng.standard_normal(s, dtype=np.float32) * np.float32(0.02), "bfloat16") for s in shapes]
    grads = [_grad(s, rng, heavy) for s in shapes]

    memo = {}
    oracle_ns = O.zeropower_via_newtonschulz5

    def shared_ns(m, steps=5, eps=1e-7):
        a = np.ascontiguousarray(m, np.float32)
        key = (hashlib.sha1(a.tobytes()).hexdigest(), a.shape, steps, eps)
        if key not in memo:
            memo[key] = oracle_ns(a, steps, eps)
        return memo[key]

    monkeypatch.setattr(O, "zeropower_via_newtonschulz5", shared_ns)

    # 1. the orthogonalised update of the first step's direction
    upd_err = {}
    for s, g in zip(shapes, grads):
        _, d = O.momentum_direction(g, np.zeros(s, np.float32), 0.95, True)
        want = shared_ns(d)
        dd = torch.from_numpy(d).to(dev)
        for prec in ("fp16", "tf32"):
            got = zeropower_via_newtonschulz5(dd, precision=prec).cpu().numpy()
            upd_err[(s, prec)] = O.rel_frobenius(got, want)
        del dd

    # 2. one full step, all classes in one grouped plan
    model = torch.nn.Module()
    for i, p in enumerate(params):
        model.register_parameter(f"p{i}", torch.nn.Parameter(torch.from_numpy(p).to(torch.bfloat16).to(dev)))
    mark_muon_parameters(model, predicate=lambda n, p: True)
    opt = MuonAdamW(model, lr=LR, betas=(0.9, 0.95), eps=1e-8, weight_decay=WD)
    tparams = list(model.parameters())
    for p, g in zip(tparams, grads):
        p.grad = torch.from_numpy(g).to(torch.bfloat16).to(dev)
    opt.step()
    stored = opt._engine.stored_updates()
    u_got = [stored[p.data_ptr()].float().cpu().numpy() for p in tparams]
    opt.check_device_errors()
    ref = O.OracleMuonAdamW(lr=LR, betas=(0.9, 0.95), eps=1e-8, weight_decay=WD)
    want_p = {str(i): p.copy() for i, p in enumerate(params)}
    updates = {}
    ref.step(want_p, {str(i): g for i, g in enumerate(grads)}, {}, {}, param_dtype="bfloat16", updates_out=updates,
             device_semantics="cuda")

    wd_factor = 1.0 - LR * WD
    failures = []
    for i, s in enumerate(shapes):
        got = tparams[i].detach().float().cpu().numpy()
        want = want_p[str(i)]
        eff = O.effective_lr(LR, 1.0, 0.2, s)
        pe = precast_error(params[i], u_got[i], updates[str(i)], wd_factor, eff)
        step_upd = O.rel_frobenius(u_got[i], O.cast_to(updates[str(i)], "bfloat16"))
        perr = O.rel_frobenius(got, want)
        print(f"parity {config} {s[0]}x{s[1]} update fp16 {upd_err[(s, 'fp16')]:.2e} tf32 {upd_err[(s, 'tf32')]:.2e}"
              f" step-update {step_upd:.2e} precast {pe:.2e} param {perr:.2e}")
        try:
            np.testing.assert_array_equal(opt.state[tparams[i]]["exp_avg"].cpu().numpy(), ref.muon_state[str(i)].exp_avg)
            for prec in ("fp16", "tf32"):
                assert upd_err[(s, prec)] < UPDATE_TOL, (s, prec, upd_err[(s, prec)])
            assert perr < BF16_PARAM_TOL
            _check_params(got, want, params[i], params[i], wd_factor, torch.bfloat16, s, max_beyond=2e-2,
                          precast=(u_got[i], updates[str(i)], eff))
        except AssertionError as exc:  # report every class before failing
            failures.append(repr(exc))
    assert not failures, failures
