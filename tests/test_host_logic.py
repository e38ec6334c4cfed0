"""Host logic of the drop-in optimizer on CPU: grouping, state layout, legacy
state, error conventions, selection, shard planning. The arithmetic is the
oracle's (tests/oracle_engine.py), so these tests need no GPU; the GPU tests
check the same flows through the CUDA library."""

import copy
import json
import os

import numpy as np
import pytest
import torch

from oracle import muon_oracle as O
from opendm_b200.optimizer import (MuonAdamW, MuonShardPlan, is_default_muon_parameter, mark_muon_parameters,
                                   zeropower_via_newtonschulz5)
from opendm_b200.optimizer.muon_adamw import _normalize_parameter_name
from opendm_b200.sharding import assign_owners, load_balance, ns_cost
from tests.oracle_engine import OracleEngine


class GoldenModel(torch.nn.Module):
    """Parameters named and shaped as in tests/golden/make_golden.py."""

    def __init__(self, z, dtype):
        super().__init__()
        keys = [k.split("/", 1)[1] for k in z.files if k.startswith("init/")]
        for k in keys:
            self.register_parameter(k, torch.nn.Parameter(torch.from_numpy(z[f"init/{k}"]).to(dtype)))
        self.muon_keys = set(z["muon_keys"].tolist())


def _golden(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def _build(z, dtype, **kw):
    model = GoldenModel(z, dtype)
    mark_muon_parameters(model, predicate=lambda n, p: n in model.muon_keys)
    opt = MuonAdamW(model, lr=float(z["meta_lr"]), betas=(0.9, 0.95), eps=1e-8, weight_decay=float(z["meta_wd"]),
                    muon_nesterov=bool(z["meta_nesterov"]), _engine=OracleEngine(), **kw)
    return model, opt


def _set_grads(model, z, s, dtype):
    for k, p in model.named_parameters():
        g = z[f"grad{s}/{k}"]
        p.grad = None if np.isnan(g).all() else torch.from_numpy(g).to(dtype)


@pytest.mark.parametrize("name,dtype", [("step_fp32.npz", torch.float32), ("step_nonesterov.npz", torch.float32),
                                        ("step_bf16.npz", torch.bfloat16)])
def test_dropin_matches_reference_steps(golden_dir, name, dtype):
    z = _golden(golden_dir, name)
    model, opt = _build(z, dtype)
    for s in range(int(z["meta_steps"])):
        _set_grads(model, z, s, dtype)
        opt.step()
        for k, p in model.named_parameters():
            ref = z[f"param{s}/{k}"]
            got = p.detach().float().numpy()
            if dtype == torch.float32:
                assert O.rel_frobenius(got, ref) < 1e-6, (s, k)
            else:
                assert np.sum(got != ref) <= max(2, 2e-3 * got.size), (s, k)
    for k, p in model.named_parameters():
        st = opt.state[p]
        assert O.rel_frobenius(st["exp_avg"].numpy(), z[f"exp_avg/{k}"]) < 1e-6
        assert float(st["step"]) == float(z[f"step/{k}"])
        assert st["step"].dtype == torch.float32 and st["step"].shape == ()


def test_state_dict_layout_matches_reference(golden_dir):
    z = _golden(golden_dir, "step_bf16.npz")
    with open(os.path.join(golden_dir, "state_layout.json")) as f:
        layout = json.load(f)
    model, opt = _build(z, torch.bfloat16)
    _set_grads(model, z, 0, torch.bfloat16)
    opt.step()
    sd = opt.state_dict()
    assert len(sd["param_groups"]) == len(layout["param_groups"])
    for got, ref in zip(sd["param_groups"], layout["param_groups"]):
        assert got["params"] == ref["params"]
        for key, value in ref.items():
            if key in ("n_params", "params"):
                continue
            if value is None and key in ("muon_shapes", "muon_names"):
                assert key not in got
                continue
            v = got[key]
            v = [list(x) for x in v] if key == "muon_shapes" else (list(v) if isinstance(v, tuple) else v)
            assert v == value, key
        assert set(got) == {k for k, v in ref.items() if k not in ("n_params",) and
                            not (v is None and k in ("muon_shapes", "muon_names"))}
    assert set(sd["state"]) == {int(k) for k in layout["state"]}
    for k, entry in layout["state"].items():
        st = sd["state"][int(k)]
        assert set(st) == set(entry)
        for sk, (dt, shape) in entry.items():
            assert str(st[sk].dtype) == dt and list(st[sk].shape) == shape


def test_state_dict_round_trip_continues_identically(golden_dir):
    z = _golden(golden_dir, "step_fp32.npz")
    model_a, opt_a = _build(z, torch.float32)
    _set_grads(model_a, z, 0, torch.float32)
    opt_a.step()
    sd = copy.deepcopy(opt_a.state_dict())  # as if saved to disk and loaded back
    model_b, opt_b = _build(z, torch.float32)
    with torch.no_grad():
        for pa, pb in zip(model_a.parameters(), model_b.parameters()):
            pb.copy_(pa)
    opt_b.load_state_dict(sd)
    for s in (1, 2):
        _set_grads(model_a, z, s, torch.float32)
        _set_grads(model_b, z, s, torch.float32)
        opt_a.step()
        opt_b.step()
    for pa, pb in zip(model_a.parameters(), model_b.parameters()):
        torch.testing.assert_close(pa, pb, rtol=0, atol=0)


def test_load_legacy_state_forms(golden_dir):
    z = _golden(golden_dir, "step_fp32.npz")
    model, opt = _build(z, torch.float32)
    _set_grads(model, z, 0, torch.float32)
    opt.step()
    sd = opt.state_dict()
    legacy = {"state": {}, "param_groups": []}
    for idx, st in sd["state"].items():
        legacy["state"][idx] = {"momentum_buffer": st["exp_avg"].clone(), "exp_avg_sq": st["exp_avg_sq"].clone(),
                                "step": float(st["step"])}
    adam_g, muon_g = [dict(g) for g in sd["param_groups"]]
    shapes = muon_g.pop("muon_shapes")
    names = muon_g.pop("muon_names")
    muon_g["muon_param_infos"] = [{"matrix_shape": s, "name": n} for s, n in zip(shapes, names)]
    legacy["param_groups"] = [adam_g, muon_g]
    model2, opt2 = _build(z, torch.float32)
    opt2.load_state_dict(legacy)
    g = opt2.param_groups[1]
    assert g["muon_shapes"] == [tuple(s) for s in shapes] and g["muon_names"] == names
    for p in g["params"]:
        st = opt2.state[p]
        assert "momentum_buffer" not in st and st["exp_avg"].dtype == torch.float32
        assert torch.is_tensor(st["step"]) and st["step"].dtype == torch.float32
    # tuple-form infos and muon_matrix_shapes
    muon_g2 = dict(sd["param_groups"][1])
    muon_g2["muon_matrix_shapes"] = muon_g2.pop("muon_shapes")
    muon_g2.pop("muon_names")
    model3, opt3 = _build(z, torch.float32)
    opt3.load_state_dict({"state": sd["state"], "param_groups": [sd["param_groups"][0], muon_g2]})
    assert opt3.param_groups[1]["muon_shapes"] == [tuple(s) for s in shapes]
    assert opt3.param_groups[1]["muon_names"] == [None] * len(shapes)
    infos_t = [(n, s) for s, n in zip(shapes, names)]
    muon_g3 = dict(sd["param_groups"][1])
    muon_g3.pop("muon_shapes")
    muon_g3.pop("muon_names")
    muon_g3["muon_param_infos"] = infos_t
    model4, opt4 = _build(z, torch.float32)
    opt4.load_state_dict({"state": sd["state"], "param_groups": [sd["param_groups"][0], muon_g3]})
    assert opt4.param_groups[1]["muon_shapes"] == [tuple(s) for s in shapes]


def test_bad_state_and_metadata_raise(golden_dir):
    z = _golden(golden_dir, "step_fp32.npz")
    model, opt = _build(z, torch.float32)
    p = opt.param_groups[1]["params"][0]
    with pytest.raises(RuntimeError, match="one value"):
        opt._state_for_param(p, {"step": torch.zeros(2)})
    opt.param_groups[1]["muon_shapes"] = opt.param_groups[1]["muon_shapes"][:-1]
    with pytest.raises(RuntimeError, match="metadata does not match"):
        opt._normalize_param_groups()
    opt.param_groups[1]["muon_shapes"] = [(1, 1)] * len(opt.param_groups[1]["params"])
    opt.param_groups[1]["muon_names"] = ["x"]
    with pytest.raises(RuntimeError, match="names do not match"):
        opt._normalize_param_groups()


class Tiny(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.model = torch.nn.Module()
        self.model.action_expert = torch.nn.Module()
        self.model.action_expert.layers = torch.nn.ModuleList([torch.nn.Linear(8, 16, bias=True)])
        self.model.action_expert.norm = torch.nn.LayerNorm(8)
        self.model.embed_tokens = torch.nn.Embedding(10, 8)
        self.head = torch.nn.Linear(8, 4)


def test_default_selection_and_marking():
    m = Tiny()
    names = mark_muon_parameters(m)
    assert names == ["model.action_expert.layers.0.weight"]
    w = m.model.action_expert.layers[0].weight
    assert w._opendm_muon_shape == (16, 8) and w._opendm_muon_name == names[0]
    assert not hasattr(m.head.weight, "_opendm_muon_shape")
    assert is_default_muon_parameter("module._fsdp_wrapped_module.model.action_expert.layers.3.mlp.up.weight",
                                     torch.nn.Parameter(torch.zeros(2, 2)))
    assert not is_default_muon_parameter("model.action_expert.layers.3.input_layernorm.weight",
                                         torch.nn.Parameter(torch.zeros(2, 2)))
    assert not is_default_muon_parameter("model.action_expert.layers.3.x.weight",
                                         torch.nn.Parameter(torch.zeros(2, 2), requires_grad=False))
    assert not is_default_muon_parameter("model.language.layers.3.x.weight", torch.nn.Parameter(torch.zeros(2, 2)))
    assert _normalize_parameter_name("module._orig_mod.module.x") == "x"


def test_marking_errors_and_missing_metadata():
    m = Tiny()
    with pytest.raises(RuntimeError, match="selected 0"):
        mark_muon_parameters(m, predicate=lambda n, p: False)
    with pytest.raises(RuntimeError, match="must be 2D"):
        mark_muon_parameters(m, predicate=lambda n, p: n.endswith("bias"))
    with pytest.raises(RuntimeError, match="metadata is missing"):
        MuonAdamW(Tiny(), lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, _engine=OracleEngine())
    mark_muon_parameters(m)
    for kw in ({"precision": "fp8"}, {"sharding": "zero3"}, {"scale_mode": "x"}):
        with pytest.raises(ValueError):
            MuonAdamW(m, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, _engine=OracleEngine(), **kw)


def test_sparse_and_mismatched_grads_raise():
    m = Tiny()
    mark_muon_parameters(m)
    opt = MuonAdamW(m, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, _engine=OracleEngine())
    w = m.model.action_expert.layers[0].weight
    w.grad = torch.zeros(16, 8)
    w.grad.data = torch.zeros(3)  # a flat shard whose gradient does not match
    with pytest.raises(RuntimeError, match="shape mismatch"):
        opt.step()
    w.grad = torch.zeros(16, 8).to_sparse()
    with pytest.raises(RuntimeError, match="sparse"):
        opt.step()
    w.grad = None
    m.head.weight.grad = torch.zeros(4, 8).to_sparse()
    with pytest.raises(RuntimeError, match="sparse"):
        opt.step()


def test_param_groups_order_and_defaults():
    m = Tiny()
    mark_muon_parameters(m)
    opt = MuonAdamW(m, lr=2e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, muon_ns_steps=3,
                    _engine=OracleEngine())
    g0, g1 = opt.param_groups
    assert g0["use_muon"] is False and g1["use_muon"] is True
    for g in (g0, g1):
        for k in ("lr", "betas", "eps", "weight_decay", "muon_momentum", "muon_nesterov", "muon_ns_steps",
                  "muon_lr_scale", "muon_moonlight_coefficient"):
            assert k in g
    assert g1["muon_shapes"] == [(16, 8)] and g1["muon_names"] == ["model.action_expert.layers.0.weight"]
    assert g1["muon_ns_steps"] == 3


def test_reference_caller_sequence_with_a_warmup_schedule():
    """The calls the reference's trainer makes, replayed on this optimizer
    (dm05_exp cannot be imported here: it needs flask): prepare_model marks
    the default Muon set (dm05_exp.py:276-278, is_default_muon_parameter),
    build_muon_adamw constructs the optimizer with DM05OptimizerConfig's
    defaults (:255-267, :280-292; DMTrainer.create_optimizer, trainer.py:122-130),
    then the HF loop's order each step: gradients, optimizer.step(),
    lr_scheduler.step() (a warmup LambdaLR rewriting group["lr"]). Only the
    action expert's layer weights go to Muon, and every step matches the
    oracle optimizer run at the scheduled learning rate."""
    gen = torch.Generator().manual_seed(11)

    def linear(o, i):
        lin = torch.nn.Linear(i, o, bias=False)
        lin.weight.data = torch.randn(o, i, generator=gen) * 0.02
        return lin

    model = torch.nn.Module()
    model.model = torch.nn.Module()
    model.model.embed_tokens = torch.nn.Embedding(40, 16)
    model.model.language_model = torch.nn.Module()
    model.model.language_model.layers = torch.nn.ModuleList([linear(16, 16)])
    model.model.action_expert = torch.nn.Module()
    model.model.action_expert.layers = torch.nn.ModuleList([linear(48, 16), linear(16, 48)])
    model.model.action_expert.norm = torch.nn.LayerNorm(16, bias=False)
    cfg = {"base_lr": 2.5e-5, "weight_decay": 1e-10, "warmup_steps": 4, "adam_beta1": 0.9, "adam_beta2": 0.95,
           "adam_epsilon": 1e-8, "muon_momentum": 0.95, "muon_nesterov": True, "muon_ns_steps": 5,
           "muon_lr_scale": 1.0, "muon_moonlight_coefficient": 0.2}
    selected = mark_muon_parameters(model, predicate=is_default_muon_parameter)
    assert sorted(selected) == ["model.action_expert.layers.0.weight", "model.action_expert.layers.1.weight"]
    opt = MuonAdamW(model, lr=cfg["base_lr"], betas=(cfg["adam_beta1"], cfg["adam_beta2"]), eps=cfg["adam_epsilon"],
                    weight_decay=cfg["weight_decay"], muon_momentum=cfg["muon_momentum"],
                    muon_nesterov=cfg["muon_nesterov"], muon_ns_steps=cfg["muon_ns_steps"],
                    muon_lr_scale=cfg["muon_lr_scale"], muon_moonlight_coefficient=cfg["muon_moonlight_coefficient"],
                    _engine=OracleEngine())
    sched = torch.optim.lr_scheduler.LambdaLR(opt, lambda s: min(1.0, (s + 1) / cfg["warmup_steps"]))
    ref = O.OracleMuonAdamW(lr=cfg["base_lr"], betas=(cfg["adam_beta1"], cfg["adam_beta2"]), eps=cfg["adam_epsilon"],
                            weight_decay=cfg["weight_decay"])
    host = {n: p.detach().numpy().copy() for n, p in model.named_parameters()}
    muon = {n: host[n] for n in selected}
    adam = {n: v for n, v in host.items() if n not in muon}
    for step in range(3):
        grads = {}
        for n, p in model.named_parameters():
            p.grad = torch.randn(p.shape, generator=gen) * 1e-3
            grads[n] = p.grad.numpy().copy()
        lrs = {g["lr"] for g in opt.param_groups}
        assert lrs == {cfg["base_lr"] * min(1.0, (step + 1) / cfg["warmup_steps"])}
        ref.lr = lrs.pop()
        ref.step(muon, {n: grads[n] for n in muon}, adam, {n: grads[n] for n in adam})
        opt.step()
        sched.step()
        for n, p in model.named_parameters():
            want = muon.get(n, adam.get(n))
            assert O.rel_frobenius(p.detach().numpy(), want) < 1e-6, (step, n)


@pytest.mark.parametrize("mode", ["reference", "shape"])
def test_update_scale_per_matrix(mode):
    """The update scale each matrix hands the engine: the reference's
    lr * lr_scale * coefficient * sqrt(max(rows, cols)) (muon_adamw.py:408-413)
    by default, lr * lr_scale * max(1, rows / cols) ** 0.5 with
    scale_mode="shape", read from the group at every step (a scheduler's new
    lr takes effect on the next step)."""
    import math

    class Recording(OracleEngine):
        def __init__(self):
            super().__init__()
            self.effs = []

        def muon_matrices(self, items, **kw):
            self.effs.append(sorted((tuple(it.param.shape), it.eff) for it in items))
            super().muon_matrices(items, **kw)

    m = torch.nn.Module()
    m.wide = torch.nn.Parameter(torch.randn(8, 32) * 0.02)
    m.tall = torch.nn.Parameter(torch.randn(32, 8) * 0.02)
    mark_muon_parameters(m, predicate=lambda n, p: p.ndim == 2)
    eng = Recording()
    opt = MuonAdamW(m, lr=0.02, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, muon_lr_scale=0.5,
                    scale_mode=mode, _engine=eng)
    for lr in (0.02, 0.005):
        opt.param_groups[1]["lr"] = lr
        for p in m.parameters():
            p.grad = torch.full_like(p, 1e-3)
        opt.step()
        want = {(8, 32): lr * 0.5 * (0.2 * math.sqrt(32) if mode == "reference" else 1.0),
                (32, 8): lr * 0.5 * (0.2 * math.sqrt(32) if mode == "reference" else 2.0)}
        got = dict(eng.effs[-1])
        assert got.keys() == want.keys()
        for k in want:
            assert got[k] == pytest.approx(want[k], rel=1e-12), (k, got[k], want[k])


def test_add_param_group_adds_an_adamw_group():
    """torch.optim.Optimizer.add_param_group after construction, which the
    reference does not override: the new group gets every default key with
    use_muon False, so its parameters take the AdamW path with the reference's
    state (step, exp_avg, exp_avg_sq), and the Muon group is unchanged."""
    m = Tiny()
    mark_muon_parameters(m)
    eng = OracleEngine()
    opt = MuonAdamW(m, lr=2e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, _engine=eng)
    extra = torch.nn.Parameter(torch.randn(32, generator=torch.Generator().manual_seed(3)) * 0.02)
    opt.add_param_group({"params": [extra]})
    new = opt.param_groups[-1]
    assert len(opt.param_groups) == 3 and new["use_muon"] is False
    assert set(new) == set(opt.param_groups[0])
    for p in list(m.parameters()) + [extra]:
        p.grad = torch.full_like(p, 1e-3)
    before = extra.detach().clone()
    opt.step()
    assert sorted(opt.state[extra]) == ["exp_avg", "exp_avg_sq", "step"]
    assert float(opt.state[extra]["step"]) == 1.0 and not torch.equal(before, extra.detach())
    assert eng.calls["muon"] == 1


def test_muon_group_inactive_without_grads():
    m = Tiny()
    mark_muon_parameters(m)
    eng = OracleEngine()
    opt = MuonAdamW(m, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, _engine=eng)
    before = m.model.action_expert.layers[0].weight.detach().clone()
    opt.step()
    assert eng.calls["muon"] == 0
    assert torch.equal(before, m.model.action_expert.layers[0].weight)
    assert opt.state == {} or all(not s for s in opt.state.values())


def test_closure_and_lr_read_each_step():
    m = Tiny()
    mark_muon_parameters(m)
    opt = MuonAdamW(m, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, _engine=OracleEngine())
    x = torch.randn(4, 8)

    def closure():
        opt.zero_grad()
        loss = m.model.action_expert.layers[0](x).sum() + m.head(x).sum()
        loss.backward()
        return loss

    loss = opt.step(closure)
    assert torch.is_tensor(loss)
    w = m.model.action_expert.layers[0].weight
    before = w.detach().clone()
    for g in opt.param_groups:
        g["lr"] = 0.0
    opt.step(closure)
    assert torch.equal(before, w)  # lr is read from the group at every step


def test_group_hyperparameters_read_each_step():
    """weight_decay, muon_momentum and muon_nesterov changed in the Muon
    group between steps (as a scheduler may) take effect on the next step:
    three steps with different values match the oracle run with the same
    values (reference muon_adamw.py:362-414 reads them from the group)."""
    gen = torch.Generator().manual_seed(5)
    w0 = torch.randn(24, 40, generator=gen) * 0.02
    m = torch.nn.Module()
    m.w = torch.nn.Parameter(w0.clone())
    mark_muon_parameters(m, predicate=lambda n, p: p.ndim == 2)
    opt = MuonAdamW(m, lr=0.02, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.01, _engine=OracleEngine())
    p_ref = {"w": w0.numpy().copy()}
    ref_state = None
    for wd, mu, nest in [(0.01, 0.95, True), (0.1, 0.9, False), (0.0, 0.5, True)]:
        g = torch.randn(24, 40, generator=gen) * 1e-3
        m.w.grad = g.clone()
        group = opt.param_groups[1]
        group["weight_decay"], group["muon_momentum"], group["muon_nesterov"] = wd, mu, nest
        opt.step()
        ref = O.OracleMuonAdamW(lr=0.02, betas=(0.9, 0.95), eps=1e-8, weight_decay=wd, muon_momentum=mu,
                                muon_nesterov=nest)
        if ref_state is not None:
            ref.muon_state = ref_state
        ref.step(p_ref, {"w": g.numpy()}, {}, {})
        ref_state = ref.muon_state
        assert O.rel_frobenius(m.w.detach().numpy(), p_ref["w"]) < 1e-6
        assert O.rel_frobenius(opt.state[m.w]["exp_avg"].numpy(), ref_state["w"].exp_avg) < 1e-6


def test_zeropower_cpu_has_no_fallback():
    with pytest.raises(ValueError):
        zeropower_via_newtonschulz5(torch.zeros(2, 3, 4))
    with pytest.raises(RuntimeError, match="CUDA"):
        zeropower_via_newtonschulz5(torch.ones(4, 4))


def test_unsupported_dtypes_and_devices_raise():
    """The kernels take bfloat16 or float32 tensors on a CUDA device; any other
    dtype, and a CPU engine, raise RuntimeError naming the problem instead of
    running some other path."""
    from opendm_b200 import engine as E

    assert E._dtype_code(torch.zeros(1, dtype=torch.bfloat16)) != E._dtype_code(torch.zeros(1))
    for dt in (torch.float16, torch.float64):
        with pytest.raises(RuntimeError, match=f"unsupported dtype {dt}"):
            E._dtype_code(torch.zeros(1, dtype=dt))
    with pytest.raises(RuntimeError, match="CUDA"):
        E.CudaMuonEngine("cpu")


def test_shard_plan_dataclass_matches_reference_fields():
    p = MuonShardPlan("local", 6, 6, (6,), (0,), 0)
    assert p.process_group is None and p.kind == "local"
    with pytest.raises(Exception):
        p.kind = "x"  # frozen


def test_lpt_assignment_balances_and_is_deterministic():
    shapes = [(2048, 2048)] * 56 + [(256, 2048)] * 56 + [(8192, 2048)] * 56 + [(2048, 8192)] * 28
    for world in (2, 4, 8):
        owners = assign_owners(shapes, world)
        assert owners == assign_owners(shapes, world)
        assert set(owners) == set(range(world))
        lb = load_balance(shapes, owners, world)
        assert lb["max_over_mean"] < 1.02, lb
    assert assign_owners(shapes, 1) == [0] * len(shapes)
    assert ns_cost((8, 4)) == ns_cost((4, 8)) == 5 * (4 * 16 * 8 + 2 * 64)


def test_waves_follow_geometric_flop_shares():
    """Each rank's matrices, most bytes per FLOP first, are cut into waves
    whose FLOP shares shrink geometrically; deterministic and identical on
    every rank."""
    from opendm_b200.sharding import assign_waves, wave_fractions

    fr = wave_fractions(3)
    assert abs(sum(fr) - 1) < 1e-12 and fr[0] > fr[1] > fr[2]
    shapes = [(2048, 2048)] * 56 + [(256, 2048)] * 56 + [(8192, 2048)] * 56 + [(2048, 8192)] * 28
    for world in (1, 2, 8):
        owners = assign_owners(shapes, world)
        waves = assign_waves(shapes, owners, world, 3)
        assert waves == assign_waves(shapes, owners, world, 3)
        for r in range(world):
            mine = [i for i, o in enumerate(owners) if o == r]
            total = sum(ns_cost(shapes[i]) for i in mine)
            share = [sum(ns_cost(shapes[i]) for i in mine if waves[i] == w) / total for w in range(3)]
            # within one matrix of the target share; waves never grow
            biggest = max(ns_cost(shapes[i]) for i in mine) / total
            for w in range(3):
                assert abs(share[w] - fr[w]) <= biggest + 1e-9, (world, r, share)
            # byte-heavy (small-m) matrices in earlier waves: waves never decrease along that order
            by_bpf = sorted(mine, key=lambda i: (-shapes[i][0] * shapes[i][1] / ns_cost(shapes[i]),
                                                 -ns_cost(shapes[i]), i))
            assert [waves[i] for i in by_bpf] == sorted(waves[i] for i in by_bpf)
    assert assign_waves(shapes, assign_owners(shapes, 2), 2, 1) == [0] * len(shapes)


def test_partial_owner_choice_is_active_and_balanced():
    """FSDP owner-only Newton-Schulz: each split matrix goes to one of its
    active ranks, by LPT on FLOPs, identically on every rank."""
    from opendm_b200.optimizer.muon_adamw import MuonAdamW, MuonShardPlan

    shapes = [(512, 512), (256, 1024), (1024, 256), (128, 128), (64, 640), (640, 64)]
    plans, idx = [], []
    for j, s in enumerate(shapes):
        n = s[0] * s[1]
        active = (0, 1, 2) if j % 2 == 0 else (1, 2)
        sizes = tuple(n // len(active) + (n % len(active) if r == active[-1] else 0) if r in active else 0
                      for r in range(3))
        plans.append(MuonShardPlan("partial", n, sizes[0], sizes, active, 0))
        idx.append(j)
    owners = MuonAdamW._partial_owners(plans, shapes, idx, 5)
    assert owners == MuonAdamW._partial_owners(plans, shapes, idx, 5)
    for j in idx:
        assert owners[j] in plans[j].active_ranks
    load = [0.0] * 3
    for j, r in owners.items():
        load[r] += ns_cost(shapes[j])
    # greedy list scheduling's bound: the busiest rank carries at most the mean plus the largest job
    assert max(load) <= sum(load) / 3 + max(ns_cost(s) for s in shapes)


def test_flat_buckets_layout_repoints_parameters():
    """Owned matrices are laid out per (wave, dtype) as [rank 0 | rank 1 | ...]
    buckets of equal, 128-element-aligned size; parameters become views of
    them with their values kept."""
    from opendm_b200.sharding import FlatParamBuckets

    torch.manual_seed(0)
    shapes = [(8, 16), (4, 4), (16, 8), (3, 5), (10, 10)]
    params = [torch.nn.Parameter(torch.randn(s)) for s in shapes]
    before = [p.detach().clone() for p in params]
    owners = [0, 1, 1, 0, 1]
    waves = [0, 0, 1, 1, 0]
    b = FlatParamBuckets(params, owners, 2, 0, None, waves)
    assert b.n_waves == 2
    for flat, bucket, wave in b.buffers:
        assert bucket % 128 == 0 and flat.numel() == 2 * bucket
        for i, p in enumerate(params):
            if waves[i] != wave:
                continue
            off = p.data.storage_offset() - flat.storage_offset()
            assert p.data.untyped_storage().data_ptr() == flat.untyped_storage().data_ptr()
            assert owners[i] * bucket <= off < (owners[i] + 1) * bucket  # inside its owner's bucket
    for p, w in zip(params, before):
        assert torch.equal(p.detach(), w)
    expect = sum(bucket * 4 for flat, bucket, _ in b.buffers)  # fp32, one peer's bucket per wave
    assert b.nbytes_received() == expect


def test_flat_adam_shards_ranges_tile_and_align():
    """AdamW sharding layout: per dtype, parameters back to back at
    64-element boundaries, the flat buffer cut into equal 64-aligned ranges;
    every parameter is covered exactly once by the ranks' pieces, each piece
    starts aligned, parameters become views with their values kept, and the
    dtypes get separate buffers."""
    from opendm_b200.sharding import FlatAdamShards

    torch.manual_seed(0)
    shapes = [(1000,), (7,), (64, 33), (130,), (5,)]
    dtypes = [torch.float32, torch.float32, torch.bfloat16, torch.float32, torch.bfloat16]
    for world in (1, 2, 3, 4, 8):
        params = [torch.nn.Parameter(torch.randn(s).to(d)) for s, d in zip(shapes, dtypes)]
        before = [p.detach().clone() for p in params]
        sh = FlatAdamShards(params, world, 0)
        assert len(sh.buffers) == 2
        for flat, per_rank, placed in sh.buffers:
            assert per_rank % FlatAdamShards.ALIGN == 0 and flat.numel() == per_rank * world
            for i, off in placed:
                assert off % FlatAdamShards.ALIGN == 0 and params[i].dtype == flat.dtype
                assert params[i].data.untyped_storage().data_ptr() == flat.untyped_storage().data_ptr()
                assert params[i].data.storage_offset() - flat.storage_offset() == off
        for p, w in zip(params, before):
            assert torch.equal(p.detach(), w)
        covered = {i: [] for i in range(len(shapes))}
        for i, r, start, length in sh.ranges(params):
            assert 0 <= r < world and length > 0
            off = dict(sh.buffers[0][2] + sh.buffers[1][2])[i]
            per_rank = next(b for _, b, pl in sh.buffers if any(j == i for j, _ in pl))
            assert (off + start) % FlatAdamShards.ALIGN == 0  # piece starts 64-element aligned in the buffer
            assert r * per_rank <= off + start and off + start + length <= (r + 1) * per_rank
            covered[i].append((start, length))
        for i, spans in covered.items():
            spans.sort()
            assert spans[0][0] == 0 and sum(n for _, n in spans) == params[i].numel()
            assert all(a + n == b for (a, n), (b, _) in zip(spans, spans[1:]))
        mine = sh.owned(params)
        assert all((i, 0, s, n) in [(j, r, a, b) for j, r, a, b in sh.ranges(params)] for i, s, n in mine)
        assert sh.nbytes_received() == sum(b * flat.element_size() * (world - 1) for flat, b, _ in sh.buffers)


def test_adamw_sharding_needs_state_sharding():
    model = torch.nn.Linear(8, 8, bias=True)
    mark_muon_parameters(model, lambda n, p: p.ndim == 2)
    with pytest.raises(ValueError, match="state_sharding"):
        MuonAdamW(model, lr=0.02, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.01, adamw_sharding=True,
                  _engine=OracleEngine())


def test_more_option_validation():
    m = Tiny()
    mark_muon_parameters(m)
    for kw in ({"ns_algo": "fast"}, {"allgather_waves": 0}, {"allgather": "mpi"}):
        with pytest.raises(ValueError):
            MuonAdamW(m, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, _engine=OracleEngine(), **kw)


def test_shard_plan_errors_single_process():
    """Reference :443-535 error paths: a local tensor larger than the marked
    matrix, a partial tensor without a process group, a local tensor that no
    longer matches its plan, and an unknown plan kind."""
    from opendm_b200.optimizer.muon_adamw import MuonShardPlan as Plan

    for numel, match in ((32, "has only 16 elements"), (8, "expected 0 or 16")):
        model = torch.nn.Module()
        p = torch.nn.Parameter(torch.zeros(numel))
        p._opendm_muon_shape, p._opendm_muon_name = (4, 4), "w"
        model.register_parameter("w", p)
        opt = MuonAdamW(model, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, _engine=OracleEngine())
        p.grad = torch.zeros(numel)
        with pytest.raises(RuntimeError, match=match):
            opt.step()
    plan = Plan("local", 16, 16, (16,), (0,), 0)
    with pytest.raises(RuntimeError, match="no longer matches"):
        MuonAdamW._gather_matrix(torch.zeros(8), plan)
    with pytest.raises(RuntimeError, match="Unknown Muon shard plan kind"):
        MuonAdamW._gather_matrix(torch.zeros(16), Plan("striped", 16, 16, (16,), (0,), 0))


def test_nvtx_ranges_balanced(monkeypatch):
    """The optimizer's NVTX ranges ("opendm/step", waves, all-gathers) close
    on every path, exceptions included."""
    from opendm_b200 import trace

    depth, names = [0], []

    def push(name):
        depth[0] += 1
        names.append(name)

    def pop():
        depth[0] -= 1

    monkeypatch.setattr(trace, "ENABLED", True)
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", push)
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", pop)
    m = Tiny()
    mark_muon_parameters(m)
    opt = MuonAdamW(m, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, _engine=OracleEngine())
    for p in m.parameters():
        p.grad = torch.zeros_like(p)
    opt.step()
    assert depth[0] == 0 and "opendm/step" in names
    with pytest.raises(ZeroDivisionError):
        with trace.nvtx("boom"):
            1 / 0
    assert depth[0] == 0


def test_default_wave_counts():
    """allgather_waves=None: 4 waves at >= 8 ranks with >= 16 dense TFLOP of
    Newton-Schulz per rank (config 4), else 3 with >= 6 matrices per rank
    (config 2 at 2-8 ranks), 1 with fewer matrices or off CUDA."""
    import bench

    m = Tiny()
    mark_muon_parameters(m)
    opt = MuonAdamW(m, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, _engine=OracleEngine())
    cuda = torch.device("cuda")
    shapes = {c: [s for n, s in bench.config_params(c) if bench.is_muon(n, s)] for c in ("c2", "c4")}
    assert opt._n_waves(shapes["c4"], 8, cuda, 5) == 4
    assert opt._n_waves(shapes["c4"], 4, cuda, 5) == 3
    for world in (2, 4, 8):
        assert opt._n_waves(shapes["c2"], world, cuda, 5) == 3
    assert opt._n_waves(shapes["c2"][:40], 8, cuda, 5) == 1  # 5 matrices per rank
    assert opt._n_waves(shapes["c2"], 8, torch.device("cpu"), 5) == 1


def test_wave_ratio_shapes_the_waves():
    """allgather_wave_ratio: 1.0 cuts a rank's matrices into waves of equal FLOP
    shares, a ratio below 1 front-loads them; every rank gets the same count."""
    from opendm_b200.sharding import assign_owners, assign_waves, ns_cost, wave_fractions

    assert wave_fractions(4, 1.0) == [0.25] * 4
    f = wave_fractions(3, 0.5)
    assert abs(sum(f) - 1.0) < 1e-12 and f[0] > f[1] > f[2]
    shapes = [(512, 512)] * 48
    owners = assign_owners(shapes, 2)
    for ratio in (0.5, 1.0, 1.5):
        waves = assign_waves(shapes, owners, 2, 4, ratio=ratio)
        for r in range(2):
            mine = [w for w, o in zip(waves, owners) if o == r]
            counts = [mine.count(w) for w in range(4)]
            assert sum(counts) == len(mine) and all(c > 0 for c in counts), (ratio, counts)
            if ratio == 1.0:
                assert max(counts) - min(counts) <= 1, counts
            if ratio == 0.5:
                assert counts[0] > counts[-1], counts
    assert ns_cost((512, 512)) > 0
