"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs the unmodified reference optimizer (``opendm/optimizer/muon_adamw.py`` of
dexmal/opendm, imported from a local checkout) on seeded inputs and stores its
outputs as ``.npz`` files next to this script. Run it where the reference
checkout exists (it is not needed at test time):

    python tests/golden/make_golden.py --reference PATH   (or OPENDM_REFERENCE=PATH)

Fixtures:
  ns_cases.npz           zeropower_via_newtonschulz5 on assorted shapes/steps
  step_fp32.npz          3 MuonAdamW steps, fp32 params (absent grad on step 2)
  step_bf16.npz          3 MuonAdamW steps, bf16 params
  step_nonesterov.npz    2 steps, nesterov=False, weight_decay=0
  state_layout.json      structure of the reference's state_dict() after a step
  clip_cases.npz         torch.nn.utils.clip_grad_norm_ (torch 2.11.0, the call the
                         reference's trainer makes before each step) on bf16,
                         fp32 and mixed gradient sets, below and above max_norm
bf16 tensors are stored as float32 holding the bf16 values.
``--only clip`` writes clip_cases.npz alone (it needs no reference checkout).
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

MUON_SHAPES = {
    "layers.0.q.weight": (32, 32),
    "layers.0.up.weight": (64, 32),     # tall
    "layers.0.down.weight": (32, 64),   # wide
    "layers.1.odd.weight": (24, 40),
    "layers.1.k.weight": (16, 16),
    "layers.1.v.weight": (16, 16),
}
ADAMW_SHAPES = {
    "norm0.weight": (32,),
    "norm1.weight": (32,),
    "bias0": (32,),
    "bias1": (32,),
    "embed_tokens.weight": (50, 16),    # 2-D but not selected for Muon
}


class _Model(torch.nn.Module):
    def __init__(self, dtype: torch.dtype, gen: torch.Generator):
        super().__init__()
        self.names = []
        for name, shape in list(MUON_SHAPES.items()) + list(ADAMW_SHAPES.items()):
            t = torch.randn(shape, generator=gen) * 0.02
            p = torch.nn.Parameter(t.to(dtype))
            self.register_parameter(name.replace(".", "_"), p)
            self.names.append(name)


def _to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy().copy()


def _run_steps(ref, dtype: torch.dtype, steps: int, *, nesterov: bool, weight_decay: float,
               absent: dict[int, str] | None = None, layout_out: dict | None = None) -> dict:
    gen = torch.Generator().manual_seed(1234)
    model = _Model(dtype, gen)
    muon_keys = {k.replace(".", "_") for k in MUON_SHAPES}
    ref.mark_muon_parameters(model, predicate=lambda n, p: n in muon_keys)
    opt = ref.MuonAdamW(model, lr=0.02, betas=(0.9, 0.95), eps=1e-8, weight_decay=weight_decay,
                        muon_momentum=0.95, muon_nesterov=nesterov, muon_ns_steps=5,
                        muon_lr_scale=1.0, muon_moonlight_coefficient=0.2)
    out = {"meta_lr": np.float64(0.02), "meta_wd": np.float64(weight_decay),
           "meta_nesterov": np.int64(nesterov), "meta_steps": np.int64(steps)}
    params = dict(model.named_parameters())
    for key, p in params.items():
        out[f"init/{key}"] = _to_np(p)
    for s in range(steps):
        ggen = torch.Generator().manual_seed(100 + s)
        for key, p in params.items():
            g = torch.randn(p.shape, generator=ggen) * 1e-3
            if absent and absent.get(s) == key:
                p.grad = None
                out[f"grad{s}/{key}"] = np.full(p.shape, np.nan, np.float32)
            else:
                p.grad = g.to(dtype)
                out[f"grad{s}/{key}"] = _to_np(p.grad)
        opt.step()
        for key, p in params.items():
            out[f"param{s}/{key}"] = _to_np(p)
    for key, p in params.items():
        st = opt.state[p]
        out[f"exp_avg/{key}"] = _to_np(st["exp_avg"])
        out[f"exp_avg_sq/{key}"] = _to_np(st["exp_avg_sq"])
        out[f"step/{key}"] = np.float32(st["step"].item())
    out["muon_keys"] = np.array(sorted(muon_keys))
    if layout_out is not None:
        sd = opt.state_dict()
        groups = []
        for g in sd["param_groups"]:
            groups.append({k: (list(v) if isinstance(v, tuple) else v) for k, v in g.items()
                           if k not in ("params", "muon_shapes", "muon_names")}
                          | {"n_params": len(g["params"]), "params": g["params"],
                             "muon_shapes": [list(x) for x in g.get("muon_shapes", [])] or None,
                             "muon_names": g.get("muon_names")})
        state = {str(k): {sk: [str(sv.dtype), list(sv.shape)] for sk, sv in v.items()}
                 for k, v in sd["state"].items()}
        layout_out.update({"param_groups": groups, "state": state})
    return out


def _ns_cases(ref) -> dict:
    gen = torch.Generator().manual_seed(7)
    cases = [((64, 64), 5), ((48, 96), 5), ((96, 48), 5), ((33, 70), 5), ((1, 16), 5),
             ((128, 32), 5), ((40, 40), 0), ((40, 24), 1), ((24, 40), 3)]
    out = {}
    for i, (shape, steps) in enumerate(cases):
        x = torch.randn(shape, generator=gen) * 1e-3 * 1.95
        out[f"in{i}"] = _to_np(x)
        out[f"steps{i}"] = np.int64(steps)
        out[f"out{i}"] = _to_np(ref.zeropower_via_newtonschulz5(x, steps=steps))
    z = torch.zeros(16, 16)
    out["in_zero"] = _to_np(z)
    out["out_zero"] = _to_np(ref.zeropower_via_newtonschulz5(z))
    inf = torch.ones(8, 12)
    inf[3, 4] = float("inf")
    out["in_inf"] = _to_np(inf)
    out["out_inf"] = _to_np(ref.zeropower_via_newtonschulz5(inf))
    out["n_cases"] = np.int64(len(cases))
    return out


def _clip_cases() -> dict:
    """Gradient sets through torch.nn.utils.clip_grad_norm_(max_norm=1.0)."""
    out = {}
    shapes = [(64, 33), (1000,), (7,), (48, 96), (3, 5)]
    kinds = [("bf16", [torch.bfloat16] * 5, 3.0), ("fp32", [torch.float32] * 5, 3.0),
             ("mixed", [torch.float32, torch.bfloat16] * 2 + [torch.bfloat16], 3.0),
             ("small_bf16", [torch.bfloat16] * 5, 1e-3), ("small_fp32", [torch.float32] * 5, 1e-3)]
    g = torch.Generator().manual_seed(13)
    out["cases"] = np.array([k for k, _, _ in kinds])
    for name, dts, scale in kinds:
        grads = [(torch.randn(s, generator=g) * scale).to(dt) for s, dt in zip(shapes, dts)]
        params = [torch.nn.Parameter(torch.zeros_like(t)) for t in grads]
        for p, t in zip(params, grads):
            p.grad = t.clone()
        total = torch.nn.utils.clip_grad_norm_(params, 1.0)
        out[f"{name}/total"] = np.array(float(total), np.float32)
        for i, (t, p) in enumerate(zip(grads, params)):
            out[f"{name}/in{i}"] = _to_np(t)
            out[f"{name}/out{i}"] = _to_np(p.grad)
            out[f"{name}/dtype{i}"] = np.array("bfloat16" if t.dtype == torch.bfloat16 else "float32")
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("OPENDM_REFERENCE"),
                    help="checkout of dexmal/opendm (default: $OPENDM_REFERENCE)")
    ap.add_argument("--only", choices=["clip"], default=None)
    args = ap.parse_args()
    np.savez_compressed(os.path.join(HERE, "clip_cases.npz"), **_clip_cases())
    if args.only == "clip":
        print("wrote clip_cases.npz to", HERE)
        return
    if not args.reference:
        ap.error("the reference fixtures need --reference PATH (or OPENDM_REFERENCE)")
    sys.path.insert(0, args.reference)
    from opendm.optimizer import muon_adamw as ref  # noqa: E402

    torch.set_num_threads(4)
    np.savez_compressed(os.path.join(HERE, "ns_cases.npz"), **_ns_cases(ref))
    np.savez_compressed(os.path.join(HERE, "step_fp32.npz"),
                        **_run_steps(ref, torch.float32, 3, nesterov=True, weight_decay=0.01,
                                     absent={1: "layers_1_odd_weight"}))
    layout: dict = {}
    np.savez_compressed(os.path.join(HERE, "step_bf16.npz"),
                        **_run_steps(ref, torch.bfloat16, 3, nesterov=True, weight_decay=0.01,
                                     layout_out=layout))
    with open(os.path.join(HERE, "state_layout.json"), "w") as f:
        json.dump(layout, f, indent=1, sort_keys=True)
    np.savez_compressed(os.path.join(HERE, "step_nonesterov.npz"),
                        **_run_steps(ref, torch.float32, 2, nesterov=False, weight_decay=0.0))
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
