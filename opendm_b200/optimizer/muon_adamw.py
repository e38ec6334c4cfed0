"""Drop-in B200 MuonAdamW: Muon for marked 2-D matrices, AdamW for the rest.

Same public surface as the reference ``opendm/optimizer/muon_adamw.py``
(dexmal/opendm): ``MuonAdamW(model, *, lr, betas, eps, weight_decay,
muon_momentum, muon_nesterov, muon_ns_steps, muon_lr_scale,
muon_moonlight_coefficient)``, param groups ``[AdamW, Muon]`` with the same
keys, ``state_dict``/``load_state_dict`` with the same per-parameter state
(``step`` 0-d fp32 tensor, ``exp_avg``, ``exp_avg_sq``) and the legacy forms,
``mark_muon_parameters``, ``is_default_muon_parameter``,
``zeropower_via_newtonschulz5`` and ``MuonShardPlan``. Parameters marked by
either library are interchangeable (same attribute names).

The arithmetic runs in the sm_100a kernels of ``libopendm_muon.so`` through
``opendm_b200.engine``; there is no CPU path. Optional keyword arguments
(defaults reproduce the reference):

* ``precision``: Newton-Schulz operand type, fp32 accumulation throughout.
  "fp16" (default): operands in fp16, each stored matrix scaled by a power
  of two to stay in fp16's range; the same 11-bit significand as tf32 at
  twice the tensor-core rate. "tf32": operands rounded to tf32, the same
  accuracy at half the rate. "bf16": ~1e-2 relative update error (opt-in).
  "parity": each fp16 operand split into a hi and a lo half and every
  product taken as hi*hi + hi*lo + lo*hi (~22-bit operands, 3x the tensor
  work): within ~1e-5 of the fp32 reference even on rank-deficient inputs,
  where the 11-bit types amplify rounding in the null space past the bar.
* ``ns_algo``: "auto" (default: per shape, the form with fewer executed
  FLOPs), "standard" (the reference's iteration on X) or "gram" (the
  iteration on the m x m gram matrix X X^T, applied to X every three
  iterations; about 1.7x fewer FLOPs for n >= 1.5 m, same accuracy).
* ``scale_mode``: "reference" (lr * lr_scale * coefficient * sqrt(max(r, c)))
  or "shape" (lr * lr_scale * max(1, r / c) ** 0.5).
* ``sharding``: "auto" (default: with world size > 1 and replicated
  parameters, each matrix is orthogonalised by one owner rank, chosen by
  FLOP-balanced LPT, and updated parameters are all-gathered) or "off"
  (every rank runs every matrix, as the reference does).
* ``state_sharding``: False (default: every rank keeps every momentum buffer
  current, so ``state_dict()`` on any rank equals the reference's) or True
  (momentum is advanced only by the owner; call ``consolidate_state_dict()``
  on all ranks before saving from one rank).
* ``process_group``: group for the sharded path (default: the world).
* ``allgather_waves``: with sharding, each rank's matrices are processed in
  this many waves of decreasing size; the all-gather of a wave overlaps the
  Newton-Schulz of the next (default on CUDA with at least 6 matrices per
  rank: 4 at 8 or more ranks carrying >= 16 dense TFLOP each, else 3;
  1 otherwise).
* ``allgather_wave_ratio``: each wave's share of a rank's Newton-Schulz
  FLOPs relative to the wave before (default 0.7: decreasing waves; 1.0:
  equal waves).
* ``comm_sms``: SMs the Newton-Schulz launches leave free while an NCCL
  all-gather overlaps them, and the CTA limit of the optimizer's own NCCL
  group for that all-gather (default 32).
* ``fsdp_owner_ns``: True (default): a matrix split into FSDP flat shards
  over several ranks is orthogonalised once, by one owner among its active
  ranks (FLOP-balanced), instead of by every active rank as in the reference
  (``:400-414``): the fp32 direction shards go to the owner in one
  all-to-all, the update shards (in the parameter dtype) come back in a
  second. Same arithmetic; False restores the reference's gather-everywhere.
* ``max_grad_norm``: None (default) or a float: clip the gradients at the
  start of every ``step()`` as ``torch.nn.utils.clip_grad_norm_`` does (the
  reference's trainer clips at 1.0 before each step, ``trainer.py:213``),
  fused: one norm pass, and the coefficient is applied by the momentum and
  AdamW kernels as they read the gradients (set the trainer's own
  ``max_grad_norm`` to 0 when using it). ``clip_grad_norm_()`` does the same
  on request; ``last_grad_norm`` holds the total norm of the last clip. With
  Muon matrices in FSDP shards ``step()`` refuses ``max_grad_norm``: the norm
  must then be reduced across ranks, which FSDP's own ``clip_grad_norm_`` does.
* ``allgather``: "nccl" (default) or "p2p": the flat parameter buckets live
  in peer-mapped memory and each rank pulls its peers' buckets with
  copy-engine memcpys ordered by cross-GPU flags (``opendm_b200.p2p``), so
  the Newton-Schulz keeps every SM.
* ``adamw_sharding``: False (default: every rank runs the whole AdamW group,
  as the reference does) or True (needs ``state_sharding=True`` and AdamW
  parameters replicated on every rank, which the first step checks): the
  AdamW parameters are split into equal contiguous element ranges, one per
  rank; each rank updates its range and the ranges are all-gathered while
  the Muon group's Newton-Schulz runs. ``consolidate_state_dict()`` brings
  the AdamW moments together too.
"""

from __future__ import annotations

import math
from collections.abc import Callable
from dataclasses import dataclass

import torch
import torch.distributed as dist

from .. import trace
from ..engine import AdamItem, CudaMuonEngine, MatrixItem, effective_lr
from ..sharding import FlatAdamShards, FlatParamBuckets, assign_owners, assign_waves

_MUON_SHAPE = "_opendm_muon_shape"
_MUON_NAME = "_opendm_muon_name"


@dataclass(frozen=True)
class MuonShardPlan:
    """How one Muon matrix is laid out over the ranks (reference :15-23).

    kind: "local" (single process, whole matrix), "empty" (no elements here),
    "owner_only" (one rank holds the whole matrix), "partial" (the matrix is
    split into flat shards over several ranks) or "replicated" (every rank
    holds the whole matrix).
    """

    kind: str
    full_numel: int
    local_numel: int
    sizes: tuple[int, ...]
    active_ranks: tuple[int, ...]
    local_offset: int
    process_group: object | None = None


def _as_matrix(t: torch.Tensor, shape) -> torch.Tensor:
    """`t` as the [rows, cols] matrix `shape`: itself when it has that shape
    already (a view costs microseconds per call, and most parameters need
    none), else a view (flat FSDP storage of a whole matrix)."""
    return t if t.shape == shape else t.view(shape)


def _dist_ready() -> bool:
    return dist.is_available() and dist.is_initialized()


def _normalize_parameter_name(name: str) -> str:
    """Strip wrapper prefixes (DDP ``module.``, FSDP ``_fsdp_wrapped_module.``,
    torch.compile ``_orig_mod.``) repeatedly (reference :30-38)."""
    prefixes = ("module.", "_fsdp_wrapped_module.", "_orig_mod.")
    changed = True
    while changed:
        changed = False
        for prefix in prefixes:
            if name.startswith(prefix):
                name = name[len(prefix):]
                changed = True
                break
    return name


_EXCLUDED_MARKERS = ("embed_tokens", "embedding", "layernorm.weight", "_norm.weight", ".norm.weight", ".norm.")


def is_default_muon_parameter(name: str, param: torch.nn.Parameter) -> bool:
    """Default Muon selection (reference :41-65): trainable 2-D ``.weight``
    matrices inside the action expert's ``.layers.``, excluding embeddings and
    norms."""
    if not param.requires_grad or param.ndim != 2:
        return False
    n = _normalize_parameter_name(name)
    in_expert = n.startswith("model.action_expert.") or n.startswith("action_expert.") or \
        ".model.action_expert." in n
    if not in_expert:
        return False
    low = n.lower()
    if ".layers." not in low or not low.endswith(".weight"):
        return False
    return not any(m in low for m in _EXCLUDED_MARKERS)


def mark_muon_parameters(model: torch.nn.Module,
                         predicate: Callable[[str, torch.nn.Parameter], bool] | None = None) -> list[str]:
    """Tag selected parameters with their pre-sharding 2-D shape and name
    (reference :68-98). Must run before FSDP flattens the parameters."""
    predicate = predicate or is_default_muon_parameter
    selected: list[str] = []
    seen: set[int] = set()
    for name, param in model.named_parameters():
        if id(param) in seen:
            continue
        seen.add(id(param))
        for attr in (_MUON_SHAPE, _MUON_NAME):
            if hasattr(param, attr):
                delattr(param, attr)
        if not predicate(name, param):
            continue
        if param.ndim != 2:
            raise RuntimeError(f"Muon parameter {name} must be 2D, got shape {tuple(param.shape)}.")
        setattr(param, _MUON_SHAPE, (int(param.shape[0]), int(param.shape[1])))
        setattr(param, _MUON_NAME, name)
        selected.append(name)
    if not selected:
        raise RuntimeError("MuonAdamW selected 0 parameters.")
    return selected


_ENGINES: dict[tuple, CudaMuonEngine] = {}


def _engine_for(device: torch.device, precision: str, ns_algo: str = "auto") -> CudaMuonEngine:
    if device.type != "cuda":
        raise RuntimeError("opendm_b200 runs on CUDA (sm_100) tensors only; got a tensor on " + str(device))
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, precision, ns_algo)
    if key not in _ENGINES:
        _ENGINES[key] = CudaMuonEngine(torch.device("cuda", idx), precision, ns_algo)
    return _ENGINES[key]


def zeropower_via_newtonschulz5(matrix: torch.Tensor, steps: int = 5, eps: float = 1e-7, *,
                                precision: str = "fp16", ns_algo: str = "auto") -> torch.Tensor:
    """Quintic Newton-Schulz orthogonalisation on the GPU (reference :101-128).

    Returns fp32 with the input's shape; a zero or non-finite input gives
    zeros. Raises ``ValueError`` for non-2-D input and ``RuntimeError`` for
    tensors that are not on an sm_100 device.
    """
    if matrix.ndim != 2:
        raise ValueError("Muon orthogonalization expects a 2D tensor.")
    engine = _engine_for(matrix.device, precision, ns_algo)
    with torch.cuda.device(matrix.device):
        return engine.orthogonalize(matrix.detach(), steps=max(int(steps), 0), eps=eps)


class MuonAdamW(torch.optim.Optimizer):
    """One optimizer with an AdamW group and a Muon group (reference :178-238)."""

    def __init__(self, model: torch.nn.Module, *, lr: float, betas: tuple[float, float], eps: float,
                 weight_decay: float, muon_momentum: float = 0.95, muon_nesterov: bool = True,
                 muon_ns_steps: int = 5, muon_lr_scale: float = 1.0, muon_moonlight_coefficient: float = 0.2,
                 precision: str = "fp16", scale_mode: str = "reference", sharding: str = "auto",
                 state_sharding: bool = False, process_group=None, ns_algo: str = "auto",
                 allgather_waves: int | None = None, allgather_wave_ratio: float = 0.7, comm_sms: int = 32,
                 allgather: str = "nccl",
                 fsdp_owner_ns: bool = True, max_grad_norm: float | None = None, adamw_sharding: bool = False,
                 _engine=None) -> None:
        adamw_params, muon_params, muon_shapes, muon_names = [], [], [], []
        for param in model.parameters():
            if not param.requires_grad:
                continue
            shape = getattr(param, _MUON_SHAPE, None)
            if shape is None:
                adamw_params.append(param)
            else:
                muon_params.append(param)
                muon_shapes.append(tuple(int(d) for d in shape))
                muon_names.append(getattr(param, _MUON_NAME, None))
        if not muon_params:
            raise RuntimeError("MuonAdamW metadata is missing; mark parameters before FSDP wrapping.")
        if sharding not in ("auto", "off"):
            raise ValueError(f"sharding must be 'auto' or 'off', got {sharding!r}")
        if precision not in ("tf32", "fp16", "bf16", "parity"):
            raise ValueError(f"precision must be 'tf32', 'fp16', 'bf16' or 'parity', got {precision!r}")
        if ns_algo not in ("auto", "standard", "gram"):
            raise ValueError(f"ns_algo must be 'auto', 'standard' or 'gram', got {ns_algo!r}")
        effective_lr(1.0, 1.0, 1.0, (1, 1), scale_mode)  # validates scale_mode
        groups = [
            {"params": adamw_params, "use_muon": False},
            {"params": muon_params, "use_muon": True, "muon_shapes": muon_shapes, "muon_names": muon_names},
        ]
        defaults = {
            "lr": lr, "betas": betas, "eps": eps, "weight_decay": weight_decay, "use_muon": False,
            "muon_momentum": muon_momentum, "muon_nesterov": muon_nesterov, "muon_ns_steps": muon_ns_steps,
            "muon_lr_scale": muon_lr_scale, "muon_moonlight_coefficient": muon_moonlight_coefficient,
        }
        super().__init__(groups, defaults)
        self._muon_shard_plan_cache: dict[int, list[MuonShardPlan]] = {}
        self._normalize_param_groups()
        self.precision = precision
        self.ns_algo = ns_algo
        self.scale_mode = scale_mode
        self.sharding = sharding
        self.state_sharding = bool(state_sharding)
        self.process_group = process_group
        self._engine = _engine
        self._host_steps: dict = {}
        self._owners: dict[int, list[int]] = {}
        self._buckets: dict[int, FlatParamBuckets] = {}
        self._waves: dict[int, list[int]] = {}
        self._flag_group = None  # host (gloo) group for the per-step activity flag
        self._ag_group = None  # NCCL group of the parameter all-gather (CTA-limited)
        if allgather_waves is not None and int(allgather_waves) < 1:
            raise ValueError("allgather_waves must be >= 1")
        if not float(allgather_wave_ratio) > 0:
            raise ValueError("allgather_wave_ratio must be > 0")
        if allgather not in ("nccl", "p2p"):
            raise ValueError(f"allgather must be 'nccl' or 'p2p', got {allgather!r}")
        self.allgather = allgather
        self.fsdp_owner_ns = bool(fsdp_owner_ns)
        if adamw_sharding and not self.state_sharding:
            raise ValueError("adamw_sharding needs state_sharding=True (each rank keeps only its range of the "
                             "AdamW moments current)")
        self.adamw_sharding = bool(adamw_sharding)
        self._adam_shards: dict[int, FlatAdamShards | None] = {}
        self._adam_pending: list[FlatAdamShards] = []  # ranges updated this step, all-gather not yet queued
        self._adam_handles: list = []
        self.max_grad_norm = None if max_grad_norm is None else float(max_grad_norm)
        self._pending_clip: torch.Tensor | None = None  # [total, coefficient] for the next step
        self.last_grad_norm: torch.Tensor | None = None
        self.allgather_waves = allgather_waves
        self.allgather_wave_ratio = float(allgather_wave_ratio)
        self.comm_sms = max(int(comm_sms), 0)

    # ---------------------------------------------------------------- groups
    def _normalize_param_groups(self) -> None:
        """Fill default keys and normalise Muon metadata, accepting the legacy
        ``muon_matrix_shapes`` / ``muon_param_infos`` forms (reference :240-276)."""
        for group in self.param_groups:
            for key, value in self.defaults.items():
                group.setdefault(key, value)
            if not group.get("use_muon", False):
                continue
            shapes = group.get("muon_shapes") or group.pop("muon_matrix_shapes", None)
            names = group.get("muon_names")
            infos = group.pop("muon_param_infos", None)
            if shapes is None and infos is not None:
                shapes = [self._info_shape(info) for info in infos]
            if names is None and infos is not None:
                names = [info.get("name") if isinstance(info, dict) else getattr(info, "name", None)
                         for info in infos]
            if shapes is None or len(shapes) != len(group["params"]):
                raise RuntimeError("Muon parameter metadata does not match parameters.")
            group["muon_shapes"] = [tuple(int(d) for d in s) for s in shapes]
            names = list(names or [None] * len(shapes))
            if len(names) != len(shapes):
                raise RuntimeError("Muon parameter names do not match parameters.")
            group["muon_names"] = names

    @staticmethod
    def _info_shape(info):
        if isinstance(info, dict):
            return info["matrix_shape"]
        if hasattr(info, "matrix_shape"):
            return info.matrix_shape
        return info[1]

    @staticmethod
    def _state_for_param(param: torch.Tensor, state: dict) -> dict:
        """Per-parameter state in the reference layout (:279-306): legacy
        ``momentum_buffer`` becomes ``exp_avg``; ``step`` is a 0-d fp32 tensor;
        ``exp_avg``/``exp_avg_sq`` are fp32 on the parameter's device."""
        if "momentum_buffer" in state:
            state.setdefault("exp_avg", state.pop("momentum_buffer"))
        step, m, v = state.get("step"), state.get("exp_avg"), state.get("exp_avg_sq")
        if (m is not None and v is not None and torch.is_tensor(step) and step.ndim == 0
                and step.dtype is torch.float32 and m.dtype is torch.float32 and v.dtype is torch.float32):
            dev = param.device
            if step.device == dev and m.device == dev and v.device == dev:
                return state  # already in the layout below (every step after the first)
        if step is None:
            state["step"] = torch.zeros((), dtype=torch.float32, device=param.device)
        elif not torch.is_tensor(step):
            state["step"] = torch.tensor(float(step), dtype=torch.float32, device=param.device)
        else:
            if step.numel() != 1:
                raise RuntimeError("Optimizer step state must contain one value.")
            state["step"] = step.detach().to(device=param.device, dtype=torch.float32).reshape(())
        for key in ("exp_avg", "exp_avg_sq"):
            value = state.get(key)
            if value is None:
                state[key] = torch.zeros_like(param, dtype=torch.float32, memory_format=torch.preserve_format)
            elif value.dtype != torch.float32 or value.device != param.device:
                state[key] = value.to(device=param.device, dtype=torch.float32)
        return state

    def load_state_dict(self, state_dict: dict) -> None:
        """Load current or legacy OpenDM optimizer state (reference :308-317)."""
        super().load_state_dict(state_dict)
        self._normalize_param_groups()
        for group in self.param_groups:
            for param in group["params"]:
                state = self.state.get(param)
                if state:
                    self._state_for_param(param, state)
        self._muon_shard_plan_cache.clear()
        self._host_steps.clear()

    # ----------------------------------------------------------------- step
    def _get_engine(self, device: torch.device):
        if self._engine is None:
            self._engine = _engine_for(device, self.precision, self.ns_algo)
        return self._engine

    def _grads_for_clip(self) -> list[torch.Tensor]:
        return [p.grad for g in self.param_groups for p in g["params"] if p.grad is not None]

    @torch.no_grad()
    def clip_grad_norm_(self, max_norm: float, norm_type: float = 2.0, error_if_nonfinite: bool = False,
                        foreach: bool | None = None) -> torch.Tensor:
        """``torch.nn.utils.clip_grad_norm_`` over this optimizer's parameters,
        fused with the next ``step()``: the total norm and the coefficient
        min(max_norm / (total + 1e-6), 1) are computed now, on the device,
        with torch's arithmetic (norm type 2); the next ``step()`` scales every
        gradient by the coefficient as its kernels read it, so ``p.grad``
        keeps its unclipped values until then. Returns the total norm (a 0-d
        tensor, bf16 when every gradient is bf16, as torch's). Other norm
        types, or parameters split over ranks (FSDP, whose own
        ``clip_grad_norm_`` reduces across ranks), run torch's function."""
        grads = self._grads_for_clip()
        if not grads:
            return torch.tensor(0.0)
        fused = float(norm_type) == 2.0 and grads[0].device.type == "cuda" and not self._split_over_ranks()
        if not fused:
            params = [p for g in self.param_groups for p in g["params"]]
            return torch.nn.utils.clip_grad_norm_(params, max_norm, norm_type, error_if_nonfinite, foreach)
        engine = self._get_engine(grads[0].device)
        out = engine.clip_grad_norm(grads, float(max_norm))
        res_dtype = torch.bfloat16 if all(g.dtype == torch.bfloat16 for g in grads) else torch.float32
        total = out[0].to(res_dtype)
        if error_if_nonfinite and not torch.isfinite(total).item():
            raise RuntimeError(f"The total norm of order {float(norm_type)} for gradients from `parameters` is "
                               "non-finite, so it cannot be clipped. To disable this error and scale the "
                               "gradients by the non-finite norm anyway, set `error_if_nonfinite=False`")
        self._pending_clip = out
        self.last_grad_norm = total
        return total

    def _split_over_ranks(self) -> bool:
        """True when some Muon matrix is split into shards over ranks (FSDP)."""
        return any(pl.kind not in ("local", "replicated", "empty")
                   for g in self.param_groups if g.get("use_muon", False) for pl in self._get_muon_shard_plans(g))

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        if self.max_grad_norm is not None and self._pending_clip is None:
            if self._split_over_ranks():
                raise RuntimeError("max_grad_norm needs parameters replicated on every rank; with FSDP shards "
                                   "clip with FSDP's clip_grad_norm_ (the trainer's max_grad_norm), which "
                                   "reduces the norm across ranks.")
            self.clip_grad_norm_(self.max_grad_norm)
        pending, self._pending_clip = self._pending_clip, None
        engine = self._engine if pending is not None else None
        if engine is not None:
            engine.grad_scale = pending[1:2]
        try:
            with trace.nvtx("step"):
                self._step_groups()
        finally:
            if engine is not None:
                engine.grad_scale = None
        return loss

    def _step_groups(self) -> None:
        # Muon groups first, then AdamW: the groups update disjoint parameters,
        # so the order changes no result, and an AdamW host-to-device table
        # copy (only when its parameters' step counts differ) then comes last,
        # where waiting behind other host-to-device transfers (e.g. the next
        # batch's upload) delays nothing after it.
        # A sharded AdamW group goes first instead, and the all-gather of its
        # ranges is queued right after the first Muon wave's (_flush_adam_sync):
        # it then overlaps the Newton-Schulz of wave 1 on, which leaves SMs
        # free for collectives. Issued earlier it would hold SMs that wave 0's
        # persistent CTAs wait for.
        adam = [g for g in self.param_groups if not g.get("use_muon", False)]
        sharded = [g for g in adam if self._adam_shards_for(g) is not None]
        self._adam_handles = []
        self._adam_pending = []
        try:
            for group in sharded:
                self._adamw_step(group)
                self._adam_pending.append(self._adam_shards[id(group)])
            for group in self.param_groups:
                if group.get("use_muon", False):
                    self._muon_step(group)
            self._flush_adam_sync()
            for group in adam:
                if not any(group is g for g in sharded):
                    self._adamw_step(group)
            for h in self._adam_handles:
                h.wait()
        finally:
            self._adam_pending, self._adam_handles = [], []

    def _flush_adam_sync(self) -> None:
        """Queue the all-gather of the sharded AdamW ranges updated this step
        (once; every rank reaches it at the same point of the step)."""
        pending, self._adam_pending = self._adam_pending, []
        for shards in pending:
            device = shards.buffers[0][0].device
            with trace.nvtx("adamw_allgather"):
                self._adam_handles += shards.sync(async_op=device.type == "cuda",
                                                  group=self._allgather_group(device))

    def _host_step(self, param, state) -> float:
        hs = self._host_steps.get(param)
        if hs is None:
            hs = float(state["step"].item())
        return hs

    def _adamw_step(self, group: dict) -> None:
        """AdamW over the group (reference :333-343); with AdamW sharding,
        over this rank's ranges only (the caller queues the all-gather of the
        ranges, which every rank joins, with or without gradients)."""
        shards = self._adam_shards_for(group)
        params = list(group["params"])
        pieces: dict[int, list[tuple[int, int]]] | None = None
        if shards is not None:
            pieces = {}
            for i, start, length in shards.owned(params):
                pieces.setdefault(i, []).append((start, length))
        items, step_tensors = [], []
        for index, param in enumerate(params):
            grad = param.grad
            if grad is None:
                continue
            if grad.is_sparse:
                raise RuntimeError("MuonAdamW does not support sparse gradients.")
            state = self._state_for_param(param, self.state[param])
            hs = self._host_step(param, state) + 1.0
            self._host_steps[param] = hs
            step_tensors.append(state["step"])
            if pieces is None:
                items.append(AdamItem(param.data, grad.detach(), state["exp_avg"], state["exp_avg_sq"], hs))
                continue
            if grad.numel() != param.numel():
                raise RuntimeError("AdamW gradient shape mismatch.")
            for key in ("exp_avg", "exp_avg_sq"):  # updated in place through flat views
                if not state[key].is_contiguous():
                    state[key] = state[key].contiguous()
            flat = [t.reshape(-1) for t in (param.data, grad.detach(), state["exp_avg"], state["exp_avg_sq"])]
            for start, length in pieces.get(index, ()):
                items.append(AdamItem(*(t[start:start + length] for t in flat), hs))
        if step_tensors:
            torch._foreach_add_(step_tensors, 1.0)
        if items:
            beta1, beta2 = group["betas"]
            self._get_engine(items[0].param.device).adamw(
                items, lr=float(group["lr"]), beta1=float(beta1), beta2=float(beta2), eps=float(group["eps"]),
                weight_decay=float(group.get("weight_decay", 0.0) or 0.0))

    def _adam_shards_for(self, group: dict) -> FlatAdamShards | None:
        """The group's flat AdamW ranges when AdamW sharding applies: on
        first use (collective, on every rank) the parameters are checked to
        be replicated (same sizes and the same float64 checksum everywhere)
        and re-pointed into the flat buffers."""
        key = id(group)
        if key in self._adam_shards:
            return self._adam_shards[key]
        world, rank = self._world()
        params = list(group["params"])
        shards = None
        if self.adamw_sharding and world > 1 and self.sharding != "off" and params:
            for g in self.param_groups:  # a model in FSDP shards has non-replicated Muon plans
                if g.get("use_muon", False) and g["params"] and \
                        any(p.kind != "replicated" for p in self._get_muon_shard_plans(g)):
                    raise RuntimeError("adamw_sharding needs replicated parameters (DDP); the Muon matrices "
                                       "are sharded here (FSDP?).")
            device = self._device_for_params(params)
            sizes = torch.tensor([float(p.numel()) for p in params], dtype=torch.float64, device=device)
            sums = torch.stack([p.detach().sum(dtype=torch.float64) for p in params])
            sig = torch.stack([sizes, sums]).view(torch.int64)  # compared bit for bit
            everyone = [torch.empty_like(sig) for _ in range(world)]
            dist.all_gather(everyone, sig, group=self.process_group)
            if any(not torch.equal(e, everyone[0]) for e in everyone[1:]):
                raise RuntimeError("adamw_sharding needs the AdamW parameters replicated on every rank "
                                   "(DDP); they differ between ranks (FSDP shards?).")
            shards = FlatAdamShards(params, world, rank, self.process_group)
        self._adam_shards[key] = shards
        return shards

    @staticmethod
    def _device_for_params(params: list[torch.Tensor]) -> torch.device:
        if params:
            return params[0].device
        return torch.device("cuda" if torch.cuda.is_available() else "cpu")

    def _host_flag_group(self):
        """A gloo group over the ranks of ``process_group``, created on first
        use (every rank reaches the first Muon step together)."""
        if self._flag_group is None:
            pg = self.process_group
            if dist.get_backend(pg) == "gloo":
                self._flag_group = (pg,)
            else:
                ranks = dist.get_process_group_ranks(pg) if pg is not None else None
                self._flag_group = (dist.new_group(ranks=ranks, backend="gloo",
                                                   use_local_synchronization=pg is not None),)
        return self._flag_group[0]

    def _muon_group_is_active(self, params: list[torch.Tensor]) -> bool:
        """True when any rank has a Muon gradient (reference :350-360).

        The reference reduces a device flag and reads it back, which waits
        for every kernel queued so far. The flag is a host fact, so here it
        is reduced over a gloo group on the host: same answer, and the host
        keeps queueing work while the GPU runs the previous step."""
        local_active = any(p.grad is not None for p in params)
        if not _dist_ready():
            return local_active
        flag = torch.tensor([int(local_active)], dtype=torch.int32)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=self._host_flag_group())
        return bool(flag[0])

    def _world(self) -> tuple[int, int]:
        if not _dist_ready():
            return 1, 0
        return dist.get_world_size(self.process_group), dist.get_rank(self.process_group)

    def _sharded(self, group: dict, plans: list[MuonShardPlan]) -> bool:
        world, _ = self._world()
        if self.sharding == "off" or world <= 1:
            return False
        return all(p.kind == "replicated" for p in plans) and \
            all(p.is_contiguous() for p in group["params"])

    def _n_waves(self, shapes: list, world: int, device: torch.device, steps: int) -> int:
        """Waves per step: one per ~1/3-1/4 of a rank's Newton-Schulz work.
        Every wave adds a full set of Newton-Schulz launches (fixed fill and
        drain time), so a fourth wave pays off only when each rank carries a
        large share (>= 16 dense TFLOP), as at 8 ranks on benchmark config 4."""
        if self.allgather_waves is not None:
            return int(self.allgather_waves)
        if device.type != "cuda" or len(shapes) < 6 * world:
            return 1
        from ..sharding import ns_cost

        per_rank = sum(ns_cost(s, steps) for s in shapes) / world
        return 4 if world >= 8 and per_rank >= 16e12 else 3

    def _owners_for(self, group: dict) -> list[int]:
        key = id(group)
        owners = self._owners.get(key)
        if owners is None or len(owners) != len(group["params"]):
            world, rank = self._world()
            shapes, steps = group["muon_shapes"], int(group["muon_ns_steps"])
            owners = assign_owners(shapes, world, steps)
            n_waves = self._n_waves(shapes, world, self._device_for_params(group["params"]), steps)
            waves = assign_waves(shapes, owners, world, n_waves, steps, self.allgather_wave_ratio)
            self._owners[key] = owners
            self._waves[key] = waves
            device = self._device_for_params(group["params"])
            if self._use_p2p(device):
                from ..p2p import P2PFlatBuckets

                engine = self._get_engine(device)
                self._buckets[key] = P2PFlatBuckets(list(group["params"]), owners, world, rank, self.process_group,
                                                    waves, engine._err)
            else:
                self._buckets[key] = FlatParamBuckets(list(group["params"]), owners, world, rank,
                                                      self.process_group, waves)
        return owners

    def _use_p2p(self, device: torch.device) -> bool:
        if self.allgather != "p2p":
            return False
        from .. import p2p

        if device.type != "cuda" or not p2p.available():
            raise RuntimeError("allgather='p2p' needs CUDA devices and torch symmetric memory")
        return True

    def _allgather_group(self, device: torch.device):
        """The group for the parameter all-gather: on CUDA with NCCL, a
        group of the same ranks whose kernels use at most ``comm_sms`` CTAs
        on a high-priority stream (created on first use, on every rank)."""
        pg = self.process_group
        if device.type != "cuda" or dist.get_backend(pg) != "nccl":
            return pg
        if self._ag_group is None:
            opts = dist.ProcessGroupNCCL.Options()
            opts.is_high_priority_stream = True
            if self.comm_sms > 0:
                opts.config.max_ctas = self.comm_sms
            ranks = dist.get_process_group_ranks(pg) if pg is not None else None
            self._ag_group = (dist.new_group(ranks=ranks, backend="nccl", pg_options=opts,
                                             use_local_synchronization=pg is not None),)
        return self._ag_group[0]

    def _muon_step(self, group: dict) -> None:
        if not self._muon_group_is_active(group["params"]):
            return
        momentum = float(group["muon_momentum"])
        nesterov = bool(group["muon_nesterov"])
        lr = float(group["lr"])
        weight_decay = float(group.get("weight_decay", 0.0) or 0.0)
        wd_factor = (1.0 - lr * weight_decay) if weight_decay else 1.0
        ns_steps = max(int(group["muon_ns_steps"]), 0)
        plans = self._get_muon_shard_plans(group)
        sharded = self._sharded(group, plans)
        owners = self._owners_for(group) if sharded else None
        _, rank = self._world()

        waves = self._waves.get(id(group)) if sharded else None
        n_waves = (max(waves) + 1) if waves else 1
        owned = [[] for _ in range(n_waves)]
        others, partial, step_tensors = [], [], []
        partial_local: dict[int, tuple] = {}  # matrix index -> (param, grad, state, eff), local shards only
        lr_scale, moonlight = float(group["muon_lr_scale"]), float(group["muon_moonlight_coefficient"])
        eff_of: dict = {}  # per shape: the update scale depends on the shape alone within a step
        for index, (param, shape, plan) in enumerate(zip(group["params"], group["muon_shapes"], plans, strict=True)):
            if plan.local_numel == 0:
                continue
            grad = param.grad
            if grad is not None and grad.is_sparse:
                raise RuntimeError("MuonAdamW does not support sparse gradients.")
            if grad is not None and grad.numel() != param.numel():
                name = group["muon_names"][index] or index
                raise RuntimeError(f"Muon gradient shape mismatch for {name}.")
            state = self._state_for_param(param, self.state[param])
            step_tensors.append(state["step"])
            other = plan.kind != "partial" and owners is not None and owners[index] != rank
            if other and self.state_sharding:
                continue  # the owner advances this matrix's momentum; the all-gather brings the parameter
            if other:  # momentum only
                others.append(MatrixItem(_as_matrix(param.data, shape),
                                         _as_matrix(grad.detach(), shape) if grad is not None else None,
                                         _as_matrix(state["exp_avg"], shape)))
                continue
            eff = eff_of.get(shape)
            if eff is None:
                eff = eff_of[shape] = effective_lr(lr, lr_scale, moonlight, shape, self.scale_mode)
            if plan.kind == "partial":
                partial.append((param, grad, state, shape, plan, eff))
                partial_local[index] = (param, grad, state, eff)
                continue
            item = MatrixItem(_as_matrix(param.data, shape),
                              _as_matrix(grad.detach(), shape) if grad is not None else None,
                              _as_matrix(state["exp_avg"], shape), eff)
            owned[waves[index] if waves else 0].append(item)
        if step_tensors:
            torch._foreach_add_(step_tensors, 1.0)
        device = self._device_for_params(group["params"])
        engine = self._get_engine(device)
        if not sharded:
            engine.muon_matrices(owned[0], momentum=momentum, nesterov=nesterov, weight_decay_factor=wd_factor,
                                 ns_steps=ns_steps)
        else:
            # Wave w's all-gather runs on the collective's stream while wave
            # w + 1 is orthogonalised with `comm_sms` SMs left free for it.
            buckets = self._buckets[id(group)]
            p2p = hasattr(buckets, "wave_done")
            handles = []
            if p2p:
                # copy engines: every SM stays with the Newton-Schulz
                buckets.begin()
                for w in range(n_waves):
                    with trace.nvtx(f"wave{w}"):
                        engine.muon_matrices(owned[w], momentum=momentum, nesterov=nesterov,
                                             weight_decay_factor=wd_factor, ns_steps=ns_steps)
                        buckets.wave_done(w)
                    if w == 0:
                        self._flush_adam_sync()
            else:
                ag_group = self._allgather_group(device)
                overlap = device.type == "cuda" and n_waves > 1 and hasattr(engine, "sm_limit")
                total_sms = torch.cuda.get_device_properties(device).multi_processor_count if overlap else 0
                try:
                    for w in range(n_waves):
                        if overlap:
                            engine.sm_limit = max(total_sms - self.comm_sms, 2) if w > 0 else 0
                        with trace.nvtx(f"wave{w}"):
                            engine.muon_matrices(owned[w], momentum=momentum, nesterov=nesterov,
                                                 weight_decay_factor=wd_factor, ns_steps=ns_steps)
                            handles += buckets.sync(wave=w, async_op=device.type == "cuda", group=ag_group)
                        if w == 0:
                            self._flush_adam_sync()
                finally:
                    if overlap:
                        engine.sm_limit = 0
        engine.momentum_only(others, momentum=momentum, nesterov=nesterov)
        if self.fsdp_owner_ns and any(p.kind == "partial" for p in plans):
            self._partial_owner_ns(engine, group, plans, partial_local, momentum, nesterov, wd_factor, ns_steps)
        else:
            for param, grad, state, shape, plan, eff in partial:
                self._partial_update(engine, param, grad, state, shape, plan, eff, momentum, nesterov, wd_factor,
                                     ns_steps)
        if sharded:
            ev = engine._event_pair("allgather_wait") if getattr(engine, "profile_events", None) is not None \
                else None
            for h in handles:
                h.wait()
            if p2p:
                buckets.finish()
            if ev is not None:
                engine._event_end(ev)

    @staticmethod
    def _partial_owners(plans: list[MuonShardPlan], shapes, idx: list[int], steps: int) -> dict[int, int]:
        """Owner rank of each partial matrix: LPT by Newton-Schulz FLOPs over
        the matrix's active ranks (deterministic, identical on every rank)."""
        from ..sharding import ns_cost

        load: dict[int, float] = {}
        owners: dict[int, int] = {}
        for j in sorted(idx, key=lambda j: (-ns_cost(shapes[j], steps), j)):
            r = min(plans[j].active_ranks, key=lambda r: (load.get(r, 0.0), r))
            owners[j] = r
            load[r] = load.get(r, 0.0) + ns_cost(shapes[j], steps)
        return owners

    def _partial_owner_ns(self, engine, group: dict, plans: list[MuonShardPlan], local: dict, momentum: float,
                          nesterov: bool, wd_factor: float, ns_steps: int) -> None:
        """Owner-only Newton-Schulz for matrices split into flat shards over
        several ranks (the reference's `partial` plans, :400-414, orthogonalise
        the gathered matrix on every active rank). Every rank takes part in
        both exchanges, including ranks without a shard of some matrix."""
        world, rank = dist.get_world_size(), dist.get_rank()
        shapes = group["muon_shapes"]
        idx = [j for j, p in enumerate(plans) if p.kind == "partial"]
        owners = self._partial_owners(plans, shapes, idx, max(ns_steps, 1))
        params = group["params"]
        device = self._device_for_params(params)

        def pad4(n):  # fp32 elements, so every shard starts 16-byte aligned
            return (n + 3) // 4 * 4

        # 1. momentum on the local shards, straight into the send buffer, by owner
        send_sizes, items, offsets, cur = [0] * world, [], [], 0
        for d in range(world):
            for j in idx:
                n = plans[j].sizes[rank]
                if owners[j] != d or n == 0:
                    continue
                param, grad, state, _ = local[j]
                items.append((grad.detach() if grad is not None else None, state["exp_avg"].view(-1)))
                offsets.append(cur)
                cur += pad4(n)
                send_sizes[d] += pad4(n)
        recv_sizes = [sum(pad4(plans[j].sizes[s]) for j in idx if owners[j] == rank and plans[j].sizes[s] > 0)
                      for s in range(world)]
        send = torch.empty(max(cur, 1), dtype=torch.float32, device=device)
        recv = torch.empty(max(sum(recv_sizes), 1), dtype=torch.float32, device=device)
        engine.directions_into(items, send, offsets, momentum=momentum, nesterov=nesterov)
        dist.all_to_all_single(recv[:sum(recv_sizes)], send[:cur], recv_sizes, send_sizes)

        # 2. the owner assembles its matrices (shards in rank order) and orthogonalises them together
        mine = [j for j in idx if owners[j] == rank]
        src_off = [sum(recv_sizes[:s]) for s in range(world)]
        fulls = []
        for j in mine:
            full = torch.empty(plans[j].full_numel, dtype=torch.float32, device=device)
            pos = 0
            for s in range(world):
                n = plans[j].sizes[s]
                if n:
                    full[pos:pos + n].copy_(recv[src_off[s]:src_off[s] + n])
                    src_off[s] += pad4(n)
                    pos += n
            fulls.append(full.view(shapes[j]))
        updates = engine.orthogonalize_many(fulls, [params[j].dtype for j in mine], steps=ns_steps)

        # 3. update shards (parameter dtype) back to their ranks, as bytes
        def pad16(b):
            return (b + 15) // 16 * 16

        def shard_bytes(j, s):
            return plans[j].sizes[s] * params[j].element_size()

        send2_sizes = [sum(pad16(shard_bytes(j, s)) for j in mine if plans[j].sizes[s] > 0) for s in range(world)]
        recv2_sizes = [sum(pad16(shard_bytes(j, rank)) for j in idx if owners[j] == o and plans[j].sizes[rank] > 0)
                       for o in range(world)]
        send2 = torch.empty(max(sum(send2_sizes), 16), dtype=torch.uint8, device=device)
        recv2 = torch.empty(max(sum(recv2_sizes), 16), dtype=torch.uint8, device=device)
        pos = 0
        flat_u = [u.contiguous().view(-1) for u in updates]
        for s in range(world):
            for j, u in zip(mine, flat_u):
                n = plans[j].sizes[s]
                if n == 0:
                    continue
                off = sum(plans[j].sizes[:s])
                nb = shard_bytes(j, s)
                send2[pos:pos + nb].view(params[j].dtype).copy_(u[off:off + n])
                pos += pad16(nb)
        dist.all_to_all_single(recv2[:sum(recv2_sizes)], send2[:sum(send2_sizes)], recv2_sizes, send2_sizes)

        # 4. weight decay + update of the local shards
        upd, pos = [], 0
        for o in range(world):
            for j in idx:
                n = plans[j].sizes[rank]
                if owners[j] != o or n == 0:
                    continue
                param, _, _, eff = local[j]
                nb = shard_bytes(j, rank)
                upd.append((param.data.view(-1), recv2[pos:pos + nb].view(param.dtype), eff))
                pos += pad16(nb)
        engine.apply_update_flat(upd, wd_factor)

    def _partial_update(self, engine, param, grad, state, shape, plan, eff, momentum, nesterov, wd_factor,
                        ns_steps) -> None:
        """A matrix split into flat shards over several ranks (FSDP): gather
        the direction among the active ranks, orthogonalise, keep the local
        slice (reference :400-414)."""
        direction = engine.direction(grad.detach().reshape(-1) if grad is not None else None,
                                     state["exp_avg"].view(-1), momentum=momentum, nesterov=nesterov)
        full, offset = self._gather_matrix(direction, plan)
        if full.numel() == 0:
            return
        update = engine.orthogonalize(full.view(shape), steps=ns_steps).reshape(-1)
        local = update.narrow(0, offset, plan.local_numel).view_as(param)
        if wd_factor != 1.0:
            param.mul_(wd_factor)
        param.add_(local.to(param.dtype), alpha=-eff)

    # --------------------------------------------------------- shard plans
    @staticmethod
    def _plan_matches_group(group: dict, plans: list[MuonShardPlan]) -> bool:
        if len(plans) != len(group["params"]):
            return False
        world = dist.get_world_size() if _dist_ready() else 1
        return all(p.full_numel == math.prod(s) and p.local_numel == param.numel() and len(p.sizes) == world
                   for param, s, p in zip(group["params"], group["muon_shapes"], plans, strict=True))

    def _get_muon_shard_plans(self, group: dict) -> list[MuonShardPlan]:
        """Cached per-matrix layout plans (reference :430-441)."""
        key = id(group)
        plans = self._muon_shard_plan_cache.get(key)
        if plans is None or not self._plan_matches_group(group, plans):
            plans = self._build_muon_shard_plans(group)
            self._muon_shard_plan_cache[key] = plans
        return plans

    def _build_muon_shard_plans(self, group: dict) -> list[MuonShardPlan]:
        """Classify every matrix (reference :443-501). With a process group,
        the local sizes of all matrices are exchanged in one all_gather."""
        params, shapes = group["params"], group["muon_shapes"]
        for param, shape in zip(params, shapes, strict=True):
            full = math.prod(shape)
            if param.numel() > full:
                raise RuntimeError(f"Muon matrix {tuple(shape)} has only {full} elements, "
                                   f"but the local tensor has {param.numel()}.")
        if not _dist_ready():
            plans = []
            for param, shape in zip(params, shapes, strict=True):
                n, full = int(param.numel()), math.prod(shape)
                if n not in (0, full):
                    raise RuntimeError(f"Muon matrix {tuple(shape)} has {n} local elements, expected 0 or {full}.")
                plans.append(MuonShardPlan("empty" if n == 0 else "local", full, n, (n,), (0,) if n else (), 0))
            return plans
        world, rank = dist.get_world_size(), dist.get_rank()
        device = self._device_for_params(params)
        local = torch.tensor([int(p.numel()) for p in params], dtype=torch.long, device=device)
        gathered = [torch.zeros_like(local) for _ in range(world)]
        dist.all_gather(gathered, local)
        table = torch.stack(gathered).cpu().tolist()  # [world][n_params]
        plans = []
        for j, (param, shape) in enumerate(zip(params, shapes, strict=True)):
            full = math.prod(shape)
            sizes = tuple(int(table[r][j]) for r in range(world))
            active = tuple(r for r, s in enumerate(sizes) if s > 0)
            total = sum(sizes)
            pg = None
            if total == 0:
                kind = "empty"
            elif total == full:
                kind = "owner_only" if len(active) == 1 else "partial"
                if kind == "partial" and len(active) < world:
                    pg = dist.new_group(ranks=list(active))
            elif all(s == full for s in sizes):
                kind = "replicated"
            else:
                raise RuntimeError(f"Muon matrix {tuple(shape)} cannot be reconstructed from local shard sizes {sizes}.")
            plans.append(MuonShardPlan(kind, full, int(param.numel()), sizes, active, sum(sizes[:rank]), pg))
        return plans

    @staticmethod
    def _gather_matrix(local: torch.Tensor, plan: MuonShardPlan) -> tuple[torch.Tensor, int]:
        """Assemble the full direction of a matrix from its shards (reference :503-535)."""
        local = local.reshape(-1).contiguous()
        if local.numel() != plan.local_numel:
            raise RuntimeError("Muon local tensor no longer matches its shard plan.")
        if plan.kind == "empty":
            return local.new_empty(0), 0
        if plan.kind in {"local", "owner_only", "replicated"}:
            return local, 0
        if plan.kind != "partial":
            raise RuntimeError(f"Unknown Muon shard plan kind: {plan.kind}.")
        rank = dist.get_rank()
        if rank not in plan.active_ranks:
            return local.new_empty(0), plan.local_offset
        sizes = tuple(plan.sizes[r] for r in plan.active_ranks)
        padded = local.new_zeros(max(sizes))
        padded[: local.numel()] = local
        shards = [torch.empty_like(padded) for _ in sizes]
        dist.all_gather(shards, padded, group=plan.process_group)
        return torch.cat([s[:n] for s, n in zip(shards, sizes, strict=True)]), plan.local_offset

    # ----------------------------------------------------------- checkpoints
    def consolidate_state_dict(self) -> None:
        """With ``state_sharding=True``: bring every momentum buffer from its
        owner to all ranks, and with ``adamw_sharding`` every AdamW moment
        range from its rank (collective; call on every rank before saving)."""
        world, _ = self._world()
        if world <= 1 or not self.state_sharding:
            return
        for group in self.param_groups:
            if not group.get("use_muon", False):
                shards = self._adam_shards.get(id(group))
                if shards is None:
                    continue
                params = list(group["params"])
                for index, owner, start, length in shards.ranges(params):
                    state = self._state_for_param(params[index], self.state[params[index]])
                    src = dist.get_global_rank(self.process_group, owner) if self.process_group is not None \
                        else owner
                    for key in ("exp_avg", "exp_avg_sq"):
                        if not state[key].is_contiguous():
                            state[key] = state[key].contiguous()
                        dist.broadcast(state[key].view(-1)[start:start + length], src=src, group=self.process_group)
                continue
            owners = self._owners.get(id(group))
            if owners is None:
                continue
            for param, owner in zip(group["params"], owners):
                state = self._state_for_param(param, self.state[param])
                src = dist.get_global_rank(self.process_group, owner) if self.process_group is not None else owner
                dist.broadcast(state["exp_avg"], src=src, group=self.process_group)

    def check_device_errors(self) -> None:
        """Synchronise and raise if a kernel recorded a device error."""
        if self._engine is not None and hasattr(self._engine, "check_errors"):
            self._engine.check_errors(block=True)
