"""Device engine: drives the sm_100a kernels of libopendm_muon.so for one GPU.

The optimizer (``opendm_b200.optimizer.MuonAdamW``) hands the engine lists of
whole matrices it must update and the AdamW-group tensors. The engine

* groups matrices by (rows, cols, param dtype) into shape classes; each class
  owns one workspace holding the Newton-Schulz operands (X ping-pong, A', B',
  M, and for the gram form A, P A and Q) for all its matrices, stacked so one
  grouped launch covers every class; the class's Newton-Schulz form (iterate
  on X, or on the gram matrix) is the library's choice by executed FLOPs;
* caches one plan state (workspaces, tensor maps, tile schedules) per matrix
  set, e.g. per all-gather wave, while the parameters stay at the same
  addresses, and device copies of segment tables while their bytes repeat
  (the AdamW table's per-step step size and bias correction are written on
  the device), so a steady-state step at a constant learning rate copies
  nothing host to device (a new rate re-uploads the small update tables);
* launches (a) momentum + Frobenius scale (in fp16 mode with the operand
  written in the same pass, scaled by a power of two carried between steps),
  (b) the grouped tcgen05 Newton-Schulz launches (3 per iteration, plus one
  per gram segment) whose last epilogue writes U in the parameter dtype,
  (c) weight decay + the scaled update, and the fused AdamW kernel, all on
  the current CUDA stream.

There is no fallback: every entry point raises if the library is missing or
the tensors are not on an sm_100 device.
"""

from __future__ import annotations

import math
from ctypes import byref, c_float, c_int, c_void_p, sizeof
from dataclasses import dataclass

import torch

from . import _native as N
from . import trace

_DTYPE_CODE = {torch.bfloat16: N.MUON_BF16, torch.float32: N.MUON_F32}
PRECISIONS = {"tf32": N.MUON_TF32, "fp16": N.MUON_F16, "bf16": N.MUON_BF16, "parity": N.MUON_F16X3}
_F16_OPS = (N.MUON_F16, N.MUON_F16X3)  # fp16 storage: power-of-two scaled operands
# Newton-Schulz algorithm per shape class: "auto" (the library's choice by
# executed FLOPs), "standard" (iterate on X) or "gram" (iterate on X X^T).
NS_ALGOS = ("auto", "standard", "gram")
_OP_TORCH = {N.MUON_TF32: torch.float32, N.MUON_F16: torch.float16, N.MUON_BF16: torch.bfloat16,
             N.MUON_F16X3: torch.float16}


@dataclass
class MatrixItem:
    """One whole matrix this rank updates: param/exp_avg viewed as [rows, cols]."""

    param: torch.Tensor
    grad: torch.Tensor | None
    exp_avg: torch.Tensor
    eff: float = 0.0


@dataclass
class AdamItem:
    param: torch.Tensor
    grad: torch.Tensor
    exp_avg: torch.Tensor
    exp_avg_sq: torch.Tensor
    step: float  # step count after this step's increment


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPE_CODE[t.dtype]
    except KeyError:
        raise RuntimeError(f"unsupported dtype {t.dtype}: the kernels take bfloat16 or float32") from None


def _pad16(cols: int, dtype: torch.dtype) -> int:
    """Row length padded so a row is a multiple of 16 bytes."""
    per = 16 // torch.empty((), dtype=dtype).element_size()
    return (cols + per - 1) // per * per


def _stream_handle() -> c_void_p:
    return c_void_p(torch.cuda.current_stream().cuda_stream)


def _upload(raw: bytes, device: torch.device) -> torch.Tensor:
    host = torch.frombuffer(bytearray(raw), dtype=torch.uint8).pin_memory()
    return host.to(device, non_blocking=True)


class _TableCache:
    """Device copies of segment tables, reused while a table's bytes repeat
    (the parameters and workspaces stay put, and gradient buffers are
    usually reused), so a steady-state step issues no host-to-device copy
    that could queue behind unrelated transfers."""

    def __init__(self, device: torch.device, capacity: int = 64):
        self.device, self.capacity = device, capacity
        self._tables: dict[bytes, torch.Tensor] = {}

    def get(self, raw: bytes, key: bytes | None = None) -> torch.Tensor:
        """The device copy of `raw`, cached under `key` (default: `raw`)."""
        key = raw if key is None else key
        t = self._tables.pop(key, None)
        if t is None:
            t = _upload(raw, self.device)
            while len(self._tables) >= self.capacity:
                self._tables.pop(next(iter(self._tables)))
        self._tables[key] = t  # most recently used last
        t.record_stream(torch.cuda.current_stream(self.device))  # reused later by kernels on this stream
        return t


class _ClassState:
    """Workspace and buffers of one shape class."""

    def __init__(self, rows: int, cols: int, param_dtype: torch.dtype, count: int, op_dtype: int,
                 device: torch.device, steps: int, algo: str = "auto"):
        lib = N.lib()
        self.rows, self.cols, self.count, self.param_dtype = rows, cols, count, param_dtype
        if algo == "auto":
            code = int(lib.muon_ns_choose_algo(rows, cols, op_dtype, steps))
        else:
            code = {"standard": N.MUON_NS_STANDARD, "gram": N.MUON_NS_GRAM}[algo]
        nbytes = lib.muon_ns_class_workspace_bytes(rows, cols, count, op_dtype, code)
        self.workspace = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
        self.cls = N.NsClass()
        self.cls.rows, self.cls.cols, self.cls.count = rows, cols, count
        self.cls.algo = code
        N.check(lib.muon_ns_class_layout(byref(self.cls), c_void_p(self.workspace.data_ptr()), op_dtype),
                "muon_ns_class_layout")
        self.op_dtype = op_dtype
        self.es = 4 if op_dtype == N.MUON_TF32 else 2
        # split operands (MUON_F16X3) keep each matrix as a hi half and, lo_offset
        # elements further on, a lo half
        halves = 2 if op_dtype == N.MUON_F16X3 else 1
        self.lo_offset = rows * int(self.cls.ld_x) if halves == 2 else 0
        self.x_stride = halves * rows * int(self.cls.ld_x) * self.es  # bytes per matrix in x0
        # fp16 operand scale S0 of the first iteration: the Newton-Schulz input is
        # X0 * S0 (stored so by the orthogonalize paths; muon_momentum_f16 stores
        # d * p and hands the plan the factor to X0 * S0).
        self.x0_scale = float(lib.muon_ns_operand_scale(rows, cols, 0, op_dtype))

    def last_x_read(self, steps: int) -> int:
        """0 or 1: the X buffer (x0, x1) the last Newton-Schulz apply reads;
        the other one is free when U is written."""
        if int(self.cls.algo) == N.MUON_NS_GRAM:
            # gram segments alternate x0, x1
            return ((steps - 1) // int(N.lib().muon_ns_gram_segment(self.op_dtype))) % 2
        return (steps - 1) % 2

    def x0_view(self, slot: int, lo: bool = False) -> torch.Tensor:
        """The stored Newton-Schulz input of matrix `slot` as a [rows, cols]
        tensor (its lo half with ``lo`` for split operands)."""
        ld = int(self.cls.ld_x)
        off = ((int(self.cls.x0) - self.workspace.data_ptr() + slot * self.x_stride) // self.es
               + (self.lo_offset if lo else 0))
        return torch.empty(0, dtype=_OP_TORCH[self.op_dtype], device=self.workspace.device).set_(
            self.workspace.untyped_storage(), off, (self.rows, self.cols), (ld, 1))

    def x0_value(self, slot: int) -> torch.Tensor:
        """The stored input's value in fp32 (hi + lo for split operands)."""
        x = self.x0_view(slot).float()
        return x + self.x0_view(slot, lo=True).float() if self.lo_offset else x


class _PlanState:
    """Everything cached for one set of matrices: shape classes with their
    workspaces, the segment order and the plan."""

    def __init__(self):
        self.plans: list = []  # one library plan per group of up to PLAN_CLASSES classes
        self.classes: list[_ClassState] = []
        self.order: list[tuple[int, int]] = []  # item index -> (class index, slot)
        self.seg_order: list[int] = []
        self.scales = None
        # fp16: the per-matrix power of two of the stored operand, kept between
        # steps (0 until the first step), and the fix-up flags (muon_momentum_f16)
        self.pscale = None
        self.redo = None
        self.ns_launches = 0
        self.sm_limit = 0


class _F16Inputs:
    """pscale / scales / redo of a one-off muon_momentum_f16 call (no carried
    power of two: every matrix is written by the fix-up pass)."""

    def __init__(self, n: int, scales: torch.Tensor, device: torch.device):
        self.scales = scales
        self.pscale = torch.zeros(max(n, 1), dtype=torch.float32, device=device)
        self.redo = torch.zeros(max(n, 1), dtype=torch.int32, device=device)


class CudaMuonEngine:
    """Runs the Muon and AdamW kernels on one CUDA device."""

    MAX_PLANS = 16  # cached matrix sets (e.g. the waves of a sharded step)
    PLAN_CLASSES = 16  # shape classes one library plan takes (two problems per class in a 32-problem launch)

    def __init__(self, device: torch.device | str | int, precision: str = "fp16", ns_algo: str = "auto"):
        if precision not in PRECISIONS:
            raise ValueError(f"precision must be one of {sorted(PRECISIONS)}, got {precision!r}")
        if ns_algo not in NS_ALGOS:
            raise ValueError(f"ns_algo must be one of {NS_ALGOS}, got {ns_algo!r}")
        self.ns_algo = ns_algo
        self.device = torch.device(device) if not isinstance(device, int) else torch.device("cuda", device)
        if self.device.type != "cuda":
            raise RuntimeError("opendm_b200 runs on CUDA (sm_100) devices only; got " + str(self.device))
        self.precision = precision
        self.op_dtype = PRECISIONS[precision]
        self.lib = N.lib()
        idx = self.device.index if self.device.index is not None else torch.cuda.current_device()
        N.check(self.lib.muon_device_check(idx), "muon_device_check")
        self._plans: dict = {}  # matrix-set key -> _PlanState, least recently used first
        self._tables = _TableCache(self.device)
        self._adam_tables = _TableCache(self.device, capacity=8)  # per-step scalars rewritten in place
        # At most this many SMs per Newton-Schulz launch (0: all), leaving the
        # rest to a collective that overlaps it.
        self.sm_limit = 0
        self._err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._err_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._err_event = None
        self.kernel_launches = 0  # launches issued by this engine (for benchmarks)
        # Device float (or None): gradient-norm clipping coefficient that the
        # momentum and AdamW kernels apply to every gradient they read.
        self.grad_scale: torch.Tensor | None = None
        self.ns_launches_per_run = 0  # Newton-Schulz launches of the last plan run
        # When a list, (name, start, end) CUDA events are appended around the
        # momentum, Newton-Schulz and AdamW launches (benchmark instrumentation).
        self.profile_events: list | None = None

    def _event_pair(self, name: str):
        """Start a phase: an NVTX range always, and a pair of CUDA events when
        ``profile_events`` collects them. Every call is closed by _event_end."""
        trace.push(name)
        if self.profile_events is None:
            return None
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        return name, start, end

    def _event_end(self, pair) -> None:
        trace.pop()
        if pair is not None:
            pair[2].record()
            self.profile_events.append(pair)

    # ------------------------------------------------------------- errors
    def _record_error_check(self) -> None:
        self._err_host.copy_(self._err, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._err_event = ev

    def check_errors(self, block: bool = False) -> None:
        """Raise if a previous kernel recorded a device error (bounded wait expired)."""
        ev = self._err_event
        if ev is None:
            return
        if block:
            ev.synchronize()
        elif not ev.query():
            return
        code = int(self._err_host.item())
        self._err_event = None
        if code != 0:
            self._err.zero_()
            raise RuntimeError(f"opendm_b200 kernel reported device error 0x{code:x} (bounded wait expired)")

    def _class_algo(self) -> str:
        if self.ns_algo == "gram" and self.op_dtype == N.MUON_BF16:
            return "standard"  # the gram form needs 11-bit operands
        return self.ns_algo

    # ------------------------------------------------------------- planning
    def _key(self, items: list[MatrixItem], ns_steps: int):
        return (ns_steps, tuple((it.param.data_ptr(), tuple(it.param.shape), it.param.dtype,
                                 it.exp_avg.data_ptr()) for it in items))

    @property
    def classes(self) -> list[_ClassState]:
        """Shape classes of every cached plan."""
        return [cs for st in self._plans.values() for cs in st.classes]

    def _state_for(self, items: list[MatrixItem], ns_steps: int) -> _PlanState:
        key = self._key(items, ns_steps)
        st = self._plans.pop(key, None)
        if st is None:
            st = self._build(items, ns_steps)
            while len(self._plans) >= self.MAX_PLANS:
                old = self._plans.pop(next(iter(self._plans)))
                for plan in old.plans:
                    self.lib.muon_ns_plan_destroy(plan)
        self._plans[key] = st  # most recently used last
        if st.plans and st.sm_limit != self.sm_limit:
            for plan in st.plans:
                N.check(self.lib.muon_ns_plan_set_sm_limit(plan, int(self.sm_limit)), "muon_ns_plan_set_sm_limit")
            st.sm_limit = self.sm_limit
        return st

    def _build(self, items: list[MatrixItem], ns_steps: int) -> _PlanState:
        st = _PlanState()
        groups: dict[tuple, list[int]] = {}
        for i, it in enumerate(items):
            r, c = it.param.shape
            groups.setdefault((int(r), int(c), it.param.dtype), []).append(i)
        st.order = [(0, 0)] * len(items)
        for ci, ((r, c, dt), idxs) in enumerate(groups.items()):
            cs = _ClassState(r, c, dt, len(idxs), self.op_dtype, self.device, ns_steps, self._class_algo())
            for slot, i in enumerate(idxs):
                st.order[i] = (ci, slot)
                st.seg_order.append(i)
            # U, rounded to the parameter dtype, for muon_apply_update; rows padded
            # to 16 bytes for the epilogue's TMA stores. It goes into the X
            # buffer that the last Newton-Schulz apply does not read when its
            # rows fit there (bf16 U in either X type; fp32 U in tf32 X), else
            # into a buffer of its own.
            ld_u = _pad16(c, dt)
            u_es = torch.empty((), dtype=dt).element_size()
            cs.u_buf = None
            if ns_steps >= 1 and ld_u * u_es <= int(cs.cls.ld_x) * cs.es:
                cs.u_base = cs.cls.x1 if cs.last_x_read(ns_steps) == 0 else cs.cls.x0
            else:
                cs.u_buf = torch.empty((len(idxs), r, ld_u), dtype=dt, device=self.device)
                cs.u_base = cs.u_buf.data_ptr()
            cs.u_stride = r * ld_u * u_es  # bytes per matrix
            cs.cls.u_dtype = _dtype_code(items[idxs[0]].param)
            cs.cls.u_out = c_void_p(cs.u_base)
            cs.cls.ld_u = ld_u
            st.classes.append(cs)
        st.scales = torch.zeros(max(len(items), 1), dtype=torch.float32, device=self.device)
        if self.op_dtype in _F16_OPS:
            st.pscale = torch.zeros_like(st.scales)
            st.redo = torch.zeros(st.scales.numel(), dtype=torch.int32, device=self.device)
        first = 0
        for cs in st.classes:
            cs.first_seg = first
            cs.cls.scales = c_void_p(st.scales.data_ptr() + 4 * first)
            if self.op_dtype in _F16_OPS:
                cs.cls.flags = N.MUON_NS_INPUT_SCALED  # x0 = d * p, scales = the factor to the normalised input
            first += cs.count
        if ns_steps >= 1:
            st.plans = self._create_plans([cs.cls for cs in st.classes], ns_steps)
            st.ns_launches = sum(int(self.lib.muon_ns_plan_launches(p)) for p in st.plans)
        return st

    def _create_plans(self, classes: list, steps: int) -> list:
        """Library plans for `classes`, PLAN_CLASSES per plan (run one after the other)."""
        plans = []
        try:
            for i in range(0, len(classes), self.PLAN_CLASSES):
                part = classes[i:i + self.PLAN_CLASSES]
                arr = (N.NsClass * len(part))(*part)
                plan = c_void_p()
                N.check(self.lib.muon_ns_plan_create(arr, len(part), self.op_dtype, int(steps), byref(plan)),
                        "muon_ns_plan_create")
                plans.append(plan)
        except Exception:
            for plan in plans:
                self.lib.muon_ns_plan_destroy(plan)
            raise
        return plans

    def _run_plans(self, plans: list) -> None:
        for plan in plans:
            N.check(self.lib.muon_ns_plan_run(plan, c_void_p(self._err.data_ptr()), _stream_handle()),
                    "muon_ns_plan_run")

    # --------------------------------------------------------------- launches
    def _momentum(self, segs: list, grad_dtype: int, momentum: float, nesterov: bool, scales_ptr: int,
                  eps: float = 1e-7, dir_dtype: int | None = None, gradients: bool = True) -> None:
        """One momentum launch; ``gradients`` False for inputs that are not
        gradients (orthogonalize's copy), which the clip coefficient skips."""
        if not segs:
            return
        total = 0
        for s in segs:
            s.chunk_begin = total
            total += int(self.lib.muon_momentum_chunks(s.rows, s.cols))
        table = self._tables.get(N.struct_bytes(segs))
        partials = torch.empty(max(total, 1), dtype=torch.float32, device=self.device)
        if dir_dtype is None:
            dir_dtype = N.MUON_F32 if self.op_dtype in _F16_OPS else self.op_dtype
        gs = self.grad_scale if gradients else None
        N.check(self.lib.muon_momentum_scaled(c_void_p(table.data_ptr()), len(segs), total, grad_dtype, dir_dtype,
                                              c_float(momentum), int(bool(nesterov)), c_float(eps),
                                              c_void_p(partials.data_ptr()), c_void_p(scales_ptr),
                                              c_void_p(gs.data_ptr() if gs is not None else None), _stream_handle()),
                "muon_momentum_scaled")
        self.kernel_launches += 2 if total > 0 else 1

    def _momentum_f16(self, st, segs: list, grad_dtype: int, momentum: float, nesterov: bool,
                      eps: float = 1e-7, gradients: bool = True) -> None:
        """One muon_momentum_f16 call: momentum, norm, the fp16 operand and
        each matrix's Newton-Schulz input factor (plus the fix-up of matrices
        whose carried power of two does not fit this step)."""
        total = 0
        for sg in segs:
            sg.chunk_begin = total
            total += int(self.lib.muon_momentum_chunks(sg.rows, sg.cols))
        table = self._tables.get(N.struct_bytes(segs))
        partials = torch.empty(max(total, 1), dtype=torch.float32, device=self.device)
        gs = self.grad_scale if gradients else None
        N.check(self.lib.muon_momentum_f16(c_void_p(table.data_ptr()), len(segs), total, grad_dtype, c_float(momentum),
                                           int(bool(nesterov)), c_float(eps), c_void_p(partials.data_ptr()),
                                           c_void_p(st.pscale.data_ptr()), c_void_p(st.scales.data_ptr()),
                                           c_void_p(st.redo.data_ptr()),
                                           c_void_p(gs.data_ptr() if gs is not None else None), _stream_handle()),
                "muon_momentum_f16")
        self.kernel_launches += 3 if total > 0 else 1

    def muon_matrices(self, items: list[MatrixItem], *, momentum: float, nesterov: bool, weight_decay_factor: float,
                      ns_steps: int) -> None:
        """Full Muon update of whole matrices: momentum, Newton-Schulz and the
        in-place weight decay + scaled update (reference muon_adamw.py:381-414)."""
        if not items:
            return
        self.check_errors()
        for it in items:
            if it.param.device != self.device or not it.param.is_contiguous() or not it.exp_avg.is_contiguous():
                raise RuntimeError("Muon matrices must be contiguous tensors on the engine's device")
        st = self._state_for(items, ns_steps)
        grads = [it.grad for it in items]
        gdt = {_dtype_code(g) for g in grads if g is not None} or {N.MUON_F32}
        # Segments in class order: segment index == scale index.
        f16 = self.op_dtype in _F16_OPS
        keep: list[torch.Tensor] = []  # contiguous copies of strided gradients
        by_dtype: dict[int, list] = {}
        for i in st.seg_order:
            it = items[i]
            ci, slot = st.order[i]
            cs = st.classes[ci]
            g = it.grad
            if g is not None and not g.is_contiguous():
                g = g.contiguous()
                keep.append(g)  # the copy must outlive the launches that read it
            if f16:
                # one pass: momentum, norm and the fp16 operand d * p (muon_momentum_f16)
                seg = N.MomentumF16Seg()
                seg.dst = cs.cls.x0 + slot * cs.x_stride
                seg.mul, seg.scale_index, seg.lo_offset = cs.x0_scale, cs.first_seg + slot, cs.lo_offset
            else:
                seg = N.MomentumSeg()
                seg.direction = cs.cls.x0 + slot * cs.x_stride
            seg.grad = g.data_ptr() if g is not None else None
            seg.exp_avg = it.exp_avg.data_ptr()
            seg.rows, seg.cols, seg.ld = cs.rows, cs.cols, int(cs.cls.ld_x)
            code = _dtype_code(g) if g is not None else next(iter(gdt))
            by_dtype.setdefault(code, []).append((cs.first_seg + slot, seg))
        ev = self._event_pair("momentum")
        for code, lst in by_dtype.items():
            lst.sort(key=lambda x: x[0])
            if f16:
                self._momentum_f16(st, [seg for _, seg in lst], code, momentum, nesterov)
                continue
            # Each launch writes scales for a contiguous run; split into runs.
            run: list = []
            start = None
            for idx, seg in lst:
                if run and idx != start + len(run):
                    self._momentum(run, code, momentum, nesterov, st.scales.data_ptr() + 4 * start)
                    run = []
                if not run:
                    start = idx
                run.append(seg)
            if run:
                self._momentum(run, code, momentum, nesterov, st.scales.data_ptr() + 4 * start)
        self._event_end(ev)
        if ns_steps >= 1:
            ev = self._event_pair("ns")
            self._run_plans(st.plans)
            self._event_end(ev)
            self.ns_launches_per_run = st.ns_launches
            self.kernel_launches += st.ns_launches
            self._record_error_check()
            self._apply_updates(st, items, weight_decay_factor)
            self._last_state = (st, [it.param.data_ptr() for it in items])
        else:
            self._last_state = None
            self._zero_step_update(st, items, weight_decay_factor)

    def stored_updates(self) -> dict[int, torch.Tensor]:
        """U of every matrix of the last ``muon_matrices`` call (ns_steps >=
        1), keyed by the parameter's data_ptr(): [rows, cols] views, in the
        parameter dtype, of the buffers the update kernel read. They stay
        valid until the next step with the same matrix set overwrites them;
        for checks of the update before it is added to the parameters."""
        last = getattr(self, "_last_state", None)
        if last is None:
            return {}
        st, ptrs = last
        out: dict[int, torch.Tensor] = {}
        for ptr, (ci, slot) in zip(ptrs, st.order):
            cs = st.classes[ci]
            dt = cs.param_dtype
            if cs.u_buf is not None:
                out[ptr] = cs.u_buf[slot, :, :cs.cols]
                continue
            es = torch.empty((), dtype=dt).element_size()
            off = cs.u_base + slot * cs.u_stride - cs.workspace.data_ptr()
            out[ptr] = torch.empty(0, dtype=dt, device=self.device).set_(
                cs.workspace.untyped_storage(), off // es, (cs.rows, cs.cols), (int(cs.cls.ld_u), 1))
        return out

    def _apply_updates(self, st: _PlanState, items: list[MatrixItem], wd_factor: float) -> None:
        """Weight decay + p -= eff * U for every matrix (muon_apply_update)."""
        segs, total = [], 0
        for i in st.seg_order:
            it = items[i]
            ci, slot = st.order[i]
            cs = st.classes[ci]
            sg = N.UpdateSeg()
            sg.param = it.param.data_ptr()
            sg.update = cs.u_base + slot * cs.u_stride
            sg.rows, sg.cols, sg.ld = cs.rows, cs.cols, int(cs.cls.ld_u)
            sg.chunk_begin = total
            sg.eff = it.eff
            sg.param_dtype = cs.cls.u_dtype
            segs.append(sg)
            total += int(self.lib.muon_momentum_chunks(cs.rows, cs.cols))
        table = self._tables.get(N.struct_bytes(segs))
        ev = self._event_pair("update")
        N.check(self.lib.muon_apply_update(c_void_p(table.data_ptr()), len(segs), total, c_float(wd_factor),
                                           _stream_handle()), "muon_apply_update")
        self._event_end(ev)
        self.kernel_launches += 1

    def _normalized_input(self, st: _PlanState, cs: _ClassState, slot: int) -> torch.Tensor:
        """The unit-norm Newton-Schulz input of one matrix, fp32 (ns_steps == 0 result)."""
        x = cs.x0_value(slot)
        if self.op_dtype in _F16_OPS:  # x0 = d * p; scales = (1 / ||d||) * x0_scale / p
            return x * st.scales[cs.first_seg + slot] / cs.x0_scale
        return x * st.scales[cs.first_seg + slot]

    def _zero_step_update(self, st: _PlanState, items: list[MatrixItem], wd_factor: float) -> None:
        # ns_steps == 0: the reference's update is the normalised direction itself.
        for i in st.seg_order:
            it = items[i]
            ci, slot = st.order[i]
            u = self._normalized_input(st, st.classes[ci], slot)
            if wd_factor != 1.0:
                it.param.mul_(wd_factor)
            it.param.add_(u.to(it.param.dtype), alpha=-it.eff)

    def momentum_only(self, items: list[MatrixItem], *, momentum: float, nesterov: bool) -> None:
        """exp_avg update without a direction (matrices another rank orthogonalises)."""
        if not items:
            return
        keep: list[torch.Tensor] = []  # contiguous copies of strided gradients
        by_dtype: dict[int, list] = {}
        for it in items:
            seg = N.MomentumSeg()
            g = it.grad
            if g is not None and not g.is_contiguous():
                g = g.contiguous()
                keep.append(g)  # the copy must outlive the launches that read it
            seg.grad = g.data_ptr() if g is not None else None
            seg.exp_avg = it.exp_avg.data_ptr()
            seg.direction = None
            r, c = it.exp_avg.shape
            seg.rows, seg.cols, seg.ld = int(r), int(c), int(c)
            by_dtype.setdefault(_dtype_code(g) if g is not None else N.MUON_F32, []).append(seg)
        scratch = torch.empty(len(items), dtype=torch.float32, device=self.device)
        for code, segs in by_dtype.items():
            self._momentum(segs, code, momentum, nesterov, scratch.data_ptr())

    def direction(self, grad: torch.Tensor | None, exp_avg: torch.Tensor, *, momentum: float,
                  nesterov: bool) -> torch.Tensor:
        """Momentum update of a flat shard; returns the fp32 direction (for
        shard plans whose matrix is split across ranks)."""
        n = exp_avg.numel()
        out = torch.empty(n, dtype=torch.float32, device=self.device)
        seg = N.MomentumSeg()
        g = grad.contiguous() if grad is not None else None
        seg.grad = g.data_ptr() if g is not None else None
        seg.exp_avg = exp_avg.data_ptr()
        seg.direction = out.data_ptr()
        seg.rows, seg.cols, seg.ld = 1, n, n
        scratch = torch.empty(1, dtype=torch.float32, device=self.device)
        self._momentum([seg], _dtype_code(g) if g is not None else N.MUON_F32, momentum, nesterov,
                       scratch.data_ptr(), dir_dtype=N.MUON_F32)
        return out

    def directions_into(self, items: list, out: torch.Tensor, offsets: list[int], *, momentum: float,
                        nesterov: bool) -> None:
        """Momentum update of flat shards ``(grad or None, exp_avg)``, writing
        each fp32 direction into ``out[offsets[k]:]`` (one launch per grad
        dtype): the send buffer of the owner-only Newton-Schulz exchange."""
        if not items:
            return
        by_dtype: dict[int, list] = {}
        keep: list[torch.Tensor] = []  # contiguous copies must outlive the launches
        for (grad, exp_avg), off in zip(items, offsets):
            seg = N.MomentumSeg()
            g = grad.reshape(-1).contiguous() if grad is not None else None
            if g is not None:
                keep.append(g)
            seg.grad = g.data_ptr() if g is not None else None
            seg.exp_avg = exp_avg.data_ptr()
            seg.direction = out.data_ptr() + 4 * int(off)
            n = exp_avg.numel()
            seg.rows, seg.cols, seg.ld = 1, n, n
            by_dtype.setdefault(_dtype_code(g) if g is not None else N.MUON_F32, []).append(seg)
        scratch = torch.empty(len(items), dtype=torch.float32, device=self.device)
        for code, segs in by_dtype.items():
            self._momentum(segs, code, momentum, nesterov, scratch.data_ptr(), dir_dtype=N.MUON_F32)

    def orthogonalize_many(self, mats: list[torch.Tensor], out_dtypes: list[torch.dtype], steps: int = 5,
                           eps: float = 1e-7) -> list[torch.Tensor]:
        """zeropower_via_newtonschulz5 of several fp32 matrices in one grouped
        plan (classes by shape and output dtype); each result is rounded to its
        ``out_dtypes`` entry (bf16 or fp32) by the last epilogue."""
        if not mats:
            return []
        if steps < 1:
            return [self.orthogonalize(m, steps=steps, eps=eps).to(dt) for m, dt in zip(mats, out_dtypes)]
        groups: dict[tuple, list[int]] = {}
        for i, (m, dt) in enumerate(zip(mats, out_dtypes)):
            if m.ndim != 2 or m.dtype != torch.float32 or not m.is_contiguous() or m.device != self.device:
                raise RuntimeError("orthogonalize_many takes contiguous fp32 matrices on the engine's device")
            groups.setdefault((int(m.shape[0]), int(m.shape[1]), dt), []).append(i)
        f16 = self.op_dtype in _F16_OPS
        classes, segs, outs = [], [], [None] * len(mats)
        scales = torch.zeros(len(mats), dtype=torch.float32, device=self.device)
        keep = []
        first = 0
        for (rows, cols, dt), idxs in groups.items():
            cs = _ClassState(rows, cols, dt, len(idxs), self.op_dtype, self.device, int(steps), self._class_algo())
            ld_u = _pad16(cols, dt)
            u_buf = torch.empty((len(idxs), rows, ld_u), dtype=dt, device=self.device)
            cs.cls.u_dtype, cs.cls.u_out, cs.cls.ld_u = _dtype_code(u_buf), c_void_p(u_buf.data_ptr()), ld_u
            cs.cls.scales = c_void_p(scales.data_ptr() + 4 * first)
            if f16:
                cs.cls.flags = N.MUON_NS_INPUT_SCALED
            for slot, i in enumerate(idxs):
                # momentum 0 with exp_avg aliasing the input: exp_avg = d = input,
                # i.e. a copy into the operand buffer plus the Frobenius norm
                seg = N.MomentumF16Seg() if f16 else N.MomentumSeg()
                seg.grad, seg.exp_avg = mats[i].data_ptr(), mats[i].data_ptr()
                seg.rows, seg.cols, seg.ld = rows, cols, int(cs.cls.ld_x)
                if f16:
                    seg.dst = cs.cls.x0 + slot * cs.x_stride
                    seg.mul, seg.scale_index, seg.lo_offset = cs.x0_scale, first + slot, cs.lo_offset
                else:
                    seg.direction = cs.cls.x0 + slot * cs.x_stride
                segs.append(seg)
                outs[i] = u_buf[slot, :, :cols]
            classes.append(cs)
            keep += [cs.workspace, u_buf]
            first += len(idxs)
        if f16:
            tmp = _F16Inputs(len(mats), scales, self.device)  # no carried scale: every matrix takes the fix-up
            self._momentum_f16(tmp, segs, N.MUON_F32, 0.0, False, eps=eps, gradients=False)
            keep += [tmp.pscale, tmp.redo]
        else:
            self._momentum(segs, N.MUON_F32, 0.0, False, scales.data_ptr(), eps=eps, gradients=False)
        plans = self._create_plans([cs.cls for cs in classes], steps)
        try:
            self._run_plans(plans)
            self.kernel_launches += sum(int(self.lib.muon_ns_plan_launches(p)) for p in plans)
        finally:
            for plan in plans:
                self.lib.muon_ns_plan_destroy(plan)
        self._record_error_check()
        stream = torch.cuda.current_stream(self.device)
        for t in keep:  # workspaces stay valid until the queued kernels have run
            t.record_stream(stream)
        return outs

    def apply_update_flat(self, items: list, wd_factor: float) -> None:
        """Weight decay + p -= eff * u for flat shards ``(param, u, eff)``,
        u in the parameter dtype (one launch)."""
        if not items:
            return
        segs, total = [], 0
        for param, u, eff in items:
            n = param.numel()
            if u.numel() != n or u.dtype != param.dtype:
                raise RuntimeError("update shard does not match its parameter shard")
            sg = N.UpdateSeg()
            sg.param, sg.update = param.data_ptr(), u.data_ptr()
            sg.rows, sg.cols, sg.ld = 1, n, n
            sg.chunk_begin, sg.eff, sg.param_dtype = total, float(eff), _dtype_code(param)
            segs.append(sg)
            total += int(self.lib.muon_momentum_chunks(1, n))
        table = _upload(N.struct_bytes(segs), self.device)
        N.check(self.lib.muon_apply_update(c_void_p(table.data_ptr()), len(segs), total, c_float(wd_factor),
                                           _stream_handle()), "muon_apply_update")
        self.kernel_launches += 1

    def orthogonalize(self, matrix: torch.Tensor, steps: int = 5, eps: float = 1e-7) -> torch.Tensor:
        """zeropower_via_newtonschulz5 on the GPU (reference muon_adamw.py:101-128): fp32 result."""
        if matrix.ndim != 2:
            raise ValueError("Muon orthogonalization expects a 2D tensor.")
        if matrix.device != self.device:
            raise RuntimeError("matrix is not on the engine's device")
        rows, cols = (int(s) for s in matrix.shape)
        if matrix.numel() == 0:
            return torch.zeros((rows, cols), dtype=torch.float32, device=self.device)
        ld_out = _pad16(cols, torch.float32)
        out_buf = torch.zeros((rows, ld_out), dtype=torch.float32, device=self.device)
        out = out_buf[:, :cols]
        src = matrix if matrix.dtype in (torch.float32, torch.bfloat16) else matrix.float()
        src = src.contiguous()
        cs = _ClassState(rows, cols, torch.float32, 1, self.op_dtype, self.device, int(steps), self._class_algo())
        scales = torch.zeros(1, dtype=torch.float32, device=self.device)
        exp_avg = torch.zeros((rows, cols), dtype=torch.float32, device=self.device)
        f16 = self.op_dtype in _F16_OPS
        seg = N.MomentumF16Seg() if f16 else N.MomentumSeg()
        seg.grad = src.data_ptr()
        seg.exp_avg = exp_avg.data_ptr()
        seg.rows, seg.cols, seg.ld = rows, cols, int(cs.cls.ld_x)
        # momentum 0, no Nesterov: exp_avg = g and d = g, i.e. a copy plus the norm.
        if f16:
            seg.dst, seg.mul, seg.scale_index, seg.lo_offset = cs.cls.x0, cs.x0_scale, 0, cs.lo_offset
            cs.cls.flags = N.MUON_NS_INPUT_SCALED
            tmp = _F16Inputs(1, scales, self.device)
            self._momentum_f16(tmp, [seg], _dtype_code(src), 0.0, False, eps=eps, gradients=False)
        else:
            seg.direction = cs.cls.x0
            self._momentum([seg], _dtype_code(src), 0.0, False, scales.data_ptr(), eps=eps, gradients=False)
        if steps < 1:  # the normalised input itself
            if f16:
                return cs.x0_value(0) * scales[0] / cs.x0_scale
            return cs.x0_view(0).float() * scales[0]
        cs.cls.scales = c_void_p(scales.data_ptr())
        cs.cls.u_out = c_void_p(out_buf.data_ptr())
        cs.cls.ld_u = ld_out
        cs.cls.u_dtype = N.MUON_F32
        plan = c_void_p()
        N.check(self.lib.muon_ns_plan_create(byref(cs.cls), 1, self.op_dtype, int(steps), byref(plan)),
                "muon_ns_plan_create")
        try:
            N.check(self.lib.muon_ns_plan_run(plan, c_void_p(self._err.data_ptr()), _stream_handle()),
                    "muon_ns_plan_run")
            self.kernel_launches += int(self.lib.muon_ns_plan_launches(plan))
        finally:
            self.lib.muon_ns_plan_destroy(plan)
        self._record_error_check()
        # Keep the workspace alive until the kernels that use it have run.
        cs.workspace.record_stream(torch.cuda.current_stream())
        return out

    def adamw(self, items: list[AdamItem], *, lr: float, beta1: float, beta2: float, eps: float,
              weight_decay: float) -> None:
        """Fused AdamW over all items (reference muon_adamw.py:333-343)."""
        if not items:
            return
        segs = []
        total = 0
        keep: list[torch.Tensor] = []
        # With one step count for all items (the usual case) the table holds
        # only pointers and sizes and stays cached on the device; the step
        # size and bias correction are written into it by two fill kernels,
        # so a steady-state step issues no host-to-device copy.
        uniform = len({it.step for it in items}) == 1
        for it in items:
            for t in (it.param, it.grad, it.exp_avg, it.exp_avg_sq):
                if t.device != self.device:
                    raise RuntimeError("AdamW tensors must be on the engine's device")
            g = it.grad if it.grad.is_contiguous() else it.grad.contiguous()
            keep.append(g)  # a contiguous copy must outlive the launch that reads it
            if not it.param.is_contiguous():
                raise RuntimeError("AdamW parameters must be contiguous")
            s = N.AdamwSeg()
            s.param, s.grad = it.param.data_ptr(), g.data_ptr()
            s.exp_avg, s.exp_avg_sq = it.exp_avg.data_ptr(), it.exp_avg_sq.data_ptr()
            s.numel = it.param.numel()
            s.chunk_begin = total
            total += int(self.lib.muon_adamw_chunks(s.numel))
            bc1 = 1 - beta1 ** it.step
            bc2 = 1 - beta2 ** it.step
            step_size, bc2_sqrt = lr / bc1, bc2 ** 0.5
            if not uniform:
                s.step_size, s.bc2_sqrt = step_size, bc2_sqrt
            s.param_dtype = _dtype_code(it.param)
            s.grad_dtype = _dtype_code(g)
            segs.append(s)
        raw = N.struct_bytes(segs)
        if uniform:
            stream = torch.cuda.current_stream(self.device)
            table = self._adam_tables.get(raw, raw + stream.cuda_stream.to_bytes(8, "little"))
            words = table.view(torch.float32).view(len(segs), sizeof(N.AdamwSeg) // 4)
            # float32 rounding of the Python values, as the c_float fields would round them
            words[:, N.AdamwSeg.step_size.offset // 4].fill_(step_size)
            words[:, N.AdamwSeg.bc2_sqrt.offset // 4].fill_(bc2_sqrt)
        else:
            table = _upload(raw, self.device)
        wd_factor = 1.0 - lr * weight_decay if weight_decay != 0 else 1.0
        ev = self._event_pair("adamw")
        gs = self.grad_scale
        N.check(self.lib.muon_adamw_scaled(c_void_p(table.data_ptr()), len(segs), total, float(beta1), float(beta2),
                                           c_float(eps), c_float(wd_factor),
                                           c_void_p(gs.data_ptr() if gs is not None else None), _stream_handle()),
                "muon_adamw_scaled")
        self._event_end(ev)
        self.kernel_launches += 1

    def clip_grad_norm(self, grads: list[torch.Tensor], max_norm: float) -> torch.Tensor:
        """torch.nn.utils.clip_grad_norm_'s total norm and coefficient (norm
        type 2) of ``grads`` on the device: returns a float32 tensor [total,
        coefficient]; nothing is rewritten (the coefficient is applied by the
        kernels that read the gradients, via ``grad_scale``)."""
        out = torch.zeros(2, dtype=torch.float32, device=self.device)
        segs, total = [], 0
        keep: list[torch.Tensor] = []  # contiguous copies must outlive the launch
        for g in grads:
            if g.device != self.device:
                raise RuntimeError("gradients must be on the engine's device")
            g = g if g.is_contiguous() else g.contiguous()
            keep.append(g)
            if g.numel() == 0:
                continue
            sg = N.NormSeg()
            sg.grad, sg.numel, sg.chunk_begin, sg.dtype = g.data_ptr(), g.numel(), total, _dtype_code(g)
            segs.append(sg)
            total += int(self.lib.muon_norm_chunks(g.numel()))
        table = self._tables.get(N.struct_bytes(segs)) if segs else None
        partials = torch.empty(max(total, 1), dtype=torch.float32, device=self.device)
        N.check(self.lib.muon_clip_grad_norm(c_void_p(table.data_ptr() if table is not None else None), len(segs),
                                             total, c_float(max_norm), c_void_p(partials.data_ptr()),
                                             c_void_p(out.data_ptr()), _stream_handle()), "muon_clip_grad_norm")
        self.kernel_launches += 2 if total > 0 else 1
        return out

    def close(self) -> None:
        for st in self._plans.values():
            for plan in st.plans:
                self.lib.muon_ns_plan_destroy(plan)
            st.plans = []
        self._plans.clear()

    def __del__(self):  # pragma: no cover - interpreter teardown order varies
        try:
            self.close()
        except Exception:
            pass


def effective_lr(lr: float, lr_scale: float, moonlight: float, shape: tuple[int, int],
                 scale_mode: str = "reference") -> float:
    """Per-matrix update scale. "reference": lr * lr_scale * coefficient *
    sqrt(max(rows, cols)) (muon_adamw.py:408-413); "shape": lr * lr_scale *
    max(1, rows / cols) ** 0.5 (the original Muon form)."""
    if scale_mode == "reference":
        return float(lr) * float(lr_scale) * float(moonlight) * math.sqrt(max(shape))
    if scale_mode == "shape":
        return float(lr) * float(lr_scale) * max(1.0, shape[0] / shape[1]) ** 0.5
    raise ValueError(f"scale_mode must be 'reference' or 'shape', got {scale_mode!r}")
