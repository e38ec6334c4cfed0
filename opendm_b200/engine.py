"""Device engine: drives the sm_100a kernels of libopendm_muon.so for one GPU.

The optimizer (``opendm_b200.optimizer.MuonAdamW``) hands the engine lists of
whole matrices it must update and the AdamW-group tensors. The engine

* groups matrices by (rows, cols, param dtype) into shape classes; each class
  owns one workspace holding the Newton-Schulz operands X (ping-pong), A' and
  M for all its matrices, stacked so one grouped launch covers the class;
* caches the Newton-Schulz plan (tensor maps, tile schedules) while the
  parameters stay at the same addresses; only the gradient pointers change
  between steps, so the per-step host work is one small segment table;
* launches (a) momentum + Frobenius scale, (b) 3 x ns_steps grouped
  tcgen05 GEMMs whose last epilogue applies (c) weight decay and the scaled
  update in place, and the fused AdamW kernel, all on the current CUDA stream.

There is no fallback: every entry point raises if the library is missing or
the tensors are not on an sm_100 device.
"""

from __future__ import annotations

import math
from ctypes import byref, c_float, c_int, c_void_p
from dataclasses import dataclass

import torch

from . import _native as N

_DTYPE_CODE = {torch.bfloat16: N.MUON_BF16, torch.float32: N.MUON_F32}
PRECISIONS = {"tf32": N.MUON_TF32, "bf16": N.MUON_BF16}


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


def _stream_handle() -> c_void_p:
    return c_void_p(torch.cuda.current_stream().cuda_stream)


def _upload(raw: bytes, device: torch.device) -> torch.Tensor:
    host = torch.frombuffer(bytearray(raw), dtype=torch.uint8).pin_memory()
    return host.to(device, non_blocking=True)


class _ClassState:
    """Workspace and buffers of one shape class."""

    def __init__(self, rows: int, cols: int, param_dtype: torch.dtype, count: int, op_dtype: int,
                 device: torch.device):
        lib = N.lib()
        self.rows, self.cols, self.count, self.param_dtype = rows, cols, count, param_dtype
        nbytes = lib.muon_ns_class_workspace_bytes(rows, cols, count, op_dtype)
        self.workspace = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
        self.cls = N.NsClass()
        self.cls.rows, self.cls.cols, self.cls.count = rows, cols, count
        N.check(lib.muon_ns_class_layout(byref(self.cls), c_void_p(self.workspace.data_ptr()), op_dtype),
                "muon_ns_class_layout")
        self.es = 2 if op_dtype == N.MUON_BF16 else 4
        self.x_stride = rows * int(self.cls.ld_x) * self.es  # bytes per matrix in x0


class CudaMuonEngine:
    """Runs the Muon and AdamW kernels on one CUDA device."""

    def __init__(self, device: torch.device | str | int, precision: str = "tf32"):
        if precision not in PRECISIONS:
            raise ValueError(f"precision must be one of {sorted(PRECISIONS)}, got {precision!r}")
        self.device = torch.device(device) if not isinstance(device, int) else torch.device("cuda", device)
        if self.device.type != "cuda":
            raise RuntimeError("opendm_b200 runs on CUDA (sm_100) devices only; got " + str(self.device))
        self.precision = precision
        self.op_dtype = PRECISIONS[precision]
        self.lib = N.lib()
        idx = self.device.index if self.device.index is not None else torch.cuda.current_device()
        N.check(self.lib.muon_device_check(idx), "muon_device_check")
        self._plan = None
        self._plan_key = None
        self._classes: list[_ClassState] = []
        self._order: list[tuple[int, int]] = []  # item index -> (class index, slot)
        self._scales = None
        self._err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._err_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._err_event = None
        self.kernel_launches = 0  # launches issued by this engine (for benchmarks)

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

    # ------------------------------------------------------------- planning
    def _key(self, items: list[MatrixItem], ns_steps: int):
        return (ns_steps, tuple((it.param.data_ptr(), tuple(it.param.shape), it.param.dtype,
                                 it.exp_avg.data_ptr()) for it in items))

    def _build(self, items: list[MatrixItem], ns_steps: int) -> None:
        if self._plan is not None:
            self.lib.muon_ns_plan_destroy(self._plan)
            self._plan = None
        groups: dict[tuple, list[int]] = {}
        for i, it in enumerate(items):
            r, c = it.param.shape
            groups.setdefault((int(r), int(c), it.param.dtype), []).append(i)
        self._classes = []
        self._order = [(0, 0)] * len(items)
        self._seg_order: list[int] = []
        ptr_tables = []
        for ci, ((r, c, dt), idxs) in enumerate(groups.items()):
            cs = _ClassState(r, c, dt, len(idxs), self.op_dtype, self.device)
            for slot, i in enumerate(idxs):
                self._order[i] = (ci, slot)
                self._seg_order.append(i)
            ptrs = torch.tensor([items[i].param.data_ptr() for i in idxs], dtype=torch.int64)
            cs.param_ptrs = ptrs.to(self.device)
            ptr_tables.append(cs.param_ptrs)
            cs.cls.param_dtype = _dtype_code(items[idxs[0]].param)
            cs.cls.params = c_void_p(cs.param_ptrs.data_ptr())
            cs.cls.u_out = None
            cs.cls.ld_u = 0
            self._classes.append(cs)
        self._scales = torch.zeros(max(len(items), 1), dtype=torch.float32, device=self.device)
        first = 0
        for cs in self._classes:
            cs.first_seg = first
            cs.cls.scales = c_void_p(self._scales.data_ptr() + 4 * first)
            first += cs.count
        if ns_steps >= 1:
            arr = (N.NsClass * len(self._classes))(*[cs.cls for cs in self._classes])
            plan = c_void_p()
            N.check(self.lib.muon_ns_plan_create(arr, len(self._classes), self.op_dtype, ns_steps, byref(plan)),
                    "muon_ns_plan_create")
            self._plan = plan
        self._plan_key = self._key(items, ns_steps)

    # --------------------------------------------------------------- launches
    def _momentum(self, segs: list, grad_dtype: int, momentum: float, nesterov: bool, scales_ptr: int,
                  eps: float = 1e-7) -> None:
        if not segs:
            return
        total = 0
        for s in segs:
            s.chunk_begin = total
            total += int(self.lib.muon_momentum_chunks(s.rows, s.cols))
        table = _upload(N.struct_bytes(segs), self.device)
        partials = torch.empty(max(total, 1), dtype=torch.float32, device=self.device)
        N.check(self.lib.muon_momentum(c_void_p(table.data_ptr()), len(segs), total, grad_dtype, self.op_dtype,
                                       c_float(momentum), int(bool(nesterov)), c_float(eps),
                                       c_void_p(partials.data_ptr()), c_void_p(scales_ptr), _stream_handle()),
                "muon_momentum")
        self.kernel_launches += 2 if total > 0 else 1

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
        if self._plan_key != self._key(items, ns_steps):
            self._build(items, ns_steps)
        grads = [it.grad for it in items]
        gdt = {_dtype_code(g) for g in grads if g is not None} or {N.MUON_F32}
        # Segments in class order: segment index == scale index.
        by_dtype: dict[int, list] = {}
        for i in self._seg_order:
            it = items[i]
            ci, slot = self._order[i]
            cs = self._classes[ci]
            seg = N.MomentumSeg()
            g = it.grad
            if g is not None and not g.is_contiguous():
                g = g.contiguous()
            seg.grad = g.data_ptr() if g is not None else None
            seg.exp_avg = it.exp_avg.data_ptr()
            seg.direction = cs.cls.x0 + slot * cs.x_stride
            seg.rows, seg.cols, seg.ld = cs.rows, cs.cols, int(cs.cls.ld_x)
            code = _dtype_code(g) if g is not None else next(iter(gdt))
            by_dtype.setdefault(code, []).append((cs.first_seg + slot, seg))
        for code, lst in by_dtype.items():
            # Each launch writes scales for a contiguous run; split into runs.
            lst.sort(key=lambda x: x[0])
            run: list = []
            start = None
            for idx, seg in lst:
                if run and idx != start + len(run):
                    self._momentum(run, code, momentum, nesterov, self._scales.data_ptr() + 4 * start)
                    run = []
                if not run:
                    start = idx
                run.append(seg)
            if run:
                self._momentum(run, code, momentum, nesterov, self._scales.data_ptr() + 4 * start)
        if ns_steps >= 1:
            eff = (c_float * len(self._classes))(*[items[self._seg_order[cs.first_seg]].eff for cs in self._classes])
            N.check(self.lib.muon_ns_plan_run(self._plan, eff, c_float(weight_decay_factor),
                                              c_void_p(self._err.data_ptr()), _stream_handle()),
                    "muon_ns_plan_run")
            self.kernel_launches += 3 * ns_steps
            self._record_error_check()
        else:
            self._zero_step_update(items, weight_decay_factor)

    def _zero_step_update(self, items: list[MatrixItem], wd_factor: float) -> None:
        # ns_steps == 0: the reference's update is the normalised direction itself.
        for i in self._seg_order:
            it = items[i]
            ci, slot = self._order[i]
            cs = self._classes[ci]
            dtype = torch.bfloat16 if self.op_dtype == N.MUON_BF16 else torch.float32
            ld = int(cs.cls.ld_x)
            x = torch.empty(0, dtype=dtype, device=self.device).set_(
                cs.workspace.untyped_storage(), (cs.cls.x0 - cs.workspace.data_ptr()) // cs.es + slot * cs.rows * ld,
                (cs.rows, cs.cols), (ld, 1))
            u = x.float() * self._scales[cs.first_seg + slot]
            if wd_factor != 1.0:
                it.param.mul_(wd_factor)
            it.param.add_(u.to(it.param.dtype), alpha=-it.eff)

    def momentum_only(self, items: list[MatrixItem], *, momentum: float, nesterov: bool) -> None:
        """exp_avg update without a direction (matrices another rank orthogonalises)."""
        if not items:
            return
        by_dtype: dict[int, list] = {}
        for it in items:
            seg = N.MomentumSeg()
            g = it.grad
            if g is not None and not g.is_contiguous():
                g = g.contiguous()
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
        saved = self.op_dtype
        self.op_dtype = N.MUON_TF32  # fp32 storage; values rounded to tf32 like the NS input
        try:
            self._momentum([seg], _dtype_code(g) if g is not None else N.MUON_F32, momentum, nesterov,
                           scratch.data_ptr())
        finally:
            self.op_dtype = saved
        return out

    def orthogonalize(self, matrix: torch.Tensor, steps: int = 5, eps: float = 1e-7) -> torch.Tensor:
        """zeropower_via_newtonschulz5 on the GPU (reference muon_adamw.py:101-128): fp32 result."""
        if matrix.ndim != 2:
            raise ValueError("Muon orthogonalization expects a 2D tensor.")
        if matrix.device != self.device:
            raise RuntimeError("matrix is not on the engine's device")
        rows, cols = (int(s) for s in matrix.shape)
        out = torch.zeros((rows, cols), dtype=torch.float32, device=self.device)
        if matrix.numel() == 0:
            return out
        src = matrix if matrix.dtype in (torch.float32, torch.bfloat16) else matrix.float()
        src = src.contiguous()
        cs = _ClassState(rows, cols, torch.float32, 1, self.op_dtype, self.device)
        scales = torch.zeros(1, dtype=torch.float32, device=self.device)
        exp_avg = torch.zeros((rows, cols), dtype=torch.float32, device=self.device)
        seg = N.MomentumSeg()
        seg.grad = src.data_ptr()
        seg.exp_avg = exp_avg.data_ptr()
        seg.direction = cs.cls.x0
        seg.rows, seg.cols, seg.ld = rows, cols, int(cs.cls.ld_x)
        # momentum 0, no Nesterov: exp_avg = g and d = g, i.e. a rounded copy plus the norm.
        self._momentum([seg], _dtype_code(src), 0.0, False, scales.data_ptr(), eps=eps)
        if steps < 1:
            dtype = torch.bfloat16 if self.op_dtype == N.MUON_BF16 else torch.float32
            ld = int(cs.cls.ld_x)
            x = torch.empty(0, dtype=dtype, device=self.device).set_(
                cs.workspace.untyped_storage(), 0, (rows, cols), (ld, 1))
            return x.float() * scales[0]
        cs.cls.scales = c_void_p(scales.data_ptr())
        cs.cls.u_out = c_void_p(out.data_ptr())
        cs.cls.ld_u = cols
        cs.cls.params = None
        cs.cls.param_dtype = N.MUON_F32
        plan = c_void_p()
        N.check(self.lib.muon_ns_plan_create(byref(cs.cls), 1, self.op_dtype, int(steps), byref(plan)),
                "muon_ns_plan_create")
        try:
            N.check(self.lib.muon_ns_plan_run(plan, None, c_float(1.0), c_void_p(self._err.data_ptr()),
                                              _stream_handle()), "muon_ns_plan_run")
        finally:
            self.lib.muon_ns_plan_destroy(plan)
        self.kernel_launches += 3 * int(steps)
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
        for it in items:
            for t in (it.param, it.grad, it.exp_avg, it.exp_avg_sq):
                if t.device != self.device:
                    raise RuntimeError("AdamW tensors must be on the engine's device")
            g = it.grad if it.grad.is_contiguous() else it.grad.contiguous()
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
            s.step_size = lr / bc1
            s.bc2_sqrt = bc2 ** 0.5
            s.param_dtype = _dtype_code(it.param)
            s.grad_dtype = _dtype_code(g)
            segs.append(s)
        table = _upload(N.struct_bytes(segs), self.device)
        wd_factor = 1.0 - lr * weight_decay if weight_decay != 0 else 1.0
        N.check(self.lib.muon_adamw(c_void_p(table.data_ptr()), len(segs), total, float(beta1), float(beta2),
                                    c_float(eps), c_float(wd_factor), _stream_handle()), "muon_adamw")
        self.kernel_launches += 1

    def close(self) -> None:
        if self._plan is not None:
            self.lib.muon_ns_plan_destroy(self._plan)
            self._plan = None

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
