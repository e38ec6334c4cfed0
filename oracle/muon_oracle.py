"""CPU oracle for the MuonAdamW optimizer step -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy float32 arithmetic, the algorithm of the
reference optimizer ``opendm/optimizer/muon_adamw.py`` (dexmal/opendm) and of
the torch functional AdamW it calls (``torch.optim.adam._single_tensor_adam``
with decoupled weight decay, torch 2.11.0). It is the checker that the CUDA
path is compared against. Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` may import it; the product package
``opendm_b200`` never does.

Pinning: ``tests/golden/make_golden.py`` runs the unmodified reference
optimizer (importable from the reference checkout in the build container) on
seeded inputs and stores its outputs in ``tests/golden/*.npz``;
``tests/test_oracle_golden.py`` checks this module against those fixtures.

Every function cites the reference lines it restates.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

# muon_adamw.py:123
NS_A, NS_B, NS_C = 3.4445, -4.7750, 2.0315


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even); returns float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = rounded.view(np.float32).copy()
    nan = np.isnan(x)
    out[nan] = np.float32("nan")
    return out


def cast_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Value of ``tensor.to(dtype)`` for dtype in {"float32", "bfloat16"} (as float32)."""
    x = np.asarray(x, dtype=np.float32)
    return bf16_round(x) if dtype == "bfloat16" else x.copy()


def zeropower_via_newtonschulz5(matrix: np.ndarray, steps: int = 5, eps: float = 1e-7) -> np.ndarray:
    """Restates muon_adamw.py:101-128 (quintic Newton-Schulz, fp32)."""
    matrix = np.asarray(matrix)
    if matrix.ndim != 2:  # :107-108
        raise ValueError("Muon orthogonalization expects a 2D tensor.")
    x = matrix.astype(np.float32)  # :110
    if x.size == 0:  # :111-112
        return x
    transposed = x.shape[0] > x.shape[1]  # :114-116
    if transposed:
        x = x.T
    norm = np.float32(np.sqrt(np.sum(x.astype(np.float64) ** 2)))  # :118
    if not np.isfinite(norm) or norm <= 0:  # :119-120
        return np.zeros(matrix.shape, dtype=np.float32)
    x = (x / np.float32(max(norm, np.float32(eps)))).astype(np.float32)  # :121
    a, b, c = np.float32(NS_A), np.float32(NS_B), np.float32(NS_C)
    for _ in range(max(int(steps), 0)):  # :124-126
        gram = x @ x.T
        x = a * x + (b * gram + c * (gram @ gram)) @ x
    return np.ascontiguousarray(x.T if transposed else x)  # :128


def effective_lr(lr: float, lr_scale: float, moonlight: float, shape: tuple[int, int]) -> float:
    """Restates muon_adamw.py:408-413 (double precision, as in Python)."""
    return float(lr) * float(lr_scale) * float(moonlight) * math.sqrt(max(shape))


def momentum_direction(grad, exp_avg, momentum: float, nesterov: bool):
    """Restates muon_adamw.py:383-394. Returns (new exp_avg, direction), fp32."""
    g = np.zeros_like(exp_avg) if grad is None else np.asarray(grad, np.float32)
    mu = np.float32(momentum)
    buf = (exp_avg * mu).astype(np.float32) + g  # buffer.mul_(m).add_(g)
    buf = buf.astype(np.float32)
    if nesterov:
        # grad.clone().add_(buffer, alpha=momentum): one fused multiply-add
        d = (g.astype(np.float64) + np.float64(mu) * buf.astype(np.float64)).astype(np.float32)
    else:
        d = buf.copy()
    return buf, d


def apply_update(param, update, *, lr: float, weight_decay: float, eff: float, param_dtype: str,
                 device_semantics: str = "cpu"):
    """Restates muon_adamw.py:395-398 and :414 with torch's rounding order.

    ``param.mul_(1 - lr*wd)`` rounds the fp32 product to the param dtype; then
    ``param.add_(update.to(dtype), alpha=-eff)`` rounds the update to the param
    dtype and computes ``p + alpha*u`` in fp32 with one rounding before the
    final cast. torch's CPU kernel first converts ``alpha`` to the param dtype
    (bf16 for bf16 params); its CUDA kernel keeps ``alpha`` in fp32.
    ``device_semantics`` ("cpu" | "cuda") selects which of the two to follow.
    """
    factor = (1.0 - float(lr) * float(weight_decay)) if weight_decay else 1.0
    return apply_update_factor(param, update, wd_factor=factor, eff=eff, param_dtype=param_dtype,
                               device_semantics=device_semantics)


def apply_update_factor(param, update, *, wd_factor: float, eff: float, param_dtype: str,
                        device_semantics: str = "cpu"):
    """``apply_update`` with the weight-decay factor 1 - lr*wd given directly
    (1.0 means no weight decay)."""
    p = np.asarray(param, np.float32)
    if wd_factor != 1.0:
        p = cast_to(p * np.float32(wd_factor), param_dtype)
    u = cast_to(update, param_dtype)
    alpha = np.float32(-eff)
    if device_semantics == "cpu" and param_dtype == "bfloat16":
        alpha = bf16_round(np.array([alpha], np.float32))[0]
    out = (p.astype(np.float64) + np.float64(alpha) * u.astype(np.float64)).astype(np.float32)
    return cast_to(out, param_dtype)


def adamw_step(param, grad, exp_avg, exp_avg_sq, step: float, *, lr, beta1, beta2, eps, weight_decay,
               param_dtype: str):
    """Restates torch.optim.adam._single_tensor_adam (decoupled weight decay,
    non-capturable) as called by muon_adamw.py:143-175 / :342.

    Returns (param, exp_avg, exp_avg_sq, step) after one step.
    """
    step = float(step) + 1.0
    p = np.asarray(param, np.float32)
    g = np.asarray(grad, np.float32)
    if weight_decay != 0:
        p = cast_to(p * np.float32(1.0 - lr * weight_decay), param_dtype)
    w = np.float32(1.0 - beta1)
    # exp_avg.lerp_(grad, 1 - beta1): weight < 0.5 -> self + w * (end - self), fused
    m = (exp_avg.astype(np.float64) + np.float64(w) * (g - exp_avg).astype(np.float64)).astype(np.float32)
    # exp_avg_sq.mul_(beta2).addcmul_(grad, grad, value=1 - beta2)
    v = (exp_avg_sq * np.float32(beta2)).astype(np.float32)
    v = (v + ((np.float32(1.0 - beta2) * g).astype(np.float32) * g).astype(np.float32)).astype(np.float32)
    bc1 = 1 - beta1 ** step
    bc2 = 1 - beta2 ** step
    step_size = lr / bc1
    bc2_sqrt = bc2 ** 0.5
    denom = ((np.sqrt(v) / np.float32(bc2_sqrt)).astype(np.float32) + np.float32(eps)).astype(np.float32)
    p = (p + np.float32(-step_size) * (m / denom).astype(np.float32)).astype(np.float32)
    return cast_to(p, param_dtype), m, v, step


@dataclass
class MatrixState:
    exp_avg: np.ndarray
    exp_avg_sq: np.ndarray
    step: float = 0.0


@dataclass
class OracleMuonAdamW:
    """Whole-optimizer restatement over plain arrays (single process, plan kind
    "local"): the Muon group (muon_adamw.py:362-414) and the AdamW group
    (:333-343), in the reference's group order [adamw, muon] (:215-223)."""

    lr: float
    betas: tuple[float, float]
    eps: float
    weight_decay: float
    muon_momentum: float = 0.95
    muon_nesterov: bool = True
    muon_ns_steps: int = 5
    muon_lr_scale: float = 1.0
    muon_moonlight_coefficient: float = 0.2
    muon_state: dict = field(default_factory=dict)
    adamw_state: dict = field(default_factory=dict)

    def step(self, muon_params: dict, muon_grads: dict, adamw_params: dict, adamw_grads: dict,
             param_dtype: str = "float32", updates_out: dict | None = None,
             device_semantics: str = "cpu") -> None:
        """Update the arrays in ``*_params`` in place (values stay float32,
        holding bf16 values when param_dtype == "bfloat16")."""
        for name, p in adamw_params.items():
            g = adamw_grads.get(name)
            if g is None:
                continue
            st = self.adamw_state.setdefault(
                name, MatrixState(np.zeros_like(p, np.float32), np.zeros_like(p, np.float32)))
            newp, st.exp_avg, st.exp_avg_sq, st.step = adamw_step(
                p, g, st.exp_avg, st.exp_avg_sq, st.step, lr=self.lr, beta1=self.betas[0],
                beta2=self.betas[1], eps=self.eps, weight_decay=self.weight_decay,
                param_dtype=param_dtype)
            p[...] = newp
        if not any(g is not None for g in muon_grads.values()):  # :350-352
            return
        for name, p in muon_params.items():
            g = muon_grads.get(name)
            st = self.muon_state.setdefault(
                name, MatrixState(np.zeros_like(p, np.float32), np.zeros_like(p, np.float32)))
            st.step += 1.0
            st.exp_avg, d = momentum_direction(g, st.exp_avg, self.muon_momentum, self.muon_nesterov)
            u = zeropower_via_newtonschulz5(d.reshape(p.shape), steps=self.muon_ns_steps)
            if updates_out is not None:
                updates_out[name] = u
            eff = effective_lr(self.lr, self.muon_lr_scale, self.muon_moonlight_coefficient, p.shape)
            p[...] = apply_update(p, u, lr=self.lr, weight_decay=self.weight_decay, eff=eff,
                                  param_dtype=param_dtype, device_semantics=device_semantics)


def clip_grad_norm(grads: list, dtypes: list[str], max_norm: float, device_semantics: str = "cpu"):
    """Gradient-norm clipping as the reference's trainer runs it before the
    optimizer step (``trainer.py:213`` sets ``max_grad_norm=1.0``; the HF
    trainer calls ``torch.nn.utils.clip_grad_norm_``, torch 2.11.0,
    ``torch/nn/utils/clip_grad.py``: ``_get_total_norm`` then
    ``_clip_grads_with_norm_``), norm type 2:

    * per-tensor norms (``_foreach_norm``): fp32 sum of squares, sqrt, rounded
      to the tensor's dtype;
    * total norm: sqrt of the sum of the squared per-tensor norms, rounded to
      the promoted dtype of all gradients (bf16 only if every gradient is bf16);
    * ``max_norm / (total + 1e-6)`` as torch evaluates it for a tensor on the
      right (``reciprocal() * max_norm``), each op rounded to that dtype, then
      clamped to at most 1;
    * every gradient multiplied in place, rounded to its dtype. torch's CPU
      ``_foreach_mul_`` multiplies by the coefficient in the promoted dtype;
      its CUDA kernel first casts the 0-d coefficient to each gradient's
      dtype (``device_semantics="cuda"``), which differs for bf16 gradients
      when some gradient is fp32.

    ``grads``: float32 arrays holding values of ``dtypes`` ("bfloat16" or
    "float32"), ``None`` for absent gradients. Returns (clipped grads, total
    norm, coefficient)."""
    present = [(g, dt) for g, dt in zip(grads, dtypes) if g is not None]
    if not present:
        return list(grads), 0.0, 1.0
    res_dt = "bfloat16" if all(dt == "bfloat16" for _, dt in present) else "float32"
    norms = []
    for g, dt in present:
        s = np.float32(np.sum(np.square(g.astype(np.float64))))  # fp32-accurate sum
        norms.append(cast_to(np.array([np.sqrt(np.float32(s))], dtype=np.float32), dt)[0])
    n32 = np.array(norms, dtype=np.float32)
    total = cast_to(np.array([np.sqrt(np.float32(np.sum(n32.astype(np.float64) ** 2)))], np.float32), res_dt)[0]
    denom = cast_to(np.array([np.float32(total) + np.float32(1e-6)], np.float32), res_dt)[0]
    recip = cast_to(np.array([np.float32(1.0) / denom], np.float32), res_dt)[0]
    coef = cast_to(np.array([recip * np.float32(max_norm)], np.float32), res_dt)[0]
    coef = min(float(coef), 1.0)
    out = []
    for g, dt in zip(grads, dtypes):
        c = np.float32(coef) if device_semantics == "cpu" else cast_to(np.array([coef], np.float32), dt)[0]
        out.append(None if g is None else cast_to(g * c, dt))
    return out, float(total), coef


def rel_frobenius(a: np.ndarray, b: np.ndarray) -> float:
    """||a - b||_F / ||b||_F in float64 (0 when both are zero)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    num = np.linalg.norm(a - b)
    if den == 0:
        return 0.0 if num == 0 else float("inf")
    return float(num / den)


def ns_flops(shape: tuple[int, int], steps: int = 5) -> float:
    """Dense Newton-Schulz FLOPs of one matrix: steps * (4 m^2 n + 2 m^3)."""
    m, n = min(shape), max(shape)
    return float(steps) * (4.0 * m * m * n + 2.0 * m ** 3)
