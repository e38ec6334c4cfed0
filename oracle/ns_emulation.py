"""TEST INFRASTRUCTURE, not part of the product: a numpy emulation of the
arithmetic of the Newton-Schulz kernels (opendm_b200/csrc/ns_gemm.cu) in
fp16 mode, used by tests/test_ns_emulation.py to check the numerics design on
the CPU against the fp32 oracle of the reference algorithm
(muon_oracle.zeropower_via_newtonschulz5, reference muon_adamw.py:101-128).

Modelled: every stored operand rounded to fp16 (subnormals included) after a
power-of-two scale, or to tf32 (ties away from zero) or bf16 (ties to even)
without one; products accumulated exactly and rounded once to fp32
(the tensor cores accumulate in fp32 in a different order, so this is an
approximation of the accumulation error, not of the operand rounding);
epilogue arithmetic in fp32. Two forms:

* standard: the reference's iteration on X in the shifted form
  X <- (alpha I + A' B') X with A' = X X^T - I, B' = gamma A' + beta I;
* gram: the iteration on A = X X^T, A <- P (P A) with P = alpha I + A' B',
  accumulating Q = P ... P and applying X <- Q X every `restart` iterations.

`emulate_split` runs either form with split fp16 operands (hi + lo pairs,
three passes per product, precision="parity"), with the accumulation either
exact (rounded once to fp32) or modelled as a truncating multi-term adder.

Scales (as the kernels choose them): X at iteration 0 times 2^round(log2
sqrt(m n)), later times 2^round(log2 sqrt(n)); gram-form A, P and P A times
2^round(log2(m / 4)), Q times 2^round(log2(m / 64)).
"""

from __future__ import annotations

import math

import numpy as np

NS_A, NS_B, NS_C = 3.4445, -4.7750, 2.0315  # reference muon_adamw.py:123
ALPHA, BETA, GAMMA = NS_A + NS_B + NS_C, NS_B + 2 * NS_C, NS_C


def _f16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, np.float64).astype(np.float16).astype(np.float64)


def _f32(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, np.float64).astype(np.float32).astype(np.float64)


def _tf32(x: np.ndarray) -> np.ndarray:
    """fp32 rounded to tf32's 10 stored mantissa bits, ties away from zero
    (the kernels' cvt.rna)."""
    u = np.ascontiguousarray(np.asarray(x, np.float64).astype(np.float32)).view(np.uint32).astype(np.uint64)
    r = ((u + 0x1000) & 0xFFFFE000).astype(np.uint32)
    return r.view(np.float32).astype(np.float64)


def _bf16(x: np.ndarray) -> np.ndarray:
    """fp32 rounded to bfloat16, ties to even."""
    u = np.ascontiguousarray(np.asarray(x, np.float64).astype(np.float32)).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32).astype(np.float64)


_ROUND = {"fp16": _f16, "tf32": _tf32, "bf16": _bf16}


def _pow2(x: float) -> float:
    """The power of two nearest to x in the log domain, halves rounded away
    from zero (C's lround, as the library rounds)."""
    e = math.log2(x)
    return 2.0 ** int(math.floor(e + 0.5) if e >= 0 else -math.floor(-e + 0.5))


def x_scale(m: int, n: int, iteration: int, op: str = "fp16") -> float:
    """Power-of-two scale of the stored X at `iteration` (m <= n): the
    unit-norm input's entries are ~1/sqrt(m n), later iterates' ~1/sqrt(n).
    Only fp16 needs one (1.0 for tf32 and bf16, which have fp32's range)."""
    if op != "fp16":
        return 1.0
    return _pow2(math.sqrt(m * n)) if iteration == 0 else _pow2(math.sqrt(n))


def _prepare(g: np.ndarray, eps: float = 1e-7) -> tuple[np.ndarray, bool]:
    """Frobenius-normalised input, wide orientation (m <= n)."""
    x = np.asarray(g, np.float64)
    norm = math.sqrt(float(np.sum(_f32(x) ** 2)))
    tall = x.shape[0] > x.shape[1]
    if tall:
        x = x.T
    return x / max(norm, eps), tall


def emulate_standard(g: np.ndarray, steps: int = 5, op: str = "fp16", shifted: bool = True) -> np.ndarray:
    """The standard (iterate-on-X) form with operands of type `op` ("fp16",
    "tf32" or "bf16"). shifted=False evaluates the reference's own grouping,
    X <- a X + (b A + c A A) X, with the same operand rounding, for
    comparison."""
    rnd = _ROUND[op]
    x, tall = _prepare(g)
    m, n = x.shape
    eye = np.eye(m)
    s = x_scale(m, n, 0, op)
    xs = rnd(x * s)
    for it in range(steps):
        last = it == steps - 1
        s_next = 1.0 if last else x_scale(m, n, it + 1, op)
        if shifted:
            a = _f32(xs @ xs.T) / (s * s)
            ap = a - eye
            bp = GAMMA * ap + BETA * eye
            mm = rnd(_f32(rnd(ap) @ rnd(bp)) + ALPHA * eye)
            acc = _f32(mm @ xs) * (s_next / s)
        else:
            a = rnd(_f32(xs @ xs.T) / (s * s))
            b = rnd(NS_B * a + NS_C * _f32(a @ a))
            acc = _f32(NS_A * xs + _f32(b @ xs)) * (s_next / s)
        xs = _f32(acc) if last else rnd(acc)
        s = s_next
    return (xs.T if tall else xs).astype(np.float32)


def emulate_gram(g: np.ndarray, steps: int = 5, restart: int = 3, op: str = "fp16") -> np.ndarray:
    """The gram form (iterate on X X^T, restart every `restart` iterations)
    with operands of type `op` ("fp16" or "tf32", the types the library runs
    it in)."""
    if op not in ("fp16", "tf32"):
        raise ValueError("the gram form runs with fp16 or tf32 operands")
    rnd = _ROUND[op]
    x, tall = _prepare(g)
    m, n = x.shape
    eye = np.eye(m)
    s = x_scale(m, n, 0, op)
    xs = rnd(x * s)
    sa, sq = (_pow2(m / 4.0), _pow2(m / 64.0)) if op == "fp16" else (1.0, 1.0)
    bounds = list(range(0, steps, restart)) + [steps]
    for s0, s1 in zip(bounds, bounds[1:]):
        p = pa = q = None
        for j in range(s0, s1):
            a = _f32(xs @ xs.T) / (s * s) if j == s0 else _f32(p @ pa) / (sa * sa)
            ap = a - eye
            bp = GAMMA * ap + BETA * eye
            p_true = _f32(rnd(ap * sa) @ rnd(bp * sa)) / (sa * sa) + ALPHA * eye
            p = rnd(p_true * sa)
            q = rnd(p_true * sq) if j == s0 else rnd(_f32(p @ q) / sa)
            if j < s1 - 1:
                pa = rnd(_f32(p @ rnd(a * sa)) / sa)
        last = s1 == steps
        s_next = 1.0 if last else x_scale(m, n, s1, op)
        acc = _f32(q @ xs) * (s_next / (sq * s))
        xs = _f32(acc) if last else rnd(acc)
        s = s_next
    return (xs.T if tall else xs).astype(np.float32)


# ------------------------------------------------- split fp16 operands
def _split_f16(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """The stored pair of a split operand: hi = fp16(x), lo = fp16(x - hi),
    subnormals included (the kernels' MUON_F16X3 epilogue stores)."""
    hi = _f16(x)
    return hi, _f16(np.asarray(x, np.float64) - hi)


def _rz_f32(x: np.ndarray) -> np.ndarray:
    """x cut toward zero to fp32's 24-bit significand."""
    m, e = np.frexp(np.asarray(x, np.float64))
    return np.ldexp(np.trunc(m * 2.0 ** 24) / 2.0 ** 24, e)


def _split_product(a, b, acc: str, bits: int, block: int) -> np.ndarray:
    """A B for split operand pairs a = (hi, lo), b = (hi, lo): the passes
    hi*hi, hi*lo and lo*hi, in that order, into one fp32 accumulator (lo*lo
    dropped), as the kernels issue them (one whole K loop per pass).

    acc "exact": the products exact, the whole sum rounded once to fp32.
    acc "truncate": K in blocks of `block` products; per block the
    accumulator and the block's exact products are cut toward zero to `bits`
    fraction bits below the leading bit of the largest of them, added exactly,
    and the sum cut toward zero to fp32. This models a fused multi-term adder
    with truncating alignment, of the kind Fasi, Higham, Mikaitis and Pranesh
    describe for earlier tensor cores ("Numerical behavior of NVIDIA tensor
    cores", PeerJ Computer Science 7:e330, 2021); its parameters are a
    hypothesis held against the errors measured on the B200, not a
    specification of its hardware."""
    passes = [(a[0], b[0]), (a[0], b[1]), (a[1], b[0])]
    if acc == "exact":
        return _f32(sum(x @ y for x, y in passes))
    if acc != "truncate":
        raise ValueError(f"unknown accumulation model {acc!r}")
    out = np.zeros((a[0].shape[0], b[0].shape[1]))
    for x, y in passes:
        for k0 in range(0, x.shape[1], block):
            terms = x[:, k0:k0 + block, None] * y[None, k0:k0 + block, :]  # exact products
            _, e = np.frexp(np.maximum(np.abs(out), np.abs(terms).max(axis=1)))
            ulp = np.ldexp(1.0, e - 1 - bits)
            cut = np.trunc(out / ulp) * ulp + (np.trunc(terms / ulp[:, None, :]) * ulp[:, None, :]).sum(axis=1)
            out = _rz_f32(cut)
    return out


def emulate_split(g: np.ndarray, steps: int = 5, form: str = "standard", restart: int = 3, acc: str = "exact",
                  bits: int = 23, block: int = 16) -> np.ndarray:
    """Newton-Schulz with split fp16 operands (precision="parity") in the
    standard or the gram form (restart every `restart` iterations; restart
    >= steps: one segment, no restart), at the fp16 power-of-two scales, with
    the products of `_split_product` under accumulation model `acc`."""
    x, tall = _prepare(g)
    m, n = x.shape
    eye = np.eye(m)

    def mm(u, v):
        return _split_product(u, v, acc, bits, block)

    def tr(u):
        return tuple(t.T for t in u)

    s = x_scale(m, n, 0)
    xs = _split_f16(x * s)
    if form == "standard":
        for it in range(steps):
            last = it == steps - 1
            s_next = 1.0 if last else x_scale(m, n, it + 1)
            ap = mm(xs, tr(xs)) / (s * s) - eye
            bp = GAMMA * ap + BETA * eye
            mmat = _split_f16(mm(_split_f16(ap), _split_f16(bp)) + ALPHA * eye)
            out = mm(mmat, xs) * (s_next / s)
            xs = (out, np.zeros_like(out)) if last else _split_f16(out)
            s = s_next
        res = xs[0]
        return (res.T if tall else res).astype(np.float32)
    if form != "gram":
        raise ValueError(f"unknown form {form!r}")
    sa, sq = _pow2(m / 4.0), _pow2(m / 64.0)
    bounds = list(range(0, steps, restart)) + [steps]
    for s0, s1 in zip(bounds, bounds[1:]):
        p = pa = q = None
        for j in range(s0, s1):
            a = mm(xs, tr(xs)) / (s * s) if j == s0 else mm(p, pa) / (sa * sa)
            ap = a - eye
            bp = GAMMA * ap + BETA * eye
            p_true = mm(_split_f16(ap * sa), _split_f16(bp * sa)) / (sa * sa) + ALPHA * eye
            p = _split_f16(p_true * sa)
            q = _split_f16(p_true * sq) if j == s0 else _split_f16(mm(p, q) / sa)
            if j < s1 - 1:
                pa = _split_f16(mm(p, _split_f16(a * sa)) / sa)
        last = s1 == steps
        s_next = 1.0 if last else x_scale(m, n, s1)
        out = mm(q, xs) * (s_next / (sq * s))
        xs = (out, np.zeros_like(out)) if last else _split_f16(out)
        s = s_next
    res = xs[0]
    return (res.T if tall else res).astype(np.float32)


def structured_input(shape: tuple[int, int], kind: str, seed: int = 0) -> np.ndarray:
    """Seeded test matrices with the spectra the numerics notes discuss:
    "gauss", "lowrank_noise" (rank 4 plus 10% noise), "heavytail" (1% of
    entries x100), "powerlaw" (singular values 1/k), "expdecay" (e^(-10 k/r)),
    "rank1"."""
    rng = np.random.default_rng(seed)
    m, n = shape
    g = rng.standard_normal(shape)
    if kind == "gauss":
        out = g
    elif kind == "lowrank_noise":
        out = 0.1 * g + rng.standard_normal((m, 4)) @ rng.standard_normal((4, n))
    elif kind == "heavytail":
        out = np.where(rng.random(shape) < 0.01, g * 100.0, g)
    elif kind == "rank1":
        out = np.outer(rng.standard_normal(m), rng.standard_normal(n))
    elif kind in ("powerlaw", "expdecay"):
        k = min(shape)
        u, _ = np.linalg.qr(rng.standard_normal((m, k)))
        v, _ = np.linalg.qr(rng.standard_normal((n, k)))
        sv = np.arange(1, k + 1) ** -1.0 if kind == "powerlaw" else np.exp(-10.0 * np.arange(k) / k)
        out = (u * sv) @ v.T
    else:
        raise ValueError(f"unknown input kind {kind!r}")
    return out.astype(np.float32)
