"""Newton-Schulz launch microbenchmark: one class's three launches of one
iteration (gram, poly, apply) through the C ABI, against torch.matmul
(cuBLAS) GEMMs of the same sizes on the same GPU.

    python nsbench.py [--reps 10]

For each shape class it prints the time of one ``muon_ns_plan_run`` with
``steps=1`` (standard form, fp16 operands), its executed FLOP rate (256x256
tiles, upper-triangle tiles of the two symmetric products) and the rate of
three dense cuBLAS batched GEMMs doing the same products without symmetry.
"""

from __future__ import annotations

import argparse
import ctypes

import torch

from opendm_b200 import _native as N
from opendm_b200.engine import _ClassState

SHAPES = [(8192, 8192, 1), (2048, 8192, 8), (8192, 2048, 8), (2048, 2048, 32)]


def _time(fn, reps: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / reps


def run(reps: int = 10) -> list[dict]:
    dev = torch.device("cuda", 0)
    lib = N.lib()
    out = []
    for rows, cols, count in SHAPES:
        cs = _ClassState(rows, cols, torch.float32, count, N.MUON_F16, dev, 1, "standard")
        scales = torch.ones(count, device=dev)
        u = torch.empty(count, rows, cols, device=dev)
        cs.cls.scales = ctypes.c_void_p(scales.data_ptr())
        cs.cls.u_out = ctypes.c_void_p(u.data_ptr())
        cs.cls.ld_u, cs.cls.u_dtype = cols, N.MUON_F32
        x0 = torch.empty(0, dtype=torch.float16, device=dev).set_(
            cs.workspace.untyped_storage(), (cs.cls.x0 - cs.workspace.data_ptr()) // 2,
            (count, rows, cs.cls.ld_x), (rows * cs.cls.ld_x, cs.cls.ld_x, 1))
        x0.normal_().mul_(0.01)
        plan = ctypes.c_void_p()
        N.check(lib.muon_ns_plan_create(ctypes.byref(cs.cls), 1, N.MUON_F16, 1, ctypes.byref(plan)),
                "muon_ns_plan_create")
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        try:
            ms = _time(lambda: N.check(lib.muon_ns_plan_run(plan, ctypes.c_void_p(err.data_ptr()), stream),
                                       "muon_ns_plan_run"), reps)
        finally:
            lib.muon_ns_plan_destroy(plan)
        m, n = min(rows, cols), max(rows, cols)
        t = (m + 255) // 256
        executed = count * 2 * 256 * 256 * (t * (t + 1) // 2 * (n + m) + ((rows + 255) // 256) * ((cols + 255) // 256) * m)
        dense = count * (4 * m * m * n + 2 * m ** 3)
        a = torch.randn(count, m, n, device=dev, dtype=torch.float16)
        b = torch.randn(count, n, m, device=dev, dtype=torch.float16)
        c = torch.randn(count, m, m, device=dev, dtype=torch.float16)
        cub = _time(lambda: (torch.bmm(a, b), torch.bmm(c, c), torch.bmm(c, a)), reps)
        out.append({"shape": f"{rows}x{cols}", "count": count, "ours_ms": ms, "ours_executed_tflops": executed / ms / 1e9,
                    "cublas_ms": cub, "cublas_dense_tflops": dense / cub / 1e9, "error_word": int(err.item())})
        del a, b, c, u, cs
    a = torch.randn(8192, 8192, device=dev, dtype=torch.float16)
    ms = _time(lambda: a @ a, reps)
    out.append({"shape": "cuBLAS 8192^3", "cublas_ms": ms, "cublas_dense_tflops": 2 * 8192 ** 3 / ms / 1e9})
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reps", type=int, default=10)
    args = ap.parse_args()
    for r in run(args.reps):
        if "ours_ms" in r:
            print(f"{r['shape']} x{r['count']}: ours {r['ours_ms']:.3f} ms, {r['ours_executed_tflops']:.0f} TFLOP/s "
                  f"executed | cuBLAS 3 bmm {r['cublas_ms']:.3f} ms, {r['cublas_dense_tflops']:.0f} TFLOP/s dense | "
                  f"device error word {r['error_word']}")
        else:
            print(f"{r['shape']}: {r['cublas_ms']:.3f} ms, {r['cublas_dense_tflops']:.0f} TFLOP/s")


if __name__ == "__main__":
    main()
