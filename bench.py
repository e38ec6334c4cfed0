"""Benchmark: one full MuonAdamW optimizer step (Muon + AdamW groups).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2|c2s|c4|c5]
                    [--precision fp16|tf32|bf16|parity] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1)

Workloads (synthetic, seeded; shapes of the configurations the reference's
metric is quoted on):
  c2  2B-class decoder, 28 layers, hidden 2048, GQA q/o 2048x2048, k/v 256x2048,
      SwiGLU gate/up 8192x2048, down 2048x8192 (196 Muon matrices) + norms and a
      151936x2048 embedding on AdamW. Default; at N > 1 the same model is
      sharded over the ranks (strong scaling): Newton-Schulz owners with
      owner-only momentum, and the AdamW group split into per-rank element
      ranges (--no-adamw-sharding keeps the whole AdamW group on every rank).
  c4  ~4B VLA stack: ViT 27x (1152, MLP 4304) + LM 36x (2560, kv 512, MLP 9728)
      + action expert 18x (1024, MLP 4096), 540 Muon matrices + norms.
  c5  7B-class decoder, 32 layers, hidden 4096, MLP 11008 (224 Muon matrices),
      gradients with 1% heavy-tail entries.
  c2s the first 4 layers of c2 (28 Muon matrices, no embedding): the small
      case for profiler captures, not a bench line.
Parameters bf16 ~ N(0, 0.02), gradients bf16 ~ N(0, 1e-3), fp32 optimizer state.

Rank 0 prints one JSON line. `value` is the device time of one optimizer step
(max over ranks, CUDA events, K steps after W warm-up steps). `e2e` is the
same step measured through the public API with the gradients copied in from
pinned host memory every step (double-buffered: the next step's upload runs
on a copy stream during the current step) and a slice of the updated
parameters read back. `roofline` is the Newton-Schulz GEMMs' algorithmic rate (the reference
algorithm's dense FLOP count per NS second) against the measured bf16 tensor
peak, plus the rate of the FLOPs the tiles actually execute (256 x 256 tiles,
upper triangle of symmetric products, gram form where chosen). The timed steps sit
inside a CUDA profiler range (ncu --profile-from-start off captures only
them). `cpu_baseline` (N = 1, rank 0) is the numpy oracle
of the reference algorithm on the host cores, timed on one matrix of every
shape class and extrapolated by multiplicity.

--impl reference prints the same metric, with the same `config` object, for
the reference algorithm on the host CPU (the numpy oracle; the reference itself
is PyTorch code that runs only from its own checkout), rank 0 only; each step
times one matrix of every shape class and extrapolates by multiplicity.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

LR, BETAS, EPS, WD = 0.02, (0.9, 0.95), 1e-8, 0.01
MOMENTUM, NS_STEPS = 0.95, 5


def decoder_layers(prefix, layers, hidden, q_out, kv_out, mlp, o_in=None):
    """(name, shape) of one decoder-style stack; nn.Linear weights are [out, in]."""
    o_in = o_in or q_out
    out = []
    for i in range(layers):
        p = f"{prefix}.layers.{i}"
        out += [(f"{p}.self_attn.q_proj.weight", (q_out, hidden)),
                (f"{p}.self_attn.k_proj.weight", (kv_out, hidden)),
                (f"{p}.self_attn.v_proj.weight", (kv_out, hidden)),
                (f"{p}.self_attn.o_proj.weight", (hidden, o_in)),
                (f"{p}.mlp.gate_proj.weight", (mlp, hidden)),
                (f"{p}.mlp.up_proj.weight", (mlp, hidden)),
                (f"{p}.mlp.down_proj.weight", (hidden, mlp)),
                (f"{p}.input_layernorm.weight", (hidden,)),
                (f"{p}.post_attention_layernorm.weight", (hidden,))]
    return out


def vit_layers(prefix, layers, hidden, mlp):
    out = []
    for i in range(layers):
        p = f"{prefix}.layers.{i}"
        out += [(f"{p}.self_attn.q_proj.weight", (hidden, hidden)),
                (f"{p}.self_attn.k_proj.weight", (hidden, hidden)),
                (f"{p}.self_attn.v_proj.weight", (hidden, hidden)),
                (f"{p}.self_attn.out_proj.weight", (hidden, hidden)),
                (f"{p}.mlp.fc1.weight", (mlp, hidden)),
                (f"{p}.mlp.fc2.weight", (hidden, mlp)),
                (f"{p}.layer_norm1.weight", (hidden,)),
                (f"{p}.layer_norm2.weight", (hidden,))]
    return out


def config_params(name: str):
    if name == "c2":
        return (decoder_layers("model", 28, 2048, 2048, 256, 8192)
                + [("model.embed_tokens.weight", (151936, 2048)), ("model.norm.weight", (2048,))])
    if name == "c4":
        return (vit_layers("vision", 27, 1152, 4304)
                + decoder_layers("language", 36, 2560, 2560, 512, 9728)
                + decoder_layers("action_expert", 18, 1024, 1024, 1024, 4096)
                + [("language.norm.weight", (2560,)), ("action_expert.norm.weight", (1024,))])
    if name == "c5":
        return decoder_layers("model", 32, 4096, 4096, 4096, 11008) + [("model.norm.weight", (4096,))]
    if name == "c2s":
        return decoder_layers("model", 4, 2048, 2048, 256, 8192) + [("model.norm.weight", (2048,))]
    raise ValueError(f"unknown config {name!r}")


def is_muon(name, shape):
    return len(shape) == 2 and ".layers." in name


DESCRIPTIONS = {
    "c2": "2B-class decoder (28L, h2048, GQA kv256, SwiGLU 8192) + 151936x2048 embedding",
    "c4": "~4B VLA (ViT 27L h1152/4304 + LM 36L h2560 kv512/9728 + AE 18L h1024/4096)",
    "c5": "7B-class decoder (32L, h4096, MHA, SwiGLU 11008), 1% heavy-tail grads",
    "c2s": "first 4 layers of the 2B-class decoder (profiling case)",
}


# ------------------------------------------------------------------ helpers
def ns_flops(shape, steps=NS_STEPS):
    m, n = min(shape), max(shape)
    return steps * (4.0 * m * m * n + 2.0 * m ** 3)


def line_config(cfg: str, precision: str, world: int, adamw_sharding: bool) -> dict:
    """The JSON line's `config` object. Both arms print this same object, so
    the reference arm's line names the same workload as this library's."""
    muon_shapes = [s for n, s in config_params(cfg) if is_muon(n, s)]
    parallelism = f"dp{world}"
    if world > 1:
        parallelism += (" (FLOP-balanced NS owners, bf16 param all-gather, owner-only momentum"
                        + (", AdamW element ranges per rank" if adamw_sharding else "") + ")")
    return {"workload": cfg, "description": DESCRIPTIONS[cfg], "muon_matrices": len(muon_shapes),
            "ns_tflop_per_step": round(sum(ns_flops(s) for s in muon_shapes) / 1e12, 2), "precision": precision,
            "parallelism": parallelism, "l2": "inputs larger than L2 (params+grads+state >> 126 MB)"}


GRAM_SEGMENT = 3  # iterations between restarts of the gram-form Newton-Schulz

# DRAM bytes (read + write) per ns_gemm launch: ncu's dram__bytes_read.sum +
# dram__bytes_write.sum over the 17 ns_gemm launches of one captured step of
# the configuration on one GPU (c2: 49.48 GB read + 22.82 GB written), divided
# by 17.
NS_TRAFFIC_PER_LAUNCH = {"c2": 72.30e9 / 17}


def ns_executed_flops(shape, steps=NS_STEPS, algo="standard"):
    """FLOPs the Newton-Schulz launches execute for one matrix: 256 x 256
    output tiles, K rounded up to the 64-deep stage, upper-triangle tiles only
    for symmetric m x m products. "standard": gram, poly and apply per
    iteration. "gram": per segment of L iterations one gram, 4L - 3 symmetric
    m x m products and one apply."""
    rows, cols = shape
    m, n = min(shape), max(shape)

    def kpad(k):
        return (k + 63) // 64 * 64

    t = (m + 255) // 256
    sym_tiles = t * (t + 1) // 2
    gram = sym_tiles * 256 * 256 * 2 * kpad(n)
    sq = sym_tiles * 256 * 256 * 2 * kpad(m)
    apply = ((rows + 255) // 256) * ((cols + 255) // 256) * 256 * 256 * 2 * kpad(m)
    if algo == "standard":
        return steps * float(gram + sq + apply)
    total = 0.0
    for s0 in range(0, steps, GRAM_SEGMENT):
        seg = min(GRAM_SEGMENT, steps - s0)
        total += gram + (4 * seg - 3) * sq + apply
    return total


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d["bf16_tflops_sustained"]), "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.gpus = {str(i) for i in gpu_indices}
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9 or f[0] not in self.gpus:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------ CPU oracle leg
def cpu_sample(cfg: str, seed: int = 0):
    """Time the numpy oracle on one matrix of every Muon shape class plus a
    slice of every AdamW tensor, and extrapolate to the full step (ms)."""
    import numpy as np

    from oracle import muon_oracle as O

    rng = np.random.default_rng(seed)
    params = config_params(cfg)
    classes: dict = {}
    adam_elems = 0
    for name, shape in params:
        if is_muon(name, shape):
            classes[shape] = classes.get(shape, 0) + 1
        else:
            adam_elems += math.prod(shape)
    total = 0.0
    for shape, count in classes.items():
        p = O.bf16_round(rng.standard_normal(shape, dtype=np.float32) * 0.02)
        g = O.bf16_round(rng.standard_normal(shape, dtype=np.float32) * 1e-3)
        m = np.zeros(shape, np.float32)
        t0 = time.perf_counter()
        m, d = O.momentum_direction(g, m, MOMENTUM, True)
        u = O.zeropower_via_newtonschulz5(d, NS_STEPS)
        O.apply_update(p, u, lr=LR, weight_decay=WD, eff=O.effective_lr(LR, 1.0, 0.2, shape),
                       param_dtype="bfloat16")
        total += (time.perf_counter() - t0) * count
    n_adam = min(adam_elems, 1 << 22)
    p = O.bf16_round(rng.standard_normal(n_adam, dtype=np.float32) * 0.02)
    g = O.bf16_round(rng.standard_normal(n_adam, dtype=np.float32) * 1e-3)
    z = np.zeros(n_adam, np.float32)
    t0 = time.perf_counter()
    O.adamw_step(p, g, z, z, 0.0, lr=LR, beta1=BETAS[0], beta2=BETAS[1], eps=EPS, weight_decay=WD,
                 param_dtype="bfloat16")
    total += (time.perf_counter() - t0) * (adam_elems / n_adam)
    sample = (f"numpy oracle: 1 matrix per Muon shape class ({len(classes)} classes) x multiplicity + AdamW on "
              f"{n_adam} of {adam_elems} elements, extrapolated")
    return total * 1e3, sample


def cpu_full_step(cfg: str, seed: int = 0):
    """Time the numpy oracle on EVERY Muon matrix and every AdamW element of
    the configuration once (ms): a full reference step on the host, one matrix
    at a time so host memory holds one matrix's arrays; random inputs are made
    outside the timed regions. Validates the extrapolation of cpu_sample."""
    import numpy as np

    from oracle import muon_oracle as O

    rng = np.random.default_rng(seed)
    total = 0.0
    n_muon = 0
    for name, shape in config_params(cfg):
        if is_muon(name, shape):
            p = O.bf16_round(rng.standard_normal(shape, dtype=np.float32) * 0.02)
            g = O.bf16_round(rng.standard_normal(shape, dtype=np.float32) * 1e-3)
            m = np.zeros(shape, np.float32)
            t0 = time.perf_counter()
            m, d = O.momentum_direction(g, m, MOMENTUM, True)
            u = O.zeropower_via_newtonschulz5(d, NS_STEPS)
            O.apply_update(p, u, lr=LR, weight_decay=WD, eff=O.effective_lr(LR, 1.0, 0.2, shape),
                           param_dtype="bfloat16")
            total += time.perf_counter() - t0
            n_muon += 1
        else:
            n = math.prod(shape)
            for a in range(0, n, 1 << 24):
                k = min(1 << 24, n - a)
                p = O.bf16_round(rng.standard_normal(k, dtype=np.float32) * 0.02)
                g = O.bf16_round(rng.standard_normal(k, dtype=np.float32) * 1e-3)
                z = np.zeros(k, np.float32)
                t0 = time.perf_counter()
                O.adamw_step(p, g, z, z.copy(), 0.0, lr=LR, beta1=BETAS[0], beta2=BETAS[1], eps=EPS,
                             weight_decay=WD, param_dtype="bfloat16")
                total += time.perf_counter() - t0
    return total * 1e3, f"numpy oracle: all {n_muon} Muon matrices and every AdamW element, once (not extrapolated)"


def cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    cfg = args.config
    for _ in range(args.warmup):
        cpu_sample(cfg)
    times = []
    sample = ""
    for _ in range(args.steps):
        ms, sample = cpu_sample(cfg)
        times.append(ms)
    value = statistics.median(times)
    line = {"metric": "muon_step_ms", "value": round(value, 3), "unit": "ms", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(value, 3),
            "higher_is_better": False, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": line_config(cfg, args.precision, world, args.adamw_sharding),
            "cpu_baseline": {"value": round(value, 3), "unit": "ms", "cores": cores(), "kind": "port",
                             "sample": sample,
                             "arithmetic": "fp32 throughout (the reference algorithm), on the host cores"},
            "e2e": {"value": round(value, 3), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# -------------------------------------------------------------- GPU leg
def run_ours(args):
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        # one copy stream per peer (p2p all-gather) next to the compute and NCCL
        # streams: enough hardware queues that they do not serialise
        os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    from datetime import timedelta
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)

    from opendm_b200.optimizer import MuonAdamW, mark_muon_parameters

    cfg = args.config
    spec = config_params(cfg)
    gen = torch.Generator(device=device).manual_seed(0)

    class Model(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.names = []
            for name, shape in spec:
                t = torch.randn(shape, generator=gen, device=device, dtype=torch.float32).mul_(0.02)
                self.register_parameter(name.replace(".", "_"), torch.nn.Parameter(t.to(torch.bfloat16)))
                self.names.append(name)

    model = Model()
    keymap = {name.replace(".", "_"): (name, shape) for name, shape in spec}
    mark_muon_parameters(model, predicate=lambda n, p: is_muon(*keymap[n]))
    opt = MuonAdamW(model, lr=LR, betas=BETAS, eps=EPS, weight_decay=WD, muon_momentum=MOMENTUM,
                    muon_ns_steps=NS_STEPS, precision=args.precision, state_sharding=world > 1,
                    allgather=args.allgather, comm_sms=args.comm_sms,
                    allgather_waves=args.waves, allgather_wave_ratio=args.wave_ratio,
                    adamw_sharding=args.adamw_sharding and world > 1)
    params = list(model.parameters())
    ggen = torch.Generator(device=device).manual_seed(1)
    grads = []
    for p in params:
        g = torch.randn(p.shape, generator=ggen, device=device, dtype=torch.float32).mul_(1e-3)
        if cfg == "c5" and p.ndim == 2:
            mask = torch.rand(p.shape, generator=ggen, device=device) < 0.01
            g = torch.where(mask, torch.randn(p.shape, generator=ggen, device=device) * 1e-1, g)
        grads.append(g.to(torch.bfloat16))
    for p, g in zip(params, grads):
        p.grad = g

    def sync_all():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        opt.step()
    engine = opt._engine
    opt.check_device_errors()

    # ---- device-timed region
    peaks = load_peaks()
    sampler = ClockSampler([local] if world == 1 else list(range(world))) if rank == 0 else None
    launches0 = engine.kernel_launches
    engine.profile_events = []
    if sampler:
        sampler.start()
        time.sleep(0.5)  # first samples land before the timed region
    sync_all()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.profiler.start()
    start.record()
    for _ in range(args.steps):
        opt.step()
    end.record()
    torch.cuda.profiler.stop()
    sync_all()
    clocks = sampler.stop() if sampler else None
    step_ms = max_over_ranks(start.elapsed_time(end) / args.steps)
    launches = (engine.kernel_launches - launches0) // args.steps
    ns_launches = engine.ns_launches_per_run
    events = engine.profile_events
    engine.profile_events = None
    opt.check_device_errors()
    # host time to enqueue one step, each from an idle GPU (median of 3, max
    # over ranks): the step is host-bound when this reaches the device time
    host_times = []
    for _ in range(3):
        sync_all()
        h0 = time.perf_counter()
        opt.step()
        host_times.append((time.perf_counter() - h0) * 1e3)
    sync_all()
    host_ms = max_over_ranks(sorted(host_times)[1])
    per = {}
    for name, s, e in events:
        per.setdefault(name, []).append(s.elapsed_time(e))
    def per_step(name):  # an event name can occur several times per step (one per wave)
        return sum(per.get(name, [])) / args.steps

    ns_ms = max_over_ranks(per_step("ns"))
    mom_ms = per_step("momentum")
    adam_ms = per_step("adamw")
    upd_ms = per_step("update")
    ag_wait_ms = max_over_ranks(per_step("allgather_wait"))

    muon_shapes = [s for n, s in spec if is_muon(n, s)]
    # FLOPs this rank ran (its owned matrices); the roofline uses the busiest rank.
    owners = opt._owners.get(id(opt.param_groups[1]))
    if owners is not None:
        mine = [s for s, o in zip(opt.param_groups[1]["muon_shapes"], owners) if o == rank]
    else:
        mine = muon_shapes
    my_flops = sum(ns_flops(s) for s in mine)
    owner_balance = None
    if owners is not None:  # Newton-Schulz FLOPs per rank, max / mean (dense count and executed)
        from opendm_b200.sharding import load_balance

        shapes_all = opt.param_groups[1]["muon_shapes"]
        dense = round(load_balance(shapes_all, owners, world, NS_STEPS)["max_over_mean"], 4)
        loads = [0.0] * world  # executed FLOPs, with the form the library picks for each shape
        for shp, o in zip(shapes_all, owners):
            form = engine.lib.muon_ns_choose_algo(shp[0], shp[1], engine.op_dtype, NS_STEPS)
            loads[o] += ns_executed_flops(shp, algo="gram" if form == 1 else "standard")
        executed = round(max(loads) / (sum(loads) / world), 4) if sum(loads) > 0 else 1.0
        owner_balance = {"dense": dense, "executed": executed}
    # the algorithm each shape class ran (the engine's classes, as planned)
    algo_of = {(cs.rows, cs.cols): ("gram" if int(cs.cls.algo) == 1 else "standard") for cs in engine.classes}
    # split operands ("parity") run every product three times (hi*hi, hi*lo, lo*hi)
    my_exec = sum(ns_executed_flops(s, algo=algo_of.get(tuple(s), "standard")) for s in mine) * (
        3 if args.precision == "parity" else 1)
    my_elems = sum(math.prod(s) for s in mine)
    my_ns_ms = per_step("ns")
    ns_tflops = my_flops / (my_ns_ms * 1e-3) / 1e12 if my_ns_ms > 0 else 0.0
    ns_exec_tflops = my_exec / (my_ns_ms * 1e-3) / 1e12 if my_ns_ms > 0 else 0.0
    ns_tflops = -max_over_ranks(-ns_tflops)  # slowest rank
    ns_exec_tflops = -max_over_ranks(-ns_exec_tflops)
    bucket = opt._buckets.get(id(opt.param_groups[1]))
    ag_bytes = bucket.nbytes_received() if bucket is not None else 0
    ag_ms = 0.0
    if bucket is not None:
        # the parameter all-gather alone (same group and CTA limit), once, untimed by the step
        sync_all()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        if hasattr(bucket, "wave_done"):
            bucket.sync()
        else:
            for h in bucket.sync(async_op=True, group=opt._allgather_group(device)):
                h.wait()
        a1.record()
        sync_all()
        ag_ms = max_over_ranks(a0.elapsed_time(a1))
    # one pass per element: grad (bf16) read + exp_avg read and write + the
    # Newton-Schulz operand write (tf32 4 B, bf16 and fp16 2 B); the fix-up of
    # the fp16 path rewrites only matrices whose stored scale no longer fits
    mom_bytes_per_el = {"tf32": 2 + 4 + 4 + 4, "bf16": 2 + 4 + 4 + 2, "fp16": 2 + 4 + 4 + 2,
                        "parity": 2 + 4 + 4 + 4}[args.precision]
    mom_bytes = my_elems * mom_bytes_per_el
    mom_gbs = mom_bytes / (mom_ms * 1e-3) / 1e9 if mom_ms > 0 else 0.0
    adam_elems = sum(math.prod(s) for n, s in spec if not is_muon(n, s))
    adam_shards = opt._adam_shards.get(id(opt.param_groups[0]))
    if adam_shards is not None:  # this rank's element ranges only
        adam_elems = sum(n for _, _, n in adam_shards.owned(list(opt.param_groups[0]["params"])))
    adam_gbs = adam_elems * (2 + 2 + 8 + 8 + 2) / (adam_ms * 1e-3) / 1e9 if adam_ms > 0 else 0.0

    # ---- end-to-end through the public API with host-resident gradients
    # The gradients this rank's step reads: with owner-only momentum a rank
    # never reads the gradients of matrices another rank owns.
    needed = list(range(len(params)))
    if owners is not None and opt.state_sharding:
        owned_ids = {id(p) for p, o in zip(opt.param_groups[1]["params"], owners) if o == rank}
        muon_ids = {id(p) for p in opt.param_groups[1]["params"]}
        needed = [i for i, p in enumerate(params) if id(p) not in muon_ids or id(p) in owned_ids]
    # Element ranges read per gradient: whole tensors, except that with AdamW
    # sharding a rank reads only its ranges of the AdamW gradients.
    spans = {i: [(0, params[i].numel())] for i in needed}
    if adam_shards is not None:
        aparams = list(opt.param_groups[0]["params"])
        index_of = {id(p): i for i, p in enumerate(params)}
        for p in aparams:
            spans[index_of[id(p)]] = []
        for j, start, length in adam_shards.owned(aparams):
            spans[index_of[id(aparams[j])]].append((start, length))
    host_grads = {i: [(a, n, grads[i].reshape(-1)[a:a + n].cpu().pin_memory()) for a, n in sp]
                  for i, sp in spans.items()}
    probe = params[-1] if params[-1].ndim == 1 else params[0]
    readback = torch.empty(min(probe.numel(), 4096), dtype=probe.dtype).pin_memory()
    h2d = sum(t.numel() * t.element_size() for lst in host_grads.values() for *_, t in lst)
    d2h = readback.numel() * readback.element_size()
    e2e_steps = max(2, min(args.steps, 10))
    # Double-buffered input pipeline: step k+1's gradients upload on a copy
    # stream into the other buffer set while step k runs; p.grad is pointed at
    # the step's buffer set (as a data loader would hand over a new batch).
    gbufs = [{i: grads[i] for i in needed}, {i: torch.empty_like(grads[i]) for i in needed}]
    copy_stream = torch.cuda.Stream(device)
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    cur = torch.cuda.current_stream(device)

    def pipeline(n_steps):
        copy_stream.wait_stream(cur)

        def upload(k):
            with torch.cuda.stream(copy_stream):
                if k >= 2:
                    copy_stream.wait_event(free[k % 2])  # step k-2 no longer reads this set
                for i, lst in host_grads.items():
                    flat = gbufs[k % 2][i].view(-1)
                    for a, n, hg in lst:
                        flat[a:a + n].copy_(hg, non_blocking=True)
                ready[k % 2].record(copy_stream)

        upload(0)
        for k in range(n_steps):
            cur.wait_event(ready[k % 2])
            for i in needed:
                params[i].grad = gbufs[k % 2][i]
            opt.step()
            free[k % 2].record(cur)
            readback.copy_(probe.detach().reshape(-1)[: readback.numel()], non_blocking=True)
            # queued after this step's own small host-to-device copies, so the
            # copy engine serves those first and the next upload overlaps the step
            if k + 1 < n_steps:
                upload(k + 1)

    pipeline(2)  # warm-up: one pass per buffer set (first-use host work, table uploads)
    sync_all()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record()
    pipeline(e2e_steps)
    e_end.record()
    sync_all()
    e2e_ms = max_over_ranks(e_start.elapsed_time(e_end) / e2e_steps)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ms, sample = cpu_sample(cfg)
        cpu = {"value": round(ms, 1), "unit": "ms", "cores": cores(), "kind": "port", "sample": sample}

    if rank == 0:
        peak = peaks["bf16_tflops_sustained"]
        line = {
            "metric": "muon_step_ms", "value": round(step_ms, 3), "unit": "ms", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 3),
            "higher_is_better": False, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": args.precision, "data": "synthetic",
            "config": line_config(cfg, args.precision, world, args.adamw_sharding),
            "e2e": {"value": round(e2e_ms, 3), "unit": "ms", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "note": "MuonAdamW.step() with this step's gradients copied in from pinned host memory; the "
                            "updated parameters stay on the device for the next forward pass, as in training, so "
                            "only a 4 KB slice of them is read back"},
            "gpu_launches": int(launches) * args.steps,
            "host_enqueue_ms_per_step": round(host_ms, 3),
            "roofline": {"bound": "tensor", "kernel": f"ns_gemm ({ns_launches} grouped launches per step)",
                         "achieved": round(ns_tflops, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(ns_tflops / peak, 4), "peak_source": f"{peaks['source']} bf16 sustained",
                         "flops": ("algorithmic: the reference's dense count steps*(4 m^2 n + 2 m^3) per matrix / "
                                   "NS time. Above 1.0 because the gram form and the symmetric products execute "
                                   "fewer FLOPs than that count; the tensor-core efficiency is executed_frac"),
                         "executed_tflops": round(ns_exec_tflops, 1),
                         "executed_frac": round(ns_exec_tflops / peak, 4),
                         "executed_flops": ("MMA work issued: 256x256 tiles, K padded to 64, upper-triangle tiles "
                                            "of symmetric products, per the algorithm each class runs"),
                         "executed_tflop_per_step": round(my_exec / 1e12, 2),
                         "ns_algorithms": {f"{r}x{c}": a for (r, c), a in sorted(algo_of.items())},
                         "frac_of_tf32_peak": round(ns_tflops / (peak / 2), 4) if args.precision == "tf32" else None,
                         "mma_kind": "kind::tf32" if args.precision == "tf32" else "kind::f16",
                         "traffic": (NS_TRAFFIC_PER_LAUNCH[cfg] if cfg in NS_TRAFFIC_PER_LAUNCH and world == 1
                                     and args.precision == "fp16" else None),
                         "traffic_unit": "bytes per ns_gemm launch: ncu dram__bytes_read.sum + dram__bytes_write.sum, "
                                         "mean over the 17 launches of one captured step of this configuration",
                         "ns_ms": round(ns_ms, 3)},
            "elementwise": {"momentum_ms": round(mom_ms, 3), "momentum_gbs": round(mom_gbs, 1),
                            "momentum_bytes_per_element": mom_bytes_per_el,
                            "momentum_frac_of_hbm": round(mom_gbs / peaks["hbm_gbs"], 4),
                            "update_ms": round(upd_ms, 3),
                            "update_gbs": round(my_elems * 6 / (upd_ms * 1e-3) / 1e9, 1) if upd_ms > 0 else 0.0,
                            "adamw_ms": round(adam_ms, 3), "adamw_gbs": round(adam_gbs, 1),
                            "hbm_peak_gbs": peaks["hbm_gbs"]},
            "collective": ({"allgather_bytes_received": ag_bytes,
                            "allgather_alone_ms": round(ag_ms, 3),
                            "allgather_alone_gbs": round(ag_bytes / (ag_ms * 1e-3) / 1e9, 1) if ag_ms > 0 else 0.0,
                            "allgather_frac_of_nvlink": (round(ag_bytes / (ag_ms * 1e-3) / 900e9, 4)
                                                         if ag_ms > 0 else 0.0),
                            "nvlink_peak_gbs": 900.0,
                            "waves": bucket.n_waves if bucket is not None else 1,
                            "transport": opt.allgather,
                            "comm_sms": opt.comm_sms if opt.allgather == "nccl" else 0,
                            "wave_ratio": opt.allgather_wave_ratio,
                            "exposed_wait_ms": round(ag_wait_ms, 3),
                            "adamw_allgather_bytes_received": (adam_shards.nbytes_received()
                                                               if adam_shards is not None else 0),
                            "owner_load_max_over_mean": owner_balance}
                           if world > 1 else None),
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c2", choices=["c2", "c2s", "c4", "c5"])
    ap.add_argument("--precision", default="fp16", choices=["fp16", "tf32", "bf16", "parity"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--allgather", default="nccl", choices=["nccl", "p2p"],
                    help="parameter all-gather of the sharded step (N > 1)")
    ap.add_argument("--comm-sms", type=int, default=32, help="SMs left to an overlapping NCCL all-gather")
    ap.add_argument("--waves", type=int, default=None,
                    help="N > 1: all-gather waves per step (default: the optimizer's choice)")
    ap.add_argument("--wave-ratio", type=float, default=0.7,
                    help="N > 1: each wave's FLOP share relative to the wave before (default 0.7)")
    ap.add_argument("--adamw-sharding", action=argparse.BooleanOptionalAction, default=True,
                    help="N > 1: each rank updates an equal range of the AdamW parameters, then all-gather "
                         "(default on; --no-adamw-sharding runs the whole AdamW group on every rank)")
    ap.add_argument("--cpu-full", action="store_true",
                    help="time one full step of the numpy oracle on the host (minutes) and exit")
    args = ap.parse_args(argv)
    if args.cpu_full:
        ms, sample = cpu_full_step(args.config)
        print(json.dumps({"cpu_full_step_ms": round(ms, 1), "config": args.config, "cores": cores(),
                          "sample": sample}), flush=True)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
