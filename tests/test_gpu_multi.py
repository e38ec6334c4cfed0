"""Two GPUs over NCCL: the FLOP-balanced Newton-Schulz sharding (each matrix
orthogonalised by one owner rank, the updated parameters all-gathered into
flat per-dtype buckets) gives bit-identical parameters to every rank running
every matrix (sharding="off", the reference's redundant schedule), with every
momentum buffer current (state_sharding=False), with owner-only momentum
consolidated afterwards (state_sharding=True), with the all-gather split
into waves that overlap the Newton-Schulz of the next wave, over NCCL or over
copy engines out of peer-mapped buffers (allgather="p2p"), and with the
AdamW group split into per-rank element ranges (adamw_sharding=True).

Bitwise equality holds because each matrix's kernels see the same inputs in
both schedules and every reduction (momentum norm partials, tile K order) is
deterministic per matrix. Needs two CUDA devices; skipped otherwise."""

import os
import socket
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2
# One benchmark config 2 decoder layer (q/o, k/v, gate/up, down) plus a tall
# and a ragged matrix, bf16 parameters, and AdamW vectors.
MUON = [(2048, 2048), (256, 2048), (256, 2048), (2048, 2048), (8192, 2048), (8192, 2048), (2048, 8192),
        (1000, 300), (72, 130)]
ADAM = [(2048,), (2048,), (37,)]
STEPS = 2
# (name, sharding, state_sharding, waves, allgather); "adamw_sharded" also
# splits the AdamW parameters into per-rank element ranges.
RUNS = (("off", "off", False, None, "nccl"),
        ("auto", "auto", False, None, "nccl"),
        ("auto_owner", "auto", True, None, "nccl"),
        ("waves", "auto", True, 3, "nccl"),
        ("p2p", "auto", True, 3, "p2p"),
        ("p2p_replicated_state", "auto", False, 2, "p2p"),
        ("adamw_sharded", "auto", True, 3, "nccl"))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _build(dev, sharding, state_sharding, waves=None, allgather="nccl", adamw_sharding=False):
    from opendm_b200.optimizer import MuonAdamW

    g = torch.Generator(device=dev).manual_seed(11)
    model = torch.nn.Module()
    for i, shape in enumerate(MUON + ADAM):
        t = torch.nn.Parameter((torch.randn(shape, generator=g, device=dev) * 0.02).to(torch.bfloat16))
        if i < len(MUON):
            t._opendm_muon_shape = tuple(shape)
            t._opendm_muon_name = f"m{i}"
        model.register_parameter(f"p{i}", t)
    opt = MuonAdamW(model, lr=0.02, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.01, sharding=sharding,
                    state_sharding=state_sharding, allgather_waves=waves, allgather=allgather,
                    adamw_sharding=adamw_sharding)
    return model, opt


def _worker(rank, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta

    import torch.distributed as dist

    result = {"rank": rank}
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60), device_id=dev)
        runs = {}
        for name, sharding, state_sharding, waves, ag in RUNS:
            model, opt = _build(dev, sharding, state_sharding, waves, ag, adamw_sharding=name == "adamw_sharded")
            gg = torch.Generator(device=dev).manual_seed(12)
            for _ in range(STEPS):
                for p in model.parameters():
                    p.grad = (torch.randn(p.shape, generator=gg, device=dev) * 1e-3).to(torch.bfloat16)
                opt.step()
            opt.consolidate_state_dict()
            opt.check_device_errors()
            owners = opt._owners.get(id(opt.param_groups[1]))
            runs[name] = {"params": [p.detach().cpu() for p in model.parameters()],
                          "exp_avg": [opt.state[p]["exp_avg"].cpu() for p in opt.param_groups[1]["params"]],
                          "adam_moments": [(opt.state[p]["exp_avg"].cpu(), opt.state[p]["exp_avg_sq"].cpu())
                                           for p in opt.param_groups[0]["params"]],
                          "owners": owners}
        result["runs"] = runs
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent
        result["error"] = f"{type(exc).__name__}: {exc}"
        result["trace"] = traceback.format_exc()
    torch.save(result, os.path.join(outdir, f"rank{rank}.pt"))


def test_two_gpu_sharded_equals_unsharded(tmp_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < WORLD:
        pytest.skip("needs two CUDA devices")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, port, str(tmp_path))) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
    res = [torch.load(os.path.join(tmp_path, f"rank{r}.pt"), weights_only=False) for r in range(WORLD)]
    for r in res:
        assert "error" not in r, r.get("trace")
    ref = res[0]["runs"]["off"]
    owners = res[0]["runs"]["auto"]["owners"]
    assert owners is not None and set(owners) == {0, 1}  # both ranks own work
    for r in res:
        for name, *_ in RUNS:
            run = r["runs"][name]
            for i, (got, want) in enumerate(zip(run["params"], ref["params"])):
                assert torch.equal(got, want), (r["rank"], name, "param", i)
            for i, (got, want) in enumerate(zip(run["exp_avg"], ref["exp_avg"])):
                assert torch.equal(got, want), (r["rank"], name, "exp_avg", i)
            for i, (got, want) in enumerate(zip(run["adam_moments"], ref["adam_moments"])):
                assert torch.equal(got[0], want[0]) and torch.equal(got[1], want[1]), (r["rank"], name, "adam", i)


def _flat_worker(rank, port, outdir):
    """Each rank holds FSDP-style flat shards (the concatenated Muon matrices
    split evenly over the ranks): owner-only and reference (gather
    everywhere) schedules, and the unsharded model for comparison."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta

    import torch.distributed as dist

    from opendm_b200.optimizer import MuonAdamW

    result = {"rank": rank}
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60), device_id=dev)
        g = torch.Generator(device=dev).manual_seed(21)
        full = [(torch.randn(s, generator=g, device=dev) * 0.02).to(torch.bfloat16) for s in MUON]
        grads = [[(torch.randn(s, generator=g, device=dev) * 1e-3).to(torch.bfloat16) for s in MUON]
                 for _ in range(STEPS)]
        sizes = [int(torch.tensor(s).prod()) for s in MUON]
        total = sum(sizes)
        per = (total + WORLD - 1) // WORLD
        lo, hi = rank * per, min((rank + 1) * per, total)
        slices, off = [], 0
        for n in sizes:
            a, b = max(lo, off), min(hi, off + n)
            slices.append((a - off, b - off) if b > a else (0, 0))
            off += n
        runs = {}
        for name in ("owner", "reference", "full"):
            model = torch.nn.Module()
            for i, (t, shape) in enumerate(zip(full, MUON)):
                a, b = slices[i]
                data = t.clone() if name == "full" else t.reshape(-1)[a:b].clone()
                prm = torch.nn.Parameter(data)
                prm._opendm_muon_shape = tuple(shape)
                prm._opendm_muon_name = f"m{i}"
                model.register_parameter(f"p{i}", prm)
            opt = MuonAdamW(model, lr=0.02, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.01,
                            sharding="off", fsdp_owner_ns=(name == "owner"))
            for s in range(STEPS):
                for i, prm in enumerate(model.parameters()):
                    a, b = slices[i]
                    prm.grad = grads[s][i].clone() if name == "full" else grads[s][i].reshape(-1)[a:b].clone()
                opt.step()
            opt.check_device_errors()
            kinds = [p.kind for p in opt._get_muon_shard_plans(opt.param_groups[1])]
            runs[name] = {"params": [p.detach().reshape(-1).cpu() for p in model.parameters()], "kinds": kinds}
        result.update(runs=runs, slices=slices)
        if rank == 0:  # the inputs, for the oracle run in the parent
            result["host"] = {"full": [t.float().cpu() for t in full],
                              "grads": [[t.float().cpu() for t in gs] for gs in grads]}
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent
        result["error"] = f"{type(exc).__name__}: {exc}"
        result["trace"] = traceback.format_exc()
    torch.save(result, os.path.join(outdir, f"flat{rank}.pt"))


def test_two_gpu_flat_shards_owner_ns_equals_unsharded(tmp_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < WORLD:
        pytest.skip("needs two CUDA devices")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_flat_worker, args=(r, port, str(tmp_path))) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
    res = [torch.load(os.path.join(tmp_path, f"flat{r}.pt"), weights_only=False) for r in range(WORLD)]
    for r in res:
        assert "error" not in r, r.get("trace")
        assert "partial" in r["runs"]["owner"]["kinds"]
        for name in ("owner", "reference"):
            for i, (got, want) in enumerate(zip(r["runs"][name]["params"], r["runs"]["full"]["params"])):
                a, b = r["slices"][i]
                assert torch.equal(got, want[a:b]), (r["rank"], name, i)
    # and the unsharded run (which both shard schedules equal bit for bit) is
    # the reference's step: the CPU oracle on the same inputs, bf16 parameters
    # within the bf16 floor over two steps (tests/test_gpu_optimizer.py)
    import numpy as np

    from oracle import muon_oracle as O

    host = res[0]["host"]
    ref = O.OracleMuonAdamW(lr=0.02, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.01)
    want = {str(i): host["full"][i].numpy().copy() for i in range(len(MUON))}
    for s in range(STEPS):
        ref.step(want, {str(i): host["grads"][s][i].numpy() for i in range(len(MUON))}, {}, {},
                 param_dtype="bfloat16", device_semantics="cuda")
    for i, shape in enumerate(MUON):
        got = res[0]["runs"]["full"]["params"][i].float().numpy().reshape(shape)
        err = O.rel_frobenius(got, want[str(i)])
        assert err < 2e-3 * np.sqrt(STEPS), (i, shape, err)
