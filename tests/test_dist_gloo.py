"""Multi-rank host logic over gloo (world size 2, CPU): the FLOP-balanced
Newton-Schulz sharding with the parameter all-gather, owner-only momentum with
consolidation, FSDP-style flat shards (the reference's owner_only / partial
plans), and a rank that fails mid-step. Arithmetic: the CPU oracle through
tests/oracle_engine.py; every rank must end with the single-process oracle's
result."""

import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import muon_oracle as O

WORLD = 2
# benchmark config 1: 8 fp32 matrices + 4 fp32 vectors of length 512 on AdamW.
C1_MUON = [(512, 512), (512, 2048), (2048, 512), (1024, 1024)] * 2
C1_ADAM = [(512,)] * 4
SMALL_MUON = [(64, 64), (64, 160), (160, 64), (96, 96), (48, 200), (33, 70)]
SMALL_ADAM = [(64,), (10,)]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _data(muon, adam, steps, seed=0, inactive=()):
    """Seeded parameters and per-step gradients; at the steps in `inactive`
    every Muon gradient is None (the Muon group has nothing to do)."""
    rng = np.random.default_rng(seed)
    params = [(rng.standard_normal(s) * 0.02).astype(np.float32) for s in muon + adam]
    grads = [[(rng.standard_normal(s) * 1e-3).astype(np.float32) for s in muon + adam] for _ in range(steps)]
    for st in inactive:
        grads[st][:len(muon)] = [None] * len(muon)
    return params, grads


def _oracle(muon, adam, steps, inactive=()):
    params, grads = _data(muon, adam, steps, inactive=inactive)
    opt = O.OracleMuonAdamW(lr=0.02, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.01)
    mp_ = {str(i): params[i].copy() for i in range(len(muon))}
    ap_ = {str(i): params[i].copy() for i in range(len(muon), len(params))}
    for s in range(steps):
        g = grads[s]
        opt.step(mp_, {str(i): g[i] for i in range(len(muon))}, ap_,
                 {str(i): g[i] for i in range(len(muon), len(params))})
    final = [mp_[str(i)] for i in range(len(muon))] + [ap_[str(i)] for i in range(len(muon), len(params))]
    exp_avg = [opt.muon_state[str(i)].exp_avg for i in range(len(muon))]
    return final, exp_avg


def _oracle_adam_moments(muon, adam, steps):
    """The oracle's AdamW (exp_avg, exp_avg_sq) per AdamW parameter."""
    params, grads = _data(muon, adam, steps)
    opt = O.OracleMuonAdamW(lr=0.02, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.01)
    mp_ = {str(i): params[i].copy() for i in range(len(muon))}
    ap_ = {str(i): params[i].copy() for i in range(len(muon), len(params))}
    for s in range(steps):
        g = grads[s]
        opt.step(mp_, {str(i): g[i] for i in range(len(muon))}, ap_,
                 {str(i): g[i] for i in range(len(muon), len(params))})
    return [(opt.adamw_state[str(i)].exp_avg, opt.adamw_state[str(i)].exp_avg_sq)
            for i in range(len(muon), len(params))]


def _worker(rank, port, scenario, muon, adam, steps, outdir, world=WORLD):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(2)
    from datetime import timedelta

    from opendm_b200.optimizer import MuonAdamW
    from tests.oracle_engine import OracleEngine

    result = {"rank": rank}
    inactive = (1,) if scenario.endswith("_inactive") else ()  # step 1 without Muon gradients
    scenario = scenario.removesuffix("_inactive")
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
        params, grads = _data(muon, adam, steps, inactive=inactive)
        model = torch.nn.Module()
        n_muon = len(muon)
        if scenario in ("replicated", "state_sharding", "fail", "waves", "adam_sharded"):
            for i, p in enumerate(params):
                t = torch.nn.Parameter(torch.from_numpy(p.copy()))
                if i < n_muon:
                    t._opendm_muon_shape = tuple(p.shape)
                    t._opendm_muon_name = f"m{i}"
                model.register_parameter(f"p{i}", t)
            slices = None
        else:  # flat shards ("flat", "flat_ref"): concatenate the Muon matrices, split evenly over the ranks
            sizes = [int(np.prod(s)) for s in muon]
            total = sum(sizes)
            per = (total + world - 1) // world
            lo, hi = rank * per, min((rank + 1) * per, total)
            slices = []
            off = 0
            for i, n in enumerate(sizes):
                a, b = max(lo, off), min(hi, off + n)
                a, b = (a - off, b - off) if b > a else (0, 0)
                slices.append((a, b))
                flat = params[i].reshape(-1)[a:b].copy()
                t = torch.nn.Parameter(torch.from_numpy(flat))
                t._opendm_muon_shape = tuple(muon[i])
                t._opendm_muon_name = f"m{i}"
                model.register_parameter(f"p{i}", t)
                off += n
            for i in range(n_muon, len(params)):
                model.register_parameter(f"p{i}", torch.nn.Parameter(torch.from_numpy(params[i].copy())))
        engine = OracleEngine()
        opt = MuonAdamW(model, lr=0.02, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.01, _engine=engine,
                        state_sharding=(scenario in ("state_sharding", "waves", "adam_sharded", "flat_adam")),
                        adamw_sharding=(scenario in ("adam_sharded", "flat_adam")),
                        max_grad_norm=1.0 if scenario == "flat_clip" else None,
                        allgather_waves=3 if scenario in ("waves", "adam_sharded") else None,
                        fsdp_owner_ns=(scenario != "flat_ref"))
        plist = list(model.parameters())
        order = []  # collective order of the last step (scenario adam_sharded)
        if scenario == "adam_sharded":
            from opendm_b200 import sharding as S

            def rec(cls, tag):
                orig = cls.sync

                def sync(self, *a, **kw):
                    order.append(tag(kw))
                    return orig(self, *a, **kw)
                cls.sync = sync
            rec(S.FlatParamBuckets, lambda kw: f"wave{kw.get('wave')}")
            rec(S.FlatAdamShards, lambda kw: "adamw")
        for s in range(steps):
            order.clear()
            if scenario == "fail" and rank == 1 and s == 1:
                raise SystemExit(3)  # this rank dies between steps
            for i, p in enumerate(plist):
                g = grads[s][i]
                if g is None:
                    p.grad = None
                    continue
                if slices is not None and i < n_muon:
                    a, b = slices[i]
                    g = g.reshape(-1)[a:b]
                p.grad = torch.from_numpy(g.copy())
            opt.step()
        if scenario == "adam_sharded":  # before consolidation: each rank's own ranges only
            result["adam_pieces"] = opt._adam_shards[id(opt.param_groups[0])].owned(list(opt.param_groups[0]["params"]))
        if scenario in ("state_sharding", "waves", "adam_sharded"):
            opt.consolidate_state_dict()
        result["params"] = [p.detach().numpy().copy() for p in plist]
        result["exp_avg"] = [opt.state[p]["exp_avg"].numpy().copy() if "exp_avg" in opt.state[p]
                             else np.zeros(0, np.float32) for p in plist[:n_muon]]
        result["order"] = list(order)
        result["adam_moments"] = [(opt.state[p]["exp_avg"].numpy().copy(), opt.state[p]["exp_avg_sq"].numpy().copy())
                                  for p in plist[n_muon:]]
        result["slices"] = slices
        result["muon_calls"] = engine.matrices_seen
        plans = opt._get_muon_shard_plans(opt.param_groups[1])
        result["kinds"] = [pl.kind for pl in plans]
        result["partial_active"] = [len(pl.active_ranks) for pl in plans if pl.kind == "partial"]
        result["waves"] = opt._waves.get(id(opt.param_groups[1]))
        dist.barrier()
        dist.destroy_process_group()
    except SystemExit:
        result["exited"] = True
    except Exception as exc:  # reported to the parent
        result["error"] = f"{type(exc).__name__}: {exc}"
        result["trace"] = traceback.format_exc()
    torch.save(result, os.path.join(outdir, f"rank{rank}.pt"))


def _run(scenario, muon, adam, steps, tmp_path, world=WORLD):
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, port, scenario, muon, adam, steps, str(tmp_path), world))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
    return [torch.load(os.path.join(tmp_path, f"rank{r}.pt"), weights_only=False) for r in range(world)]


def _check(res, muon, adam, steps, check_exp_avg=True, inactive=()):
    final, exp_avg = _oracle(muon, adam, steps, inactive=inactive)
    for r in res:
        assert "error" not in r, r.get("trace")
        for i, got in enumerate(r["params"]):
            want = final[i]
            if r["slices"] is not None and i < len(muon):
                a, b = r["slices"][i]
                want = want.reshape(-1)[a:b]
            assert O.rel_frobenius(got, want) < 1e-5, (r["rank"], i, O.rel_frobenius(got, want))
        if check_exp_avg:
            for i, got in enumerate(r["exp_avg"]):
                want = exp_avg[i]
                if r["slices"] is not None:
                    a, b = r["slices"][i]
                    want = want.reshape(-1)[a:b]
                assert O.rel_frobenius(got.reshape(-1), want.reshape(-1)) < 1e-6, (r["rank"], i)


def test_c1_sharded_two_ranks(tmp_path):
    """benchmark config 1 on gloo world size 2: each matrix orthogonalised by one
    owner, parameters all-gathered; both ranks equal the single-process oracle."""
    res = _run("replicated", C1_MUON, C1_ADAM, 2, tmp_path)
    _check(res, C1_MUON, C1_ADAM, 2)
    assert all(k == "replicated" for k in res[0]["kinds"])
    assert res[0]["muon_calls"] + res[1]["muon_calls"] == 2 * len(C1_MUON)  # no redundant NS
    assert 0 < res[0]["muon_calls"] < 2 * len(C1_MUON)


def test_allgather_waves_two_ranks(tmp_path):
    """All-gather waves (each rank's matrices cut by FLOPs, one flat bucket
    per wave; here a large matrix fills a wave on its own): same result as
    the single-process oracle."""
    res = _run("waves", C1_MUON + SMALL_MUON, C1_ADAM, 2, tmp_path)
    _check(res, C1_MUON + SMALL_MUON, C1_ADAM, 2)
    assert res[0]["waves"] == res[1]["waves"] and len(set(res[0]["waves"])) >= 2


def test_more_ranks_than_muon_matrices(tmp_path):
    """Replicated parameters on 3 ranks with only 2 Muon matrices: one rank
    owns none, and with 3 waves requested some waves are empty on every rank.
    That rank still takes part in every all-gather (its bucket is padding),
    and every rank ends with the single-process oracle's parameters, in both
    the replicated-state and the owner-only-state (waves) schedules."""
    muon = [(64, 32), (32, 96)]
    adam = [(16,)]
    for scenario in ("replicated", "waves"):
        res = _run(scenario, muon, adam, 2, tmp_path, world=3)
        _check(res, muon, adam, 2)
        assert sum(r["muon_calls"] for r in res) == len(muon) * 2  # each matrix orthogonalised once per step
        assert min(r["muon_calls"] for r in res) == 0


def test_step_without_muon_gradients_on_every_rank(tmp_path):
    """A step in which no rank has a Muon gradient (reference muon_adamw.py:350-360:
    the group is inactive, so momentum, step counts and parameters stay as
    they are while AdamW still steps). The check is reduced on the host
    (gloo), and every rank skips the same collectives: the replicated, the
    owner-only-state (waves) and the FSDP flat-shard schedules all end with
    the single-process oracle's parameters and momentum."""
    muon = SMALL_MUON[:4]
    for scenario in ("replicated", "waves", "flat"):
        res = _run(scenario + "_inactive", muon, SMALL_ADAM, 3, tmp_path)
        _check(res, muon, SMALL_ADAM, 3, inactive=(1,))


def test_owner_only_momentum_consolidates(tmp_path):
    res = _run("state_sharding", SMALL_MUON, SMALL_ADAM, 3, tmp_path)
    _check(res, SMALL_MUON, SMALL_ADAM, 3)


def test_adamw_sharding_two_three_and_four_ranks(tmp_path):
    """adamw_sharding: each rank updates an equal contiguous range of the
    flat AdamW parameters (a vector split between ranks, whole small ones),
    the ranges are all-gathered, and consolidation brings the moments
    together; parameters and moments equal the single-process oracle."""
    adam = [(5000,), (10,), (700,), (3,)]
    muon = C1_MUON[:4] + SMALL_MUON  # three Muon waves: the ranges' all-gather goes between waves 0 and 1
    for world in (2, 3, 4):
        res = _run("adam_sharded", muon, adam, 3, tmp_path, world=world)
        _check(res, muon, adam, 3)
        assert len(set(res[0]["waves"])) >= 2
        for r in res:  # the ranges' all-gather is queued right after wave 0's
            assert r["order"][0] == "wave0" and r["order"][1] == "adamw", r["order"]
            assert r["order"].count("adamw") == 1
        want = _oracle_adam_moments(muon, adam, 3)
        for r in res:
            for (m, v), (wm, wv) in zip(r["adam_moments"], want, strict=True):
                assert O.rel_frobenius(m, wm) < 1e-6 and O.rel_frobenius(v, wv) < 1e-6, r["rank"]
        pieces = [r["adam_pieces"] for r in res]
        assert all(pieces)  # every rank owns a range
        covered = {}
        for ps in pieces:
            for i, start, length in ps:
                covered.setdefault(i, []).append((start, length))
        for i, shape in enumerate(adam):  # the ranges tile every parameter exactly once
            spans = sorted(covered[i])
            assert spans[0][0] == 0 and sum(n for _, n in spans) == shape[0]
            assert all(a + n == b for (a, n), (b, _) in zip(spans, spans[1:]))
        assert len(covered[0]) >= 2  # the long vector is split between ranks


def test_adamw_sharding_refuses_fsdp_shards(tmp_path):
    """adamw_sharding with Muon matrices in FSDP-style flat shards: the first
    step raises on every rank (the AdamW parameters may be shards too, even
    where their sizes and checksums agree)."""
    res = _run("flat_adam", SMALL_MUON, SMALL_ADAM, 1, tmp_path)
    for r in res:
        assert "adamw_sharding needs replicated parameters" in r.get("error", ""), r


def test_max_grad_norm_refuses_fsdp_shards(tmp_path):
    """max_grad_norm with Muon matrices in FSDP-style flat shards: a local
    norm would clip by the wrong total, so step() raises on every rank."""
    res = _run("flat_clip", SMALL_MUON, SMALL_ADAM, 1, tmp_path)
    for r in res:
        assert "max_grad_norm needs parameters replicated" in r.get("error", ""), r


def test_flat_shards_partial_and_owner_only(tmp_path):
    """FSDP-style flat shards: each matrix split over both ranks is
    orthogonalised once, by its owner (direction shards in, update shards
    out through two all-to-alls); same result as the single-process oracle."""
    res = _run("flat", SMALL_MUON, SMALL_ADAM, 2, tmp_path)
    kinds = set(res[0]["kinds"]) | set(res[1]["kinds"])
    assert "partial" in kinds and ("owner_only" in kinds or "empty" in kinds)
    _check(res, SMALL_MUON, SMALL_ADAM, 2)
    assert res[0]["muon_calls"] + res[1]["muon_calls"] == len(SMALL_MUON) * 2  # once per matrix and step


def test_flat_shards_three_ranks(tmp_path):
    """World size 3: matrices split over two of the three ranks (the third
    has no shard of them, and some ranks own nothing), plus whole-matrix
    owners; every rank takes part in both all-to-alls."""
    muon = SMALL_MUON + [(40, 90), (128, 64)]
    res = _run("flat", muon, SMALL_ADAM, 2, tmp_path, world=3)
    _check(res, muon, SMALL_ADAM, 2)
    assert sum(r["muon_calls"] for r in res) == len(muon) * 2
    kinds = set().union(*(set(r["kinds"]) for r in res))
    assert {"partial", "owner_only"} <= kinds
    assert min(res[0]["partial_active"]) < 3  # some split matrix has a rank without a shard


def test_flat_shards_reference_gather_everywhere(tmp_path):
    """fsdp_owner_ns=False: the reference's schedule (every active rank
    gathers the direction and orthogonalises the whole matrix)."""
    res = _run("flat_ref", SMALL_MUON, SMALL_ADAM, 2, tmp_path)
    _check(res, SMALL_MUON, SMALL_ADAM, 2)


def test_rank_failure_surfaces_as_error(tmp_path):
    """A rank that exits between steps: the surviving rank's next collective
    raises instead of hanging (host-side failure detection)."""
    res = _run("fail", SMALL_MUON, SMALL_ADAM, 3, tmp_path)
    assert res[1].get("exited")
    assert "error" in res[0], "surviving rank should report a collective error"


def _bad_shards_worker(rank, port, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    from opendm_b200.optimizer import MuonAdamW
    from tests.oracle_engine import OracleEngine

    result = {"rank": rank}
    try:
        dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=20))
        model = torch.nn.Module()
        p = torch.nn.Parameter(torch.zeros(6))  # 6 + 6 elements of a 4 x 4 matrix: neither shards nor copies
        p._opendm_muon_shape, p._opendm_muon_name = (4, 4), "w"
        model.register_parameter("w", p)
        opt = MuonAdamW(model, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, _engine=OracleEngine())
        p.grad = torch.zeros(6)
        opt.step()
    except Exception as exc:
        result["error"] = f"{type(exc).__name__}: {exc}"
    torch.save(result, os.path.join(outdir, f"rank{rank}.pt"))


def test_unreconstructable_shard_sizes_raise(tmp_path):
    """Reference :487-491: local sizes that are neither a split of the matrix
    nor full copies raise on every rank."""
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_bad_shards_worker, args=(r, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
    for r in range(2):
        res = torch.load(os.path.join(tmp_path, f"rank{r}.pt"), weights_only=False)
        assert "cannot be reconstructed from local shard sizes (6, 6)" in res.get("error", ""), res


def _checkpoint_worker(rank, port, outdir, world=WORLD):
    """Save after one step the way the HF Trainer does (rank 0 writes
    optimizer.state_dict() with torch.save, after consolidate_state_dict() on
    every rank), resume a fresh optimizer on every rank from that file
    (torch.load, weights_only), and continue: bit-identical to the run that
    never stopped."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(2)
    from datetime import timedelta

    from opendm_b200.optimizer import MuonAdamW
    from tests.oracle_engine import OracleEngine

    result = {"rank": rank}
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
        muon, adam, steps = SMALL_MUON, SMALL_ADAM, 3
        params, grads = _data(muon, adam, steps)

        def build(values):
            model = torch.nn.Module()
            for i, p in enumerate(values):
                t = torch.nn.Parameter(torch.from_numpy(np.array(p, np.float32, copy=True)))
                if i < len(muon):
                    t._opendm_muon_shape = tuple(muon[i])
                    t._opendm_muon_name = f"m{i}"
                model.register_parameter(f"p{i}", t)
            opt = MuonAdamW(model, lr=0.02, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.01, _engine=OracleEngine(),
                            state_sharding=True, adamw_sharding=True)
            return model, opt

        def step(model, opt, s):
            for i, p in enumerate(model.parameters()):
                p.grad = torch.from_numpy(grads[s][i].copy())
            opt.step()

        ma, oa = build(params)
        step(ma, oa, 0)
        oa.consolidate_state_dict()  # every rank, before rank 0 saves
        path = os.path.join(outdir, "optimizer.pt")
        if rank == 0:
            torch.save(oa.state_dict(), path)
        dist.barrier()
        mb, ob = build([p.detach().numpy() for p in ma.parameters()])
        ob.load_state_dict(torch.load(path, map_location="cpu", weights_only=True))
        for s in range(1, steps):
            step(ma, oa, s)
            step(mb, ob, s)
        oa.consolidate_state_dict()
        ob.consolidate_state_dict()
        result["same_params"] = all(torch.equal(a, b) for a, b in zip(ma.parameters(), mb.parameters()))
        sa, sb = oa.state_dict()["state"], ob.state_dict()["state"]
        result["same_state"] = sa.keys() == sb.keys() and all(
            torch.equal(sa[k][f], sb[k][f]) for k in sa for f in ("exp_avg", "exp_avg_sq", "step"))
        result["params"] = [p.detach().numpy().copy() for p in mb.parameters()]
        result["exp_avg"] = [ob.state[p]["exp_avg"].numpy().copy() for p in list(mb.parameters())[:len(muon)]]
        result["slices"] = None
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent
        result["error"] = f"{type(exc).__name__}: {exc}"
        result["trace"] = traceback.format_exc()
    torch.save(result, os.path.join(outdir, f"rank{rank}.pt"))


def test_checkpoint_save_resume_continues_bit_identically(tmp_path):
    """State sharding (owner-only momentum) with AdamW sharding, saved as the
    HF Trainer saves an optimizer (torch.save of rank 0's state_dict() after
    consolidate_state_dict()) and resumed on every rank (torch.load with
    weights_only=True, load_state_dict): the two continuations agree bit for
    bit and equal the single-process oracle (reference muon_adamw.py:240-317
    for the state layout; trainer save/resume, opendm/exp/dm05_exp.py:1625)."""
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_checkpoint_worker, args=(r, port, str(tmp_path))) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
    res = [torch.load(os.path.join(tmp_path, f"rank{r}.pt"), weights_only=False) for r in range(WORLD)]
    for r in res:
        assert "error" not in r, r.get("trace")
        assert r["same_params"] and r["same_state"], r["rank"]
    _check(res, SMALL_MUON, SMALL_ADAM, 3)
