"""GPU parity of the sm_100a kernels against the CPU oracle (and through it,
the reference). Every call goes through the C ABI (libopendm_muon.so).

Tolerances (relative Frobenius error vs the fp32 reference math):
  orthogonalised update U: tf32 and fp16 modes < 5e-3 on Gaussian inputs,
  < 1e-2 (the bar) on structured spectra; bf16 mode < 3e-2
  exp_avg: bit-exact (same fp32 operations)
  direction (stored NS operand): within tf32 / bf16 rounding of the fp32 value
"""

import os

import numpy as np
import pytest
import torch

from oracle import muon_oracle as O

pytestmark = pytest.mark.gpu

TF32_TOL = 5e-3
BF16_TOL = 3e-2


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


@pytest.fixture(scope="module")
def engine():
    from opendm_b200.engine import CudaMuonEngine

    return CudaMuonEngine(_dev(), "tf32")


@pytest.fixture(scope="module")
def engine_fp16():
    from opendm_b200.engine import CudaMuonEngine

    return CudaMuonEngine(_dev(), "fp16")


@pytest.fixture(scope="module")
def engine_bf16():
    from opendm_b200.engine import CudaMuonEngine

    return CudaMuonEngine(_dev(), "bf16")


def _rand(shape, seed, scale=1e-3):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g) * scale


SHAPES = [(64, 64), (48, 96), (96, 48), (33, 70), (70, 33), (1, 16), (128, 32), (256, 256), (130, 300),
          (300, 130), (512, 2048), (2048, 512), (384, 1152), (1152, 384), (1000, 1000)]


@pytest.mark.parametrize("shape", SHAPES)
def test_orthogonalize_matches_oracle_tf32(engine, shape):
    x = _rand(shape, hash(shape) % 1000) * 1.95
    got = engine.orthogonalize(x.to(engine.device)).cpu().numpy()
    torch.cuda.synchronize()
    engine.check_errors(block=True)
    ref = O.zeropower_via_newtonschulz5(x.numpy())
    err = O.rel_frobenius(got, ref)
    assert got.shape == ref.shape
    assert err < TF32_TOL, err


@pytest.mark.parametrize("shape", SHAPES)
def test_orthogonalize_matches_oracle_fp16(engine_fp16, shape):
    x = _rand(shape, hash(shape) % 1000) * 1.95
    got = engine_fp16.orthogonalize(x.to(engine_fp16.device)).cpu().numpy()
    engine_fp16.check_errors(block=True)
    err = O.rel_frobenius(got, O.zeropower_via_newtonschulz5(x.numpy()))
    assert err < TF32_TOL, err


def test_fp16_small_gradients_stay_accurate(engine_fp16):
    """Gradients of 1e-7 would be fp16 subnormals: the input is normalised and
    power-of-two scaled before rounding, so accuracy does not depend on scale."""
    x = _rand((256, 512), 9) * 1e-4
    got = engine_fp16.orthogonalize(x.to(engine_fp16.device)).cpu().numpy()
    assert O.rel_frobenius(got, O.zeropower_via_newtonschulz5(x.numpy())) < TF32_TOL


def test_fp16_golden_and_degenerate_cases(engine_fp16, golden_dir):
    z = np.load(os.path.join(golden_dir, "ns_cases.npz"))
    for i in range(int(z["n_cases"])):
        x = torch.from_numpy(z[f"in{i}"]).to(engine_fp16.device)
        got = engine_fp16.orthogonalize(x, steps=int(z[f"steps{i}"])).cpu().numpy()
        assert O.rel_frobenius(got, z[f"out{i}"]) < TF32_TOL, i
    for key in ("zero", "inf"):
        got = engine_fp16.orthogonalize(torch.from_numpy(z[f"in_{key}"]).to(engine_fp16.device)).cpu().numpy()
        assert not got.any(), key


@pytest.mark.parametrize("shape", [(64, 64), (96, 48), (512, 2048), (2048, 512), (130, 300)])
def test_orthogonalize_matches_oracle_bf16(engine_bf16, shape):
    x = _rand(shape, 7) * 1.95
    got = engine_bf16.orthogonalize(x.to(engine_bf16.device)).cpu().numpy()
    engine_bf16.check_errors(block=True)
    err = O.rel_frobenius(got, O.zeropower_via_newtonschulz5(x.numpy()))
    assert err < BF16_TOL, err


def test_orthogonalize_golden_cases(engine, golden_dir):
    z = np.load(os.path.join(golden_dir, "ns_cases.npz"))
    for i in range(int(z["n_cases"])):
        x = torch.from_numpy(z[f"in{i}"]).to(engine.device)
        got = engine.orthogonalize(x, steps=int(z[f"steps{i}"])).cpu().numpy()
        assert O.rel_frobenius(got, z[f"out{i}"]) < TF32_TOL, i
    for key in ("zero", "inf"):
        got = engine.orthogonalize(torch.from_numpy(z[f"in_{key}"]).to(engine.device)).cpu().numpy()
        assert not got.any(), key
    engine.check_errors(block=True)


_ENGINES = {}


def _engine_for(precision, algo):
    from opendm_b200.engine import CudaMuonEngine

    key = (precision, algo)
    if key not in _ENGINES:
        _ENGINES[key] = CudaMuonEngine(_dev(), precision, algo)
    return _ENGINES[key]


ALGO_SHAPES = [(1, 16), (33, 70), (70, 33), (64, 64), (130, 300), (300, 130), (256, 2560), (2560, 256),
               (512, 2048), (2048, 512), (1000, 1000)]


@pytest.mark.parametrize("shape", ALGO_SHAPES)
@pytest.mark.parametrize("precision,algo", [("fp16", "standard"), ("fp16", "gram"), ("tf32", "standard"),
                                            ("tf32", "gram")])
def test_orthogonalize_each_algorithm(precision, algo, shape):
    """Both Newton-Schulz forms (iteration on X; iteration on the gram matrix
    with a restart every 3 iterations) in both 11-bit operand types, forced
    regardless of which one the library would pick for the shape."""
    eng = _engine_for(precision, algo)
    x = _rand(shape, sum(shape)) * 1.95
    got = eng.orthogonalize(x.to(eng.device)).cpu().numpy()
    eng.check_errors(block=True)
    err = O.rel_frobenius(got, O.zeropower_via_newtonschulz5(x.numpy()))
    assert err < TF32_TOL, err


@pytest.mark.parametrize("precision,algo", [("fp16", "standard"), ("fp16", "gram"), ("tf32", "gram")])
def test_orthogonalize_steps_variants(engine, precision, algo):
    """Iteration counts that give the gram form segments of 1, 2 and 3
    iterations, one or several restarts."""
    eng = _engine_for(precision, algo)
    x = _rand((80, 200), 3)
    for steps in (0, 1, 2, 3, 4, 5, 7):
        got = eng.orthogonalize(x.to(eng.device), steps=steps).cpu().numpy()
        ref = O.zeropower_via_newtonschulz5(x.numpy(), steps=steps)
        assert O.rel_frobenius(got, ref) < TF32_TOL, steps


def _structured(shape, kind, seed):
    """Gradient-like inputs with structured spectra (numpy, fp32)."""
    rng = np.random.default_rng(seed)
    m, n = shape
    g = rng.standard_normal(shape)
    if kind == "rank4_noise":
        return (0.1 * g + rng.standard_normal((m, 4)) @ rng.standard_normal((4, n))).astype(np.float32)
    k = min(shape)
    u, _ = np.linalg.qr(rng.standard_normal((m, k)))
    v, _ = np.linalg.qr(rng.standard_normal((n, k)))
    s = np.arange(1, k + 1) ** -1.0 if kind == "powerlaw" else np.exp(-np.arange(k) / (k / 10))
    return ((u * s) @ v.T).astype(np.float32)


@pytest.mark.parametrize("kind", ["rank4_noise", "powerlaw", "expdecay"])
@pytest.mark.parametrize("shape", [(512, 2048), (2048, 512)])
def test_structured_spectra_both_algorithms(kind, shape):
    """Low-rank-plus-noise, power-law and exponentially decaying spectra: both
    forms within the 1e-2 update bar of the fp32 reference, and within 2x of
    each other (the gram form's restart keeps it from drifting)."""
    x = _structured(shape, kind, 21)
    ref = O.zeropower_via_newtonschulz5(x)
    errs = {}
    for algo in ("standard", "gram"):
        eng = _engine_for("fp16", algo)
        got = eng.orthogonalize(torch.from_numpy(x).to(eng.device)).cpu().numpy()
        errs[algo] = O.rel_frobenius(got, ref)
    assert max(errs.values()) < 1e-2, errs
    assert errs["gram"] < 2 * errs["standard"] + 1e-3, errs


def test_orthogonalize_heavy_tail(engine):
    g = torch.Generator().manual_seed(11)
    x = torch.randn(1024, 1024, generator=g) * 1e-3
    mask = torch.rand(1024, 1024, generator=g) < 0.01
    x[mask] = torch.randn(int(mask.sum()), generator=g) * 1e-1
    got = engine.orthogonalize(x.to(engine.device)).cpu().numpy()
    assert O.rel_frobenius(got, O.zeropower_via_newtonschulz5(x.numpy())) < TF32_TOL


def test_orthogonalize_bf16_input(engine):
    x = _rand((256, 512), 5).to(torch.bfloat16)
    got = engine.orthogonalize(x.to(engine.device)).cpu().numpy()
    ref = O.zeropower_via_newtonschulz5(x.float().numpy())
    assert O.rel_frobenius(got, ref) < TF32_TOL


def _items(shapes, dtype, seed, device, with_grad=True):
    from opendm_b200.engine import MatrixItem

    items, host = [], []
    for i, s in enumerate(shapes):
        p = _rand(s, seed + i, 0.02).to(dtype)
        g = _rand(s, seed + 100 + i, 1e-3).to(dtype)
        m = _rand(s, seed + 200 + i, 1e-3)
        items.append(MatrixItem(p.to(device), g.to(device) if with_grad else None, m.clone().to(device),
                                O.effective_lr(0.02, 1.0, 0.2, s)))
        host.append((p.float().numpy(), g.float().numpy() if with_grad else None, m.numpy()))
    return items, host


@pytest.mark.parametrize("mode", ["tf32", "fp16"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_full_matrix_step_grouped(engine, engine_fp16, dtype, mode):
    """Several shape classes (wide, tall, square, repeated) in one grouped plan:
    momentum, Newton-Schulz and the fused weight decay + update."""
    engine = engine if mode == "tf32" else engine_fp16
    shapes = [(256, 256), (256, 256), (128, 512), (512, 128), (512, 128), (96, 160), (64, 64)]
    items, host = _items(shapes, dtype, 10, engine.device)
    lr, wd = 0.02, 0.01
    engine.muon_matrices(items, momentum=0.95, nesterov=True, weight_decay_factor=1 - lr * wd, ns_steps=5)
    torch.cuda.synchronize()
    engine.check_errors(block=True)
    pdt = "bfloat16" if dtype == torch.bfloat16 else "float32"
    for it, (p, g, m) in zip(items, host):
        m_ref, d = O.momentum_direction(g, m, 0.95, True)
        np.testing.assert_array_equal(it.exp_avg.cpu().numpy(), m_ref)
        u = O.zeropower_via_newtonschulz5(d)
        p_ref = O.apply_update(p, u, lr=lr, weight_decay=wd, eff=it.eff, param_dtype=pdt, device_semantics="cuda")
        got = it.param.float().cpu().numpy()
        # parameters: fp32 within the 1e-3 bar; bf16 within its rounding floor
        # (one-ulp flips, see test_gpu_optimizer.py)
        tol = 1e-3 if dtype == torch.float32 else 2e-3
        assert O.rel_frobenius(got, p_ref) < tol, O.rel_frobenius(got, p_ref)
        # the update itself, recovered from the parameter change (fp32 only)
        if dtype == torch.float32:
            p_wd = p * np.float32(1 - lr * wd)
            u_got = (p_wd - got) / np.float32(it.eff)
            assert O.rel_frobenius(u_got, u) < TF32_TOL


def test_second_step_uses_momentum(engine):
    shapes = [(128, 256), (256, 128)]
    items, host = _items(shapes, torch.float32, 40, engine.device)
    for _ in range(2):
        engine.muon_matrices(items, momentum=0.95, nesterov=True, weight_decay_factor=1.0, ns_steps=5)
    torch.cuda.synchronize()
    for it, (p, g, m) in zip(items, host):
        m1, _ = O.momentum_direction(g, m, 0.95, True)
        m2, _ = O.momentum_direction(g, m1, 0.95, True)
        np.testing.assert_array_equal(it.exp_avg.cpu().numpy(), m2)


def test_absent_grad_and_plain_momentum(engine):
    shapes = [(64, 128), (128, 64)]
    items, host = _items(shapes, torch.float32, 60, engine.device, with_grad=False)
    engine.muon_matrices(items, momentum=0.9, nesterov=False, weight_decay_factor=1.0, ns_steps=5)
    torch.cuda.synchronize()
    for it, (p, g, m) in zip(items, host):
        m_ref, d = O.momentum_direction(None, m, 0.9, False)
        np.testing.assert_array_equal(it.exp_avg.cpu().numpy(), m_ref)
        u = O.zeropower_via_newtonschulz5(d)
        p_ref = O.apply_update(p, u, lr=0.02, weight_decay=0.0, eff=it.eff, param_dtype="float32")
        assert O.rel_frobenius(it.param.cpu().numpy(), p_ref) < 1e-3


def test_momentum_only(engine):
    from opendm_b200.engine import MatrixItem

    g = _rand((300, 77), 1).to(engine.device)
    m = _rand((300, 77), 2).to(engine.device)
    ref, _ = O.momentum_direction(g.cpu().numpy(), m.cpu().numpy(), 0.95, True)
    engine.momentum_only([MatrixItem(torch.empty(0), g, m, 0.0)], momentum=0.95, nesterov=True)
    np.testing.assert_array_equal(m.cpu().numpy(), ref)


@pytest.mark.parametrize("pdt,gdt", [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16),
                                     (torch.bfloat16, torch.float32)])
def test_adamw_matches_oracle(engine, pdt, gdt):
    from opendm_b200.engine import AdamItem

    shapes = [(1000,), (64, 33), (4096,), (7,)]
    items, host = [], []
    for i, s in enumerate(shapes):
        p = _rand(s, 300 + i, 0.02).to(pdt)
        g = _rand(s, 400 + i, 1e-3).to(gdt)
        items.append(AdamItem(p.to(engine.device), g.to(engine.device), torch.zeros(s, device=engine.device),
                              torch.zeros(s, device=engine.device), 1.0))
        host.append((p.float().numpy(), g.float().numpy()))
    engine.adamw(items, lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.01)
    torch.cuda.synchronize()
    name = "bfloat16" if pdt == torch.bfloat16 else "float32"
    for it, (p, g) in zip(items, host):
        z = np.zeros_like(p)
        p_ref, m_ref, v_ref, _ = O.adamw_step(p, g, z, z, 0.0, lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8,
                                              weight_decay=0.01, param_dtype=name)
        assert O.rel_frobenius(it.exp_avg.cpu().numpy(), m_ref) < 1e-6
        assert O.rel_frobenius(it.exp_avg_sq.cpu().numpy(), v_ref) < 1e-6
        assert O.rel_frobenius(it.param.float().cpu().numpy(), p_ref) < (1e-3 if pdt == torch.bfloat16 else 1e-6)


def test_adamw_cached_table_over_steps(engine):
    """Three AdamW steps with a changing lr: items sharing one step count use
    the device-cached table with the step size and bias correction filled in
    place; the same items next to one a step ahead use an uploaded table.
    Bit-identical every step, and equal to the oracle at the end."""
    from opendm_b200.engine import AdamItem

    shapes = [(1000,), (64, 33), (4096,), (7,)]
    init = [(_rand(s, 500 + i, 0.02).to(torch.bfloat16), _rand(s, 600 + i, 1e-3).to(torch.bfloat16))
            for i, s in enumerate(shapes)]

    def fresh():
        return [[p.to(engine.device), g.to(engine.device), torch.zeros(p.shape, device=engine.device),
                 torch.zeros(p.shape, device=engine.device)] for p, g in init]

    a, b = fresh(), fresh()
    extra = [t.clone() for t in a[0]]
    host = [(p.float().numpy(), g.float().numpy(), np.zeros(p.shape, np.float32), np.zeros(p.shape, np.float32))
            for p, g in init]
    for step in (1, 2, 3):
        lr = 1e-3 * step
        engine.adamw([AdamItem(*t, float(step)) for t in a], lr=lr, beta1=0.9, beta2=0.95, eps=1e-8,
                     weight_decay=0.01)
        engine.adamw([AdamItem(*t, float(step)) for t in b] + [AdamItem(*extra, float(step + 1))], lr=lr,
                     beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.01)
        torch.cuda.synchronize()
        for ta, tb in zip(a, b):
            for x, y in zip(ta, tb):
                assert torch.equal(x, y), step
        nxt = []
        for p, g, m, v in host:
            p, m, v, _ = O.adamw_step(p, g, m, v, step - 1.0, lr=lr, beta1=0.9, beta2=0.95, eps=1e-8,
                                      weight_decay=0.01, param_dtype="bfloat16")
            nxt.append((p, g, m, v))
        host = nxt
    for t, (p, _, m, v) in zip(a, host):
        assert O.rel_frobenius(t[2].cpu().numpy(), m) < 1e-6
        assert O.rel_frobenius(t[3].cpu().numpy(), v) < 1e-6
        assert O.rel_frobenius(t[0].float().cpu().numpy(), p) < 1e-3


def test_rejects_cpu_tensors():
    from opendm_b200.engine import CudaMuonEngine

    with pytest.raises(RuntimeError):
        CudaMuonEngine("cpu")


@pytest.mark.parametrize("kind", ["bf16", "fp32", "mixed", "unclipped"])
def test_clip_grad_norm_matches_torch(kind):
    """The fused clip's total norm and coefficient against torch.nn.utils.
    clip_grad_norm_ on the same GPU gradients, and momentum with the
    coefficient applied on read against momentum on torch-clipped gradients."""
    from opendm_b200.engine import CudaMuonEngine, MatrixItem

    eng = _engine_for("fp16", "auto")
    dev = eng.device
    g = torch.Generator(device=dev).manual_seed(17)
    shapes = [(300, 77), (2048,), (64, 64), (5,), (1000, 130)]
    dts = {"bf16": [torch.bfloat16] * 5, "fp32": [torch.float32] * 5, "unclipped": [torch.bfloat16] * 5,
           "mixed": [torch.bfloat16, torch.float32] * 2 + [torch.bfloat16]}[kind]
    scale = 1e-4 if kind == "unclipped" else 1.0
    grads = [(torch.randn(s, generator=g, device=dev) * scale).to(dt) for s, dt in zip(shapes, dts)]
    out = eng.clip_grad_norm(grads, 1.0)
    params = [torch.nn.Parameter(torch.zeros_like(t)) for t in grads]
    for p, t in zip(params, grads):
        p.grad = t.clone()
    want_total = torch.nn.utils.clip_grad_norm_(params, 1.0)
    total, coef = float(out[0]), float(out[1])
    assert abs(total - float(want_total)) <= 1e-6 * float(want_total), (total, float(want_total))
    if kind == "unclipped":
        assert coef == 1.0
    # momentum reading the gradients with the coefficient == momentum on torch's clipped gradients
    ms = [s for s in shapes if len(s) == 2]
    mats = [t for t in grads if t.ndim == 2]
    clipped = [p.grad for p in params if p.grad.ndim == 2]
    m_a = [torch.randn(s, generator=g, device=dev) * 1e-3 for s in ms]
    m_b = [m.clone() for m in m_a]
    eng.grad_scale = out[1:2]
    try:
        eng.momentum_only([MatrixItem(torch.empty(0), t, m, 0.0) for t, m in zip(mats, m_a)], momentum=0.95,
                          nesterov=True)
    finally:
        eng.grad_scale = None
    eng.momentum_only([MatrixItem(torch.empty(0), t, m, 0.0) for t, m in zip(clipped, m_b)], momentum=0.95,
                      nesterov=True)
    for a, b in zip(m_a, m_b):
        assert (torch.linalg.norm(a - b) / torch.linalg.norm(b)).item() <= 1e-6


def test_more_shape_classes_than_one_plan_holds():
    """20 distinct shapes (one plan takes 16 classes): the engine splits them
    over plans; the grouped step and orthogonalize_many stay exact."""
    eng = _engine_for("fp16", "auto")
    shapes = [(64 + 16 * k, 96 + 32 * (k % 5)) for k in range(20)]
    items, host = _items(shapes, torch.float32, 70, eng.device)
    eng.muon_matrices(items, momentum=0.95, nesterov=True, weight_decay_factor=1.0, ns_steps=5)
    torch.cuda.synchronize()
    eng.check_errors(block=True)
    assert len(eng._plans[next(reversed(eng._plans))].plans) == 2
    for it, (p, g, m) in zip(items, host):
        m_ref, d = O.momentum_direction(g, m, 0.95, True)
        np.testing.assert_array_equal(it.exp_avg.cpu().numpy(), m_ref)
        u = O.zeropower_via_newtonschulz5(d)
        p_ref = O.apply_update(p, u, lr=0.02, weight_decay=0.0, eff=it.eff, param_dtype="float32",
                               device_semantics="cuda")
        assert O.rel_frobenius(it.param.cpu().numpy(), p_ref) < 1e-3
    mats = [_rand(s, 90 + k).to(eng.device) for k, s in enumerate(shapes)]
    outs = eng.orthogonalize_many(mats, [torch.float32] * len(mats))
    for x, u in zip(mats, outs):
        assert O.rel_frobenius(u.cpu().numpy(), O.zeropower_via_newtonschulz5(x.cpu().numpy())) < TF32_TOL


def test_momentum_f16_one_pass_operand_and_fixup():
    """muon_momentum_f16 (one pass: momentum, norm and the fp16 operand d * p)
    through the C ABI: exp_avg bit-exact with muon_momentum; the stored
    operand times the returned factor equals the normalised direction times
    the operand scale within fp16 rounding; the first call (no p yet) and a
    call whose norm jumped by 2^14 take the fix-up pass, a steady call does
    not; a zero gradient on zero momentum gives factor 0."""
    import ctypes

    from opendm_b200 import _native as N

    dev = _dev()
    lib = N.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    shapes = [(256, 2048), (300, 130), (64, 64)]
    g = torch.Generator(device=dev).manual_seed(41)
    m_ref = [torch.zeros(s, device=dev) for s in shapes]
    m_new = [torch.zeros(s, device=dev) for s in shapes]
    lds = [(c + 7) // 8 * 8 for _, c in shapes]
    x0 = [torch.zeros(r, ld, dtype=torch.float16, device=dev) for (r, _), ld in zip(shapes, lds)]
    pscale = torch.zeros(len(shapes), device=dev)
    scales = torch.zeros(len(shapes), device=dev)
    redo = torch.zeros(len(shapes), dtype=torch.int32, device=dev)
    muls = [float(lib.muon_ns_operand_scale(r, c, 0, N.MUON_F16)) for r, c in shapes]
    chunks = [int(lib.muon_momentum_chunks(r, c)) for r, c in shapes]
    total = sum(chunks)
    partials = torch.empty(total, device=dev)
    for step, gain in enumerate([1.0, 1.0, 16384.0, 0.0]):
        grads = [(torch.randn(s, generator=g, device=dev) * 1e-3 * gain).to(torch.bfloat16) for s in shapes]
        if gain == 0.0:
            for m in m_ref + m_new:
                m.zero_()
        segs, ref_segs, begin = [], [], 0
        for i, (r, c) in enumerate(shapes):
            sg = N.MomentumF16Seg()
            sg.grad, sg.exp_avg, sg.dst = grads[i].data_ptr(), m_new[i].data_ptr(), x0[i].data_ptr()
            sg.rows, sg.cols, sg.ld, sg.chunk_begin, sg.mul, sg.scale_index = r, c, lds[i], begin, muls[i], i
            segs.append(sg)
            rs = N.MomentumSeg()
            rs.grad, rs.exp_avg, rs.direction = grads[i].data_ptr(), m_ref[i].data_ptr(), None
            rs.rows, rs.cols, rs.ld, rs.chunk_begin = r, c, c, begin
            ref_segs.append(rs)
            begin += chunks[i]
        table = torch.frombuffer(bytearray(N.struct_bytes(segs)), dtype=torch.uint8).to(dev)
        ref_table = torch.frombuffer(bytearray(N.struct_bytes(ref_segs)), dtype=torch.uint8).to(dev)
        ref_scales = torch.zeros(len(shapes), device=dev)
        N.check(lib.muon_momentum(ctypes.c_void_p(ref_table.data_ptr()), len(shapes), total, N.MUON_BF16, N.MUON_F32,
                                  ctypes.c_float(0.95), 1, ctypes.c_float(1e-7),
                                  ctypes.c_void_p(torch.empty(total, device=dev).data_ptr()),
                                  ctypes.c_void_p(ref_scales.data_ptr()), stream), "muon_momentum")
        p_prev = pscale.clone()
        N.check(lib.muon_momentum_f16(ctypes.c_void_p(table.data_ptr()), len(shapes), total, N.MUON_BF16,
                                      ctypes.c_float(0.95), 1, ctypes.c_float(1e-7), ctypes.c_void_p(partials.data_ptr()),
                                      ctypes.c_void_p(pscale.data_ptr()), ctypes.c_void_p(scales.data_ptr()),
                                      ctypes.c_void_p(redo.data_ptr()), None, stream), "muon_momentum_f16")
        torch.cuda.synchronize()
        for i, (r, c) in enumerate(shapes):
            assert torch.equal(m_new[i], m_ref[i]), (step, i)
        if gain == 0.0:
            assert torch.all(scales == 0) and torch.all(redo == 0)
            continue
        want_redo = [1, 1, 1] if step in (0, 2) else [0, 0, 0]
        assert redo.tolist() == want_redo, (step, redo.tolist())
        p_used = torch.where(redo.bool(), pscale, p_prev)  # the fix-up writes with the new p
        # the norm's partial sums run in another order where a row is padded
        # (scalar path here, vector path in muon_momentum): last-bit differences
        torch.testing.assert_close(scales, ref_scales * torch.tensor(muls, device=dev) / p_used, rtol=1e-6, atol=0)
        for i, (r, c) in enumerate(shapes):
            d = grads[i].float() + 0.95 * m_new[i]  # Nesterov direction (fp32 rounding aside)
            want = d * ref_scales[i] * muls[i]
            got = x0[i][:, :c].float() * scales[i]
            assert O.rel_frobenius(got.cpu().numpy(), want.cpu().numpy()) < 1e-3, (step, i)
            # the stored entries stay far inside fp16's range
            assert float(x0[i][:, :c].abs().max()) < 2048.0


# ---------------------------------------------------- split operands ("parity")
PARITY_TOL = 2e-4  # Gaussian inputs; the emulation predicts ~3e-6 plus fp32 accumulation


@pytest.mark.parametrize("shape", [(1, 16), (33, 70), (70, 33), (130, 300), (300, 130), (512, 2048), (2048, 512),
                                   (1000, 1000)])
@pytest.mark.parametrize("algo", ["standard", "gram"])
def test_orthogonalize_parity_precision(algo, shape):
    """Split fp16 operands (hi + lo halves, three MMAs per product) against the
    fp32 reference: far inside the bar on Gaussian inputs, both forms."""
    eng = _engine_for("parity", algo)
    x = _rand(shape, sum(shape)) * 1.95
    got = eng.orthogonalize(x.to(eng.device)).cpu().numpy()
    eng.check_errors(block=True)
    err = O.rel_frobenius(got, O.zeropower_via_newtonschulz5(x.numpy()))
    print(f"parity-mode {algo} {shape} {err:.2e}")
    assert err < PARITY_TOL, err


def _rank_deficient(shape, kind, seed):
    rng = np.random.default_rng(seed)
    m, n = shape
    if kind == "rank1":
        return np.outer(rng.standard_normal(m), rng.standard_normal(n)).astype(np.float32) * 1e-3
    k = min(shape)  # singular values decaying by e^-20 across the rank
    u, _ = np.linalg.qr(rng.standard_normal((m, k)))
    v, _ = np.linalg.qr(rng.standard_normal((n, k)))
    return ((u * np.exp(-20.0 * np.arange(k) / k)) @ v.T).astype(np.float32) * 1e-3


@pytest.mark.parametrize("kind", ["rank1", "expdecay20"])
@pytest.mark.parametrize("shape", [(512, 2048), (2048, 512), (1024, 1024)])
def test_rank_deficient_inputs_parity_vs_fp16(kind, shape):
    """Inputs with a large null space, where any 11-bit operand type exceeds the
    1e-2 bar (rounding noise in the null directions is amplified ~a^5 by the
    quintic): the parity precision stays within it in both forms. The fp16
    result is measured alongside and must indeed exceed the parity one."""
    x = _rank_deficient(shape, kind, 5)
    ref = O.zeropower_via_newtonschulz5(x)
    errs = {}
    for prec, algo in (("parity", "standard"), ("parity", "gram"), ("fp16", "auto")):
        eng = _engine_for(prec, algo)
        got = eng.orthogonalize(torch.from_numpy(x).to(eng.device)).cpu().numpy()
        eng.check_errors(block=True)
        errs[(prec, algo)] = O.rel_frobenius(got, ref)
    print(f"rank-deficient {kind} {shape} " + " ".join(f"{k[0]}/{k[1]} {v:.2e}" for k, v in errs.items()))
    assert errs[("parity", "standard")] < 2e-3 and errs[("parity", "gram")] < 2e-3, errs
    assert errs[("fp16", "auto")] > errs[("parity", "standard")], errs
