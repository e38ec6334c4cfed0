"""Pin the numpy oracle to the reference's own outputs (tests/golden/*.npz,
produced by tests/golden/make_golden.py from the unmodified reference)."""

import os

import numpy as np
import pytest

from oracle import muon_oracle as O


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name), allow_pickle=False)


def test_ns_cases_match_reference(golden_dir):
    z = _load(golden_dir, "ns_cases.npz")
    for i in range(int(z["n_cases"])):
        got = O.zeropower_via_newtonschulz5(z[f"in{i}"], steps=int(z[f"steps{i}"]))
        ref = z[f"out{i}"]
        assert got.shape == ref.shape
        assert O.rel_frobenius(got, ref) < 2e-5, (i, O.rel_frobenius(got, ref))


def test_ns_zero_and_nonfinite_give_zeros(golden_dir):
    z = _load(golden_dir, "ns_cases.npz")
    for key in ("zero", "inf"):
        got = O.zeropower_via_newtonschulz5(z[f"in_{key}"])
        np.testing.assert_array_equal(got, z[f"out_{key}"])
        assert not got.any()


def test_ns_rejects_non_2d():
    with pytest.raises(ValueError):
        O.zeropower_via_newtonschulz5(np.zeros((2, 3, 4), np.float32))


def _replay(z, dtype):
    keys = sorted({k.split("/", 1)[1] for k in z.files if k.startswith("init/")})
    muon_keys = set(z["muon_keys"].tolist())
    steps = int(z["meta_steps"])
    opt = O.OracleMuonAdamW(lr=float(z["meta_lr"]), betas=(0.9, 0.95), eps=1e-8,
                            weight_decay=float(z["meta_wd"]), muon_nesterov=bool(z["meta_nesterov"]))
    params = {k: z[f"init/{k}"].copy() for k in keys}
    results = []
    for s in range(steps):
        grads = {}
        for k in keys:
            g = z[f"grad{s}/{k}"]
            grads[k] = None if np.isnan(g).all() else g
        opt.step({k: params[k] for k in keys if k in muon_keys}, {k: grads[k] for k in keys if k in muon_keys},
                 {k: params[k] for k in keys if k not in muon_keys},
                 {k: grads[k] for k in keys if k not in muon_keys}, param_dtype=dtype)
        results.append({k: params[k].copy() for k in keys})
    return keys, muon_keys, opt, results


@pytest.mark.parametrize("name,dtype", [("step_fp32.npz", "float32"), ("step_nonesterov.npz", "float32"),
                                        ("step_bf16.npz", "bfloat16")])
def test_optimizer_steps_match_reference(golden_dir, name, dtype):
    z = _load(golden_dir, name)
    keys, muon_keys, opt, results = _replay(z, dtype)
    for s, res in enumerate(results):
        for k in keys:
            ref = z[f"param{s}/{k}"]
            got = res[k]
            if dtype == "float32":
                assert O.rel_frobenius(got, ref) < 1e-6, (s, k, O.rel_frobenius(got, ref))
            else:
                # bf16 params: identical up to rare one-ulp flips (BLAS summation order)
                diff = np.abs(got - ref)
                ulp = np.abs(ref) * 2.0 ** -7 + 1e-30
                assert np.sum(diff > 0) <= max(2, 2e-3 * diff.size), (s, k)
                assert np.all(diff <= ulp), (s, k)
    for k in keys:
        st = opt.muon_state.get(k) or opt.adamw_state.get(k)
        assert O.rel_frobenius(st.exp_avg, z[f"exp_avg/{k}"]) < 1e-6, k
        if k not in muon_keys:
            assert O.rel_frobenius(st.exp_avg_sq, z[f"exp_avg_sq/{k}"]) < 1e-6, k
        assert st.step == float(z[f"step/{k}"]), k


def test_exp_avg_bit_exact_fp32(golden_dir):
    z = _load(golden_dir, "step_fp32.npz")
    keys, muon_keys, opt, _ = _replay(z, "float32")
    for k in muon_keys:
        np.testing.assert_array_equal(opt.muon_state[k].exp_avg, z[f"exp_avg/{k}"])


def test_bf16_round_ties_to_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 0.0], np.float32)
    got = O.bf16_round(x)
    np.testing.assert_array_equal(got, np.array([1.0, 1.0, 1.0 + 2 ** -6, -2.5, 0.0], np.float32))


def test_ns_flops_formula():
    assert O.ns_flops((2048, 8192)) == 5 * (4 * 2048 ** 2 * 8192 + 2 * 2048 ** 3)
    assert O.ns_flops((8192, 2048)) == O.ns_flops((2048, 8192))


def test_clip_oracle_matches_torch_clip_grad_norm(golden_dir):
    """The gradient-norm clipping restatement against torch.nn.utils.
    clip_grad_norm_ (the call the reference's trainer makes before each
    step): bit-exact whenever a bf16 gradient sets the arithmetic or no
    clipping happens; fp32 within the last bit of the norm's reduction order."""
    z = np.load(os.path.join(golden_dir, "clip_cases.npz"))
    for case in z["cases"]:
        n = len([k for k in z.files if k.startswith(f"{case}/in")])
        grads = [z[f"{case}/in{i}"] for i in range(n)]
        dtypes = [str(z[f"{case}/dtype{i}"]) for i in range(n)]
        out, total, coef = O.clip_grad_norm(grads, dtypes, 1.0)
        assert abs(total - float(z[f"{case}/total"])) <= 1e-6 * abs(float(z[f"{case}/total"])), case
        for i, o in enumerate(out):
            want = z[f"{case}/out{i}"]
            if case == "fp32":
                np.testing.assert_allclose(o, want, rtol=1e-6, atol=0)
            else:
                np.testing.assert_array_equal(o, want, err_msg=f"{case}/{i}")
