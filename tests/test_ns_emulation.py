"""The Newton-Schulz numerics design checked on the CPU (no GPU): an emulation
of the fp16 kernels' operand rounding (oracle/ns_emulation.py) against the
fp32 oracle of the reference algorithm (reference muon_adamw.py:101-128).

* both forms, the shifted standard iteration and the gram iteration with a
  restart every 3 iterations, stay within the 1e-2 update bar on Gaussian,
  heavy-tailed, low-rank-plus-noise, power-law and e^-10-decaying spectra, and
  the gram form stays within 2x of the standard form (the GPU tests check the
  same bars on the kernels themselves, test_gpu_kernels.py);
* a rank-1 input exceeds the bar in both forms: rounding noise in the null
  space is amplified by the quintic (~a^5), which any 11-bit operand type
  (TF32 included) shares;
* the emulation's operand scales are the library's own
  (muon_ns_operand_scale through the C ABI, host-only);
* the operand choice: fp16 and tf32 equal, bf16 ~8x worse (at the bar), the
  shifted grouping no worse than the reference's.
"""

import itertools

import pytest

from oracle import muon_oracle as O
from oracle import ns_emulation as E

BAR = 1e-2


def _errors(x):
    ref = O.zeropower_via_newtonschulz5(x, 5)
    return O.rel_frobenius(E.emulate_standard(x), ref), O.rel_frobenius(E.emulate_gram(x), ref)


@pytest.mark.parametrize("kind", ["lowrank_noise", "powerlaw", "expdecay"])
@pytest.mark.parametrize("shape", [(512, 2048), (2048, 512)])
def test_structured_spectra_within_bar(kind, shape):
    std, gram = _errors(E.structured_input(shape, kind, 21))
    assert std < BAR and gram < BAR, (std, gram)
    assert gram < 2 * std + 1e-3, (std, gram)


@pytest.mark.parametrize("kind", ["gauss", "heavytail"])
@pytest.mark.parametrize("shape", [(128, 512), (512, 128), (256, 256)])
def test_full_rank_inputs_far_below_bar(kind, shape):
    std, gram = _errors(E.structured_input(shape, kind, 3))
    assert std < 3e-3 and gram < 3e-3, (std, gram)


def test_rank_one_input_exceeds_bar_in_both_forms():
    std, gram = _errors(E.structured_input((256, 640), "rank1", 3))
    assert std > 0.1 and gram > 0.1, (std, gram)


def test_emulation_uses_the_library_operand_scales():
    from opendm_b200 import _native as N

    lib = N.lib()
    sizes = [1, 16, 33, 70, 256, 1152, 2048, 2560, 4304, 8192, 11008, 32768]
    for r, c in itertools.product(sizes, repeat=2):
        m, n = min(r, c), max(r, c)
        for it in range(3):
            assert lib.muon_ns_operand_scale(r, c, it, N.MUON_F16) == E.x_scale(m, n, it), (r, c, it)


@pytest.mark.parametrize("shape", [(256, 1024), (1024, 256), (512, 512)])
def test_operand_types_and_the_shifted_form(shape):
    """The operand choice of the design: fp16 (power-of-two scaled) and tf32
    give the same error (both 11-bit significands); bf16 operands are ~8x
    worse and sit at the bar; the shifted grouping is no worse than the
    reference's a X + (b A + c A^2) X with the same operands, and the gram form
    runs in tf32 as well as in fp16."""
    x = E.structured_input(shape, "gauss", 5)
    ref = O.zeropower_via_newtonschulz5(x, 5)
    err = {op: O.rel_frobenius(E.emulate_standard(x, op=op), ref) for op in ("fp16", "tf32", "bf16")}
    ref_form = O.rel_frobenius(E.emulate_standard(x, op="tf32", shifted=False), ref)
    gram_tf32 = O.rel_frobenius(E.emulate_gram(x, op="tf32"), ref)
    assert abs(err["fp16"] - err["tf32"]) < 0.2 * err["tf32"], err
    assert err["bf16"] > 5 * err["fp16"] and err["bf16"] > 5e-3, err
    assert err["tf32"] <= 1.05 * ref_form, (err, ref_form)
    assert gram_tf32 < 3e-3, gram_tf32


def test_tf32_rounding_ties_away_from_zero():
    import numpy as np

    x = np.array([1.0, 1.0 + 2 ** -11, 1.0 + 3 * 2 ** -11, -1.0 - 2 ** -11, 1.0 + 2 ** -12], np.float32)
    want = [1.0, 1.0 + 2 ** -10, 1.0 + 2 ** -9, -1.0 - 2 ** -10, 1.0]
    assert E._tf32(x).tolist() == want


@pytest.mark.parametrize("kind", ["lowrank_noise", "powerlaw", "expdecay"])
def test_gram_form_needs_its_restart(kind):
    """Why X is re-formed every 3 iterations: iterating on X X^T alone for all
    5 steps lets the m x m products' rounding grow along the small singular
    directions (several times the bar on structured spectra); the restart
    every 3 iterations keeps the gram form under the bar."""
    x = E.structured_input((256, 1024), kind, 21)
    ref = O.zeropower_via_newtonschulz5(x, 5)
    restarted = O.rel_frobenius(E.emulate_gram(x, restart=3), ref)
    pure = O.rel_frobenius(E.emulate_gram(x, restart=5), ref)
    assert restarted < BAR < 5 * BAR < pure, (restarted, pure)
