"""The arithmetic behind bench.py's roofline fields, on the CPU:

* the configurations' Muon element counts and the reference's dense
  Newton-Schulz FLOP count, steps * (4 m^2 n + 2 m^3) per matrix, equal the
  figures the benchmark is specified with (config 2: 196 matrices, 1.674 G
  elements, 79.53 TFLOP; config 4: 540, 3.969 G, 212.61; config 5: 224,
  6.476 G, 684.45);
* the executed-FLOP model (`roofline.executed_tflops`) gives 59.5 -> 39.7
  TFLOP for config 2 and 159.7 -> 109.3 for config 4 with the library's
  choice of form per shape;
* that model is the one the library decides with: over a sweep of shapes and
  step counts, muon_ns_choose_algo (C ABI, host-only) picks the gram form
  exactly where the model's gram count is below 0.9x the standard count
  (with at least one 3-iteration segment);
* the clock record (nvidia-smi parsing) that decides whether a run counts.
"""

import itertools
import math

import pytest

import bench


def _muon_shapes(cfg):
    return [s for n, s in bench.config_params(cfg) if bench.is_muon(n, s)]


@pytest.mark.parametrize("cfg,count,gel,tflop", [("c2", 196, 1.674, 79.53), ("c4", 540, 3.969, 212.61),
                                                  ("c5", 224, 6.476, 684.45)])
def test_config_sizes_and_dense_flops(cfg, count, gel, tflop):
    shapes = _muon_shapes(cfg)
    assert len(shapes) == count
    assert round(sum(math.prod(s) for s in shapes) / 1e9, 3) == gel
    assert round(sum(bench.ns_flops(s) for s in shapes) / 1e12, 2) == tflop
    m, n = 2048, 8192
    assert bench.ns_flops((n, m)) == bench.ns_flops((m, n)) == 5 * (4 * m * m * n + 2 * m ** 3)


def _lib_algo(lib, N, s, steps=5):
    return "gram" if lib.muon_ns_choose_algo(s[0], s[1], N.MUON_F16, steps) == N.MUON_NS_GRAM else "standard"


@pytest.mark.parametrize("cfg,standard,chosen", [("c2", 59.5, 39.7), ("c4", 159.7, 109.3)])
def test_executed_flops_with_the_library_choice(cfg, standard, chosen):
    from opendm_b200 import _native as N

    lib = N.lib()
    shapes = _muon_shapes(cfg)
    assert round(sum(bench.ns_executed_flops(s, 5, "standard") for s in shapes) / 1e12, 1) == standard
    got = sum(bench.ns_executed_flops(s, 5, _lib_algo(lib, N, s)) for s in shapes)
    assert round(got / 1e12, 1) == chosen


def test_library_choice_follows_the_executed_flop_model():
    from opendm_b200 import _native as N

    lib = N.lib()
    sizes = [16, 128, 200, 256, 300, 640, 1000, 1152, 1300, 2048, 3000, 4304, 8192, 11008]
    for r, c in itertools.product(sizes, repeat=2):
        for steps in (1, 2, 3, 5, 7):
            gram = bench.ns_executed_flops((r, c), steps, "gram")
            std = bench.ns_executed_flops((r, c), steps, "standard")
            want = "gram" if steps >= bench.GRAM_SEGMENT and gram < 0.9 * std else "standard"
            assert _lib_algo(lib, N, (r, c), steps) == want, (r, c, steps)


def test_clock_sampler_parses_nvidia_smi_lines():
    """bench.ClockSampler on canned `nvidia-smi --format=csv,noheader,nounits`
    output: only the sampled GPUs count, the median SM clock and the max clock
    are taken, a reason counts when any sample shows it "Active" ("Not Active"
    does not), and malformed lines are skipped."""

    class FakeProc:
        def terminate(self):
            pass

        def communicate(self, timeout=None):
            return ("0, 1900, 1965, 900.1, 0x4, Not Active, Not Active, Not Active, Active\n"
                    "0, 1800, 1965, 950.0, 0x4, Not Active, Not Active, Not Active, Active\n"
                    "1, 1000, 1965, 400.0, 0x0, Active, Not Active, Not Active, Not Active\n"
                    "0, [N/A], 1965, 1.0, 0x0, Not Active, Not Active, Not Active, Not Active\n"
                    "garbage\n"
                    "0, 1700, 1965, 990.0, 0x0, Not Active, Not Active, Not Active, Not Active\n", "")

    s = bench.ClockSampler([0])
    s.proc = FakeProc()
    got = s.stop()
    assert got == {"sm_mhz": 1800.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 3}
    s2 = bench.ClockSampler([0, 1])
    s2.proc = FakeProc()
    assert s2.stop()["reasons"] == ["hw_slowdown", "sw_power_cap"]
    assert bench.ClockSampler([0]).stop() is None  # never started


def test_reference_arm_line_names_the_same_workload(monkeypatch, capsys):
    """`--impl reference` prints one line, on rank 0 only, whose `config` is
    the object this library's arm prints for the same arguments, with the
    reference-arm keys (impl, cpu_baseline, e2e without copies). The timed
    sample is replaced by a fixed figure: the line's assembly is what is
    checked here, not the CPU time."""
    import json

    monkeypatch.setattr(bench, "cpu_sample", lambda cfg: (1234.5, f"stub sample of {cfg}"))
    for world in (1, 8):
        monkeypatch.setenv("WORLD_SIZE", str(world))
        monkeypatch.setenv("RANK", "1")
        bench.main(["--impl", "reference", "--gpus", str(world), "--steps", "2", "--warmup", "3"])
        assert capsys.readouterr().out == ""  # other ranks exit without work
        monkeypatch.setenv("RANK", "0")
        bench.main(["--impl", "reference", "--gpus", str(world), "--steps", "2", "--warmup", "3"])
        lines = [ln for ln in capsys.readouterr().out.splitlines() if ln.startswith("{")]
        assert len(lines) == 1
        d = json.loads(lines[0])
        assert d["config"] == bench.line_config("c2", "fp16", world, True)
        assert d["impl"] == "reference" and d["metric"] == "muon_step_ms" and d["unit"] == "ms"
        assert d["higher_is_better"] is False and d["value"] == 1234.5 and d["n_gpus"] == world
        assert d["scaling"] == ("strong" if world > 1 else "weak")
        assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["kind"] == "port"
        assert d["e2e"] == {"value": 1234.5, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
