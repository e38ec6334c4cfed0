"""The C-ABI library loads and exports every function declared in
include/opendm_muon.h (no compute calls: these run without a GPU)."""

import ctypes
import os
import re

import pytest

from opendm_b200 import _native as N
from opendm_b200.build import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    text = open(os.path.join(ROOT, "include", "opendm_muon.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(muon_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    build()
    return N.lib()


def test_every_declared_symbol_is_exported_and_bound(lib):
    names = _declared()
    assert len(names) >= 12
    raw = ctypes.CDLL(str(N.LIB_PATH))
    for name in names:
        assert hasattr(raw, name), name
        assert name in N.SIGNATURES, name
    assert set(N.SIGNATURES) == set(names)


def test_host_only_entry_points(lib):
    assert lib.muon_version() == N.ABI_VERSION
    assert lib.muon_momentum_chunks(2048, 8192) == (2048 * 8192 + 16383) // 16384
    assert lib.muon_momentum_chunks(0, 5) == 0
    assert lib.muon_adamw_chunks(8193) == 2
    std, gram = N.MUON_NS_STANDARD, N.MUON_NS_GRAM
    # two x buffers (ld padded to 16 bytes) + three m x m buffers (seven for
    # the gram form), 256-byte aligned parts
    assert lib.muon_ns_class_workspace_bytes(3, 5, 2, N.MUON_TF32, std) == 2 * 256 + 3 * 256
    assert lib.muon_ns_class_workspace_bytes(256, 2048, 1, N.MUON_BF16, std) == 2 * 256 * 2048 * 2 + 3 * 256 * 256 * 2
    assert lib.muon_ns_class_workspace_bytes(256, 2048, 1, N.MUON_F16, std) == 2 * 256 * 2048 * 2 + 3 * 256 * 256 * 2
    assert lib.muon_ns_class_workspace_bytes(256, 2048, 1, N.MUON_F16, gram) == 2 * 256 * 2048 * 2 + 7 * 256 * 256 * 2
    assert lib.muon_ns_class_workspace_bytes(4, 4, 1, N.MUON_F32, std) == 0  # not an operand type
    assert lib.muon_ns_class_workspace_bytes(4, 4, 1, N.MUON_F16, 7) == 0  # not an algorithm
    # algorithm choice: the gram form where it executes >= 10% fewer FLOPs, 11-bit operands, >= 3 steps
    assert lib.muon_ns_choose_algo(2048, 8192, N.MUON_F16, 5) == gram
    assert lib.muon_ns_choose_algo(8192, 2048, N.MUON_TF32, 5) == gram
    assert lib.muon_ns_choose_algo(2048, 2048, N.MUON_F16, 5) == std
    assert lib.muon_ns_choose_algo(2048, 8192, N.MUON_BF16, 5) == std
    assert lib.muon_ns_choose_algo(2048, 8192, N.MUON_F16, 2) == std
    # gram-form segment length (iterations between re-formings of X), per operand type
    for op in (N.MUON_F16, N.MUON_F16X3, N.MUON_TF32):
        assert lib.muon_ns_gram_segment(op) == 3
    assert lib.muon_ns_gram_segment(N.MUON_BF16) == 0 and lib.muon_ns_gram_segment(N.MUON_F32) == 0
    # fp16 operand scales: powers of two bringing entries to magnitude ~1
    assert lib.muon_ns_operand_scale(2048, 8192, 0, N.MUON_F16) == 4096.0
    assert lib.muon_ns_operand_scale(2048, 8192, 1, N.MUON_F16) == 128.0
    assert lib.muon_ns_operand_scale(2048, 8192, 0, N.MUON_TF32) == 1.0


def test_argument_validation_reports_errors(lib):
    plan = ctypes.c_void_p()
    cls = N.NsClass()
    status = lib.muon_ns_plan_create(ctypes.byref(cls), 1, N.MUON_TF32, 5, ctypes.byref(plan))
    assert status == N.MUON_ERR_ARG
    assert "empty" in N.last_error()
    assert lib.muon_ns_plan_create(ctypes.byref(cls), 1, N.MUON_F32, 5, ctypes.byref(plan)) == N.MUON_ERR_ARG
    assert lib.muon_ns_plan_create(ctypes.byref(cls), 1, N.MUON_TF32, 0, ctypes.byref(plan)) == N.MUON_ERR_UNSUPPORTED
    # a well-formed class (pointers are only checked, never read, before the
    # device query) asking for the gram form with bf16 operands
    cls.rows, cls.cols, cls.count, cls.u_dtype = 64, 128, 1, N.MUON_BF16
    for f in ("x0", "x1", "ap", "bp", "mm", "scales", "u_out", "aa", "pa", "qa", "qb"):
        setattr(cls, f, 4096)
    cls.ld_x, cls.ld_m, cls.ld_u = 128, 64, 128
    cls.algo = N.MUON_NS_GRAM
    assert lib.muon_ns_plan_create(ctypes.byref(cls), 1, N.MUON_BF16, 5, ctypes.byref(plan)) == N.MUON_ERR_UNSUPPORTED
    assert "MUON_NS_GRAM" in N.last_error()
    cls.qb = None
    assert lib.muon_ns_plan_create(ctypes.byref(cls), 1, N.MUON_F16, 5, ctypes.byref(plan)) == N.MUON_ERR_ARG
    cls.algo = 5
    assert lib.muon_ns_plan_create(ctypes.byref(cls), 1, N.MUON_F16, 5, ctypes.byref(plan)) == N.MUON_ERR_ARG
    assert lib.muon_momentum(None, 2, 4, N.MUON_BF16, N.MUON_TF32, 0.9, 1, 1e-7, None, None, None) == N.MUON_ERR_ARG
    assert lib.muon_apply_update(None, 2, 4, 1.0, None) == N.MUON_ERR_ARG
    # cross-GPU flags: list size, null and misaligned pointers are rejected before any launch
    fl = N.FlagList()
    fl.n = N.MUON_MAX_FLAGS + 1
    assert lib.muon_flags_set(ctypes.byref(fl), 1, None) == N.MUON_ERR_ARG
    fl.n = 1
    assert lib.muon_flags_set(ctypes.byref(fl), 1, None) == N.MUON_ERR_ARG  # null flag
    fl.ptr[0] = 4098
    assert lib.muon_flags_wait(ctypes.byref(fl), 1, 1000, ctypes.c_void_p(4096), None) == N.MUON_ERR_ARG
    fl.ptr[0] = 4096
    assert lib.muon_flags_wait(ctypes.byref(fl), 1, 0, ctypes.c_void_p(4096), None) == N.MUON_ERR_ARG
    assert lib.muon_flags_wait(None, 1, 1000, ctypes.c_void_p(4096), None) == N.MUON_ERR_ARG
    # gradient-norm clipping: output and tables are checked before any launch
    assert lib.muon_clip_grad_norm(None, 1, 4, ctypes.c_float(1.0), None, None, None) == N.MUON_ERR_ARG
    assert lib.muon_clip_grad_norm(None, 1, 4, ctypes.c_float(1.0), None, ctypes.c_void_p(4096), None) == N.MUON_ERR_ARG
    assert lib.muon_clip_grad_norm(None, -1, 0, ctypes.c_float(1.0), None, ctypes.c_void_p(4096), None) == N.MUON_ERR_ARG
    assert lib.muon_norm_chunks(16384) == 1 and lib.muon_norm_chunks(16385) == 2 and lib.muon_norm_chunks(0) == 0
    with pytest.raises(RuntimeError, match="failed"):
        N.check(N.MUON_ERR_ARG, "probe")


def test_noalloc_size_limit_rejected_on_host(lib):
    """muon_momentum_single_noalloc refuses shapes beyond its fixed scratch
    before touching the device: the pointers here are never dereferenced
    (there is no GPU), and a regression of the check would surface as a CUDA
    error status, not as a launch."""

    def call(rows, cols, ld):
        p = ctypes.c_void_p(4096)
        return lib.muon_momentum_single_noalloc(None, p, p, rows, cols, ld, N.MUON_F32, N.MUON_F32,
                                                ctypes.c_float(0.95), 1, ctypes.c_float(1e-7), p, None)

    limit = 16384 * 16384
    for rows, cols, ld in [(1, limit + 1, limit + 1),           # one element too many
                           (16385, 16384, 16384),                # rows x cols just above
                           (16384, 16384, 16392),                # padded rows push rows x ld above
                           (1 << 40, 1 << 40, 1 << 40),          # rows x cols overflows int64
                           ((1 << 62) + 1, 4, 4)]:
        assert call(rows, cols, ld) == N.MUON_ERR_ARG, (rows, cols, ld)
        assert "allocation-free limit" in N.last_error()
    assert call(-1, 4, 4) == N.MUON_ERR_ARG  # negative shape
    assert call(4, 8, 4) == N.MUON_ERR_ARG  # ld < cols


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(N, "_LIB", None)
    monkeypatch.setenv("OPENDM_MUON_LIB", str(tmp_path / "absent.so"))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        N.lib()
