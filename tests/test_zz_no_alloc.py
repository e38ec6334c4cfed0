"""muon_momentum_single_noalloc: the allocation-free momentum entry point, for
callers that cannot allocate device memory (its scratch lives in a fixed
array inside the library). Compared through the C ABI with muon_momentum,
the entry point that takes caller-provided scratch, on two calls in a row
(the second continues from the momentum state the first left). Both compute
the same fp32 operations in the same order, so the tolerance is the one the
other momentum tests use: exact equality.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _reference_call(lib, N, grad, exp_avg, direction, rows, cols, ld, gdt, ddt, scale):
    """One muon_momentum call (segment table + scratch allocated by torch here)."""
    seg = N.MomentumSeg()
    seg.grad = grad.data_ptr()
    seg.exp_avg = exp_avg.data_ptr()
    seg.direction = direction.data_ptr()
    seg.rows, seg.cols, seg.ld = rows, cols, ld
    seg.chunk_begin = 0
    chunks = int(lib.muon_momentum_chunks(rows, cols))
    table = torch.frombuffer(bytearray(N.struct_bytes([seg])), dtype=torch.uint8).to(grad.device)
    partials = torch.empty(max(chunks, 1), dtype=torch.float32, device=grad.device)
    N.check(lib.muon_momentum(ctypes.c_void_p(table.data_ptr()), 1, chunks, gdt, ddt, ctypes.c_float(0.95), 1,
                              ctypes.c_float(1e-7), ctypes.c_void_p(partials.data_ptr()),
                              ctypes.c_void_p(scale.data_ptr()), _stream()), "muon_momentum")


@pytest.mark.parametrize("rows,cols,ld,gdt_name,ddt_name", [
    (300, 520, 520, "bf16", "tf32"),   # vectorised path
    (2048, 8192, 8192, "bf16", "f32"),  # many chunks, fp32 direction (fp16 mode input)
    (33, 70, 72, "f32", "bf16"),        # scalar path, padded leading dimension
])
def test_noalloc_matches_muon_momentum_two_calls(rows, cols, ld, gdt_name, ddt_name):
    from opendm_b200 import _native as N

    dev = _dev()
    lib = N.lib()
    gdt = {"bf16": N.MUON_BF16, "f32": N.MUON_F32}[gdt_name]
    ddt = {"bf16": N.MUON_BF16, "tf32": N.MUON_TF32, "f32": N.MUON_F32}[ddt_name]
    tdt = torch.bfloat16 if gdt == N.MUON_BF16 else torch.float32
    ddtype = torch.bfloat16 if ddt == N.MUON_BF16 else torch.float32
    g = torch.Generator(device=dev).manual_seed(rows + cols)
    m_ref = torch.randn(rows, cols, generator=g, device=dev) * 1e-3
    m_new = m_ref.clone()
    d_ref = torch.zeros(rows, ld, dtype=ddtype, device=dev)
    d_new = torch.zeros(rows, ld, dtype=ddtype, device=dev)
    s_ref = torch.zeros(1, dtype=torch.float32, device=dev)
    s_new = torch.zeros(1, dtype=torch.float32, device=dev)
    for _ in range(2):
        grad = (torch.randn(rows, cols, generator=g, device=dev) * 1e-3).to(tdt)
        _reference_call(lib, N, grad, m_ref, d_ref, rows, cols, ld, gdt, ddt, s_ref)
        N.check(lib.muon_momentum_single_noalloc(
            ctypes.c_void_p(grad.data_ptr()), ctypes.c_void_p(m_new.data_ptr()), ctypes.c_void_p(d_new.data_ptr()),
            rows, cols, ld, gdt, ddt, ctypes.c_float(0.95), 1, ctypes.c_float(1e-7),
            ctypes.c_void_p(s_new.data_ptr()), _stream()), "muon_momentum_single_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(m_new, m_ref)
        assert torch.equal(d_new[:, :cols], d_ref[:, :cols])
        assert torch.equal(s_new, s_ref) and float(s_new) > 0


def test_noalloc_zero_gradient():
    from opendm_b200 import _native as N

    dev = _dev()
    lib = N.lib()
    m = torch.zeros(64, 64, device=dev)
    d = torch.ones(64, 64, device=dev)
    s = torch.full((1,), 7.0, device=dev)
    # absent gradient and zero momentum: direction 0, scale 0 (zero norm)
    N.check(lib.muon_momentum_single_noalloc(None, ctypes.c_void_p(m.data_ptr()), ctypes.c_void_p(d.data_ptr()),
                                             64, 64, 64, N.MUON_F32, N.MUON_F32, ctypes.c_float(0.95), 1,
                                             ctypes.c_float(1e-7), ctypes.c_void_p(s.data_ptr()), _stream()),
            "muon_momentum_single_noalloc")
    torch.cuda.synchronize()
    assert not d.any() and float(s) == 0.0
    # Shapes beyond the fixed scratch are rejected on the host before any
    # launch; that check runs without a GPU in tests/test_capi.py, so no
    # out-of-bounds shape is ever passed here with real buffers.
