"""ctypes binding of ``libopendm_muon.so`` (declared in include/opendm_muon.h).

The library is the only compute path of this package: there is no CPU or
PyTorch fallback. ``lib()`` raises ``RuntimeError`` when the library cannot be
loaded (build it with ``python -m opendm_b200.build``).
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, Structure, c_char_p, c_double, c_float, c_int, c_int32, c_int64, c_uint32, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libopendm_muon.so"

MUON_OK = 0
MUON_ERR_ARG = 1
MUON_ERR_CUDA = 2
MUON_ERR_DEVICE = 3
MUON_ERR_UNSUPPORTED = 4
MUON_ERR_KERNEL = 5

MUON_BF16 = 0
MUON_F32 = 1
MUON_TF32 = 2
MUON_F16 = 3
MUON_F16X3 = 4  # Newton-Schulz operands as fp16 hi/lo pairs
MUON_NS_STANDARD = 0
MUON_NS_GRAM = 1
MUON_NS_INPUT_SCALED = 1  # muon_ns_class.flags

ABI_VERSION = 4


class MomentumSeg(Structure):
    _fields_ = [
        ("grad", c_void_p),
        ("exp_avg", c_void_p),
        ("direction", c_void_p),
        ("rows", c_int64),
        ("cols", c_int64),
        ("ld", c_int64),
        ("chunk_begin", c_int64),
    ]


class NsClass(Structure):
    _fields_ = [
        ("rows", c_int32),
        ("cols", c_int32),
        ("count", c_int32),
        ("u_dtype", c_int32),
        ("x0", c_void_p),
        ("x1", c_void_p),
        ("ld_x", c_int64),
        ("ap", c_void_p),
        ("bp", c_void_p),
        ("mm", c_void_p),
        ("ld_m", c_int64),
        ("scales", c_void_p),
        ("u_out", c_void_p),
        ("ld_u", c_int64),
        ("algo", c_int32),
        ("flags", c_int32),
        ("aa", c_void_p),
        ("pa", c_void_p),
        ("qa", c_void_p),
        ("qb", c_void_p),
    ]


MUON_MAX_FLAGS = 32


class FlagList(Structure):
    _fields_ = [("ptr", c_void_p * MUON_MAX_FLAGS), ("n", c_int32)]


class MomentumF16Seg(Structure):
    _fields_ = [("grad", c_void_p), ("exp_avg", c_void_p), ("dst", c_void_p), ("rows", c_int64), ("cols", c_int64),
                ("ld", c_int64), ("chunk_begin", c_int64), ("lo_offset", c_int64), ("mul", c_float),
                ("scale_index", c_int32)]


class NormSeg(Structure):
    _fields_ = [("grad", c_void_p), ("numel", c_int64), ("chunk_begin", c_int64), ("dtype", c_int32),
                ("reserved", c_int32)]


class UpdateSeg(Structure):
    _fields_ = [
        ("param", c_void_p),
        ("update", c_void_p),
        ("rows", c_int64),
        ("cols", c_int64),
        ("ld", c_int64),
        ("chunk_begin", c_int64),
        ("eff", c_float),
        ("param_dtype", c_int32),
    ]


class AdamwSeg(Structure):
    _fields_ = [
        ("param", c_void_p),
        ("grad", c_void_p),
        ("exp_avg", c_void_p),
        ("exp_avg_sq", c_void_p),
        ("numel", c_int64),
        ("chunk_begin", c_int64),
        ("step_size", c_float),
        ("bc2_sqrt", c_float),
        ("param_dtype", c_int32),
        ("grad_dtype", c_int32),
    ]


# name -> (restype, argtypes); every symbol declared in include/opendm_muon.h.
SIGNATURES = {
    "muon_version": (c_int, []),
    "muon_last_error": (c_char_p, []),
    "muon_device_check": (c_int, [c_int]),
    "muon_read_error": (c_int, [c_void_p, POINTER(c_int), c_void_p]),
    "muon_selftest_bounded_wait": (c_int, [c_void_p, c_int, c_void_p]),
    "muon_momentum_chunks": (c_int64, [c_int64, c_int64]),
    "muon_momentum": (c_int, [c_void_p, c_int, c_int64, c_int, c_int, c_float, c_int, c_float, c_void_p,
                              c_void_p, c_void_p]),
    "muon_momentum_single_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int, c_int,
                                             c_float, c_int, c_float, c_void_p, c_void_p]),
    "muon_ns_operand_scale": (c_float, [c_int32, c_int32, c_int, c_int]),
    "muon_ns_plan_create": (c_int, [POINTER(NsClass), c_int, c_int, c_int, POINTER(c_void_p)]),
    "muon_ns_plan_run": (c_int, [c_void_p, c_void_p, c_void_p]),
    "muon_apply_update": (c_int, [c_void_p, c_int, c_int64, c_float, c_void_p]),
    "muon_ns_plan_destroy": (None, [c_void_p]),
    "muon_ns_plan_launches": (c_int, [c_void_p]),
    "muon_ns_plan_set_sm_limit": (c_int, [c_void_p, c_int]),
    "muon_flags_set": (c_int, [POINTER(FlagList), c_uint32, c_void_p]),
    "muon_norm_chunks": (c_int64, [c_int64]),
    "muon_momentum_f16": (c_int, [c_void_p, c_int, c_int64, c_int, c_float, c_int, c_float, c_void_p, c_void_p,
                                  c_void_p, c_void_p, c_void_p, c_void_p]),
    "muon_clip_grad_norm": (c_int, [c_void_p, c_int, c_int64, c_float, c_void_p, c_void_p, c_void_p]),
    "muon_momentum_scaled": (c_int, [c_void_p, c_int, c_int64, c_int, c_int, c_float, c_int, c_float, c_void_p,
                                     c_void_p, c_void_p, c_void_p]),
    "muon_adamw_scaled": (c_int, [c_void_p, c_int, c_int64, c_double, c_double, c_float, c_float, c_void_p,
                                  c_void_p]),
    "muon_flags_wait": (c_int, [POINTER(FlagList), c_uint32, c_int64, c_void_p, c_void_p]),
    "muon_ns_class_workspace_bytes": (c_int64, [c_int32, c_int32, c_int32, c_int, c_int]),
    "muon_ns_choose_algo": (c_int, [c_int32, c_int32, c_int, c_int]),
    "muon_ns_gram_segment": (c_int, [c_int]),
    "muon_ns_class_layout": (c_int, [POINTER(NsClass), c_void_p, c_int]),
    "muon_adamw_chunks": (c_int64, [c_int64]),
    "muon_adamw": (c_int, [c_void_p, c_int, c_int64, c_double, c_double, c_float, c_float, c_void_p]),
}

_LIB = None


def lib() -> ctypes.CDLL:
    """Load (once) and return the library with typed signatures."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = Path(os.environ.get("OPENDM_MUON_LIB", LIB_PATH))
    if not path.exists():
        raise RuntimeError(
            f"opendm_b200 CUDA library not found at {path}; build it with `python -m opendm_b200.build` "
            "(there is no CPU fallback)")
    try:
        handle = ctypes.CDLL(str(path))
    except OSError as exc:  # pragma: no cover - depends on the host
        raise RuntimeError(f"cannot load {path}: {exc}") from exc
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = restype
        fn.argtypes = argtypes
    if handle.muon_version() != ABI_VERSION:
        raise RuntimeError(f"{path} has ABI version {handle.muon_version()}, expected {ABI_VERSION}")
    _LIB = handle
    return handle


def last_error() -> str:
    msg = lib().muon_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str) -> None:
    """Raise RuntimeError for a nonzero library status."""
    if status != MUON_OK:
        raise RuntimeError(f"{what} failed (status {status}): {last_error()}")


def struct_bytes(items) -> bytes:
    """Concatenate ctypes structures into one byte string (a device table)."""
    if not items:
        return b""
    arr = (type(items[0]) * len(items))(*items)
    return bytes(arr)
