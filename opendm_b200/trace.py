"""NVTX ranges for the phases of an optimizer step, so a timeline profiler
(nsys) shows on the host thread where each step's momentum, Newton-Schulz,
update, AdamW and all-gather work was queued. The ranges are named
"opendm/<phase>". A push and a pop cost well under a microsecond when no
profiler is attached, so they are always on. If this torch build has no
NVTX binding, the ranges turn themselves off.
"""

from __future__ import annotations

import contextlib

import torch


def _probe() -> bool:
    try:
        torch.cuda.nvtx.range_push("opendm/probe")
        torch.cuda.nvtx.range_pop()
        return True
    except Exception:  # pragma: no cover - builds without NVTX
        return False


ENABLED = _probe()


def push(name: str) -> None:
    if ENABLED:
        torch.cuda.nvtx.range_push("opendm/" + name)


def pop() -> None:
    if ENABLED:
        torch.cuda.nvtx.range_pop()


@contextlib.contextmanager
def nvtx(name: str):
    """A range around a block (popped on exceptions too)."""
    push(name)
    try:
        yield
    finally:
        pop()
