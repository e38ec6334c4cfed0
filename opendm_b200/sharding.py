"""Newton-Schulz work sharding across the ranks of one node.

The reference runs every Newton-Schulz redundantly on every rank of a
replicated (DDP) job (opendm/optimizer/muon_adamw.py:485-486, :513-514). Here
each matrix gets one owner rank:

* ``assign_owners`` -- longest-processing-time (LPT) assignment by dense
  Newton-Schulz FLOPs: matrices in decreasing cost order, each to the least
  loaded rank (ties to the lower rank). Deterministic, so every rank computes
  the same plan without communication.
* ``FlatParamBuckets`` -- after the owners update their matrices in place, one
  ``all_gather_into_tensor`` per dtype delivers them to every rank. The
  parameters are re-pointed once to views of a flat buffer laid out as
  [rank 0 bucket | rank 1 bucket | ...] (each bucket padded to the same
  size), so the collective writes straight into the parameters: no pack or
  unpack copies.
"""

from __future__ import annotations

import heapq

import torch
import torch.distributed as dist


def ns_cost(shape: tuple[int, int], steps: int = 5) -> float:
    """Dense Newton-Schulz FLOPs: steps * (4 m^2 n + 2 m^3), m <= n."""
    m, n = min(shape), max(shape)
    return float(max(steps, 1)) * (4.0 * m * m * n + 2.0 * m ** 3)


def assign_owners(shapes: list[tuple[int, int]], world_size: int, steps: int = 5) -> list[int]:
    """LPT owner rank for each matrix (index-aligned with ``shapes``)."""
    order = sorted(range(len(shapes)), key=lambda i: (-ns_cost(shapes[i], steps), i))
    heap = [(0.0, r) for r in range(world_size)]
    owners = [0] * len(shapes)
    for i in order:
        load, r = heapq.heappop(heap)
        owners[i] = r
        heapq.heappush(heap, (load + ns_cost(shapes[i], steps), r))
    return owners


def load_balance(shapes: list[tuple[int, int]], owners: list[int], world_size: int, steps: int = 5) -> dict:
    """Per-rank Newton-Schulz FLOPs and the max/mean imbalance of a plan."""
    loads = [0.0] * world_size
    for s, r in zip(shapes, owners):
        loads[r] += ns_cost(s, steps)
    mean = sum(loads) / max(world_size, 1)
    return {"loads": loads, "max_over_mean": (max(loads) / mean) if mean > 0 else 1.0}


class FlatParamBuckets:
    """Re-points owned-by-rank parameters into per-dtype flat buffers and
    all-gathers the owners' buckets into every rank."""

    def __init__(self, params: list[torch.Tensor], owners: list[int], world_size: int, rank: int,
                 process_group=None):
        self.world_size = world_size
        self.rank = rank
        self.group = process_group
        self.buffers: list[tuple[torch.Tensor, int]] = []  # (flat buffer, bucket elements)
        by_dtype: dict[torch.dtype, list[int]] = {}
        for i, p in enumerate(params):
            by_dtype.setdefault(p.dtype, []).append(i)
        for dtype, idxs in by_dtype.items():
            sizes = [0] * world_size
            for i in idxs:
                sizes[owners[i]] += params[i].numel()
            bucket = max(sizes)
            bucket = (bucket + 127) // 128 * 128  # keep every bucket 256-byte aligned
            device = params[idxs[0]].device
            flat = torch.zeros(bucket * world_size, dtype=dtype, device=device)
            offsets = [r * bucket for r in range(world_size)]
            for i in idxs:
                p = params[i]
                r = owners[i]
                n = p.numel()
                view = flat[offsets[r]:offsets[r] + n].view(p.shape)
                view.copy_(p.data)
                p.data = view
                offsets[r] += n
            self.buffers.append((flat, bucket))

    def sync(self) -> None:
        """All-gather every owner's bucket into all ranks (in place)."""
        for flat, bucket in self.buffers:
            if bucket == 0:
                continue
            mine = flat[self.rank * bucket:(self.rank + 1) * bucket]
            if flat.device.type == "cuda":
                dist.all_gather_into_tensor(flat, mine, group=self.group)
            else:
                # gloo has no in-place all_gather_into_tensor: gather a list and copy back.
                parts = [torch.empty_like(mine) for _ in range(self.world_size)]
                dist.all_gather(parts, mine.clone(), group=self.group)
                for r, part in enumerate(parts):
                    if r != self.rank:
                        flat[r * bucket:(r + 1) * bucket].copy_(part)

    def nbytes_received(self) -> int:
        """Bytes each rank receives per sync."""
        return sum(b * flat.element_size() * (self.world_size - 1) for flat, b in self.buffers)
