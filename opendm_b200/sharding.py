"""Newton-Schulz work sharding across the ranks of one node.

The reference runs every Newton-Schulz redundantly on every rank of a
replicated (DDP) job (opendm/optimizer/muon_adamw.py:485-486, :513-514). Here
each matrix gets one owner rank:

* ``assign_owners`` -- longest-processing-time (LPT) assignment by dense
  Newton-Schulz FLOPs: matrices in decreasing cost order, each to the least
  loaded rank (ties to the lower rank). Deterministic, so every rank computes
  the same plan without communication.
* ``assign_waves`` -- each rank's owned matrices, those with the most bytes
  per Newton-Schulz FLOP (the smallest m = min(rows, cols)) first, cut into
  waves whose FLOPs shrink geometrically. The all-gather of wave w runs on
  the collective's stream while wave w + 1 is orthogonalised: byte-heavy
  matrices go early, where their transfer has the most compute to hide
  behind, and the last wave, whose transfer is exposed, carries few bytes.
* ``FlatParamBuckets`` -- after the owners update their matrices in place, one
  ``all_gather_into_tensor`` per (dtype, wave) delivers them to every rank.
  The parameters are re-pointed once to views of flat buffers laid out as
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


def wave_fractions(n_waves: int, ratio: float = 0.7) -> list[float]:
    """FLOP share of each wave: geometric, each wave `ratio` times the one
    before (the all-gather of a wave must hide behind the next wave's
    Newton-Schulz, which takes ~1.4x longer per byte at 8 ranks)."""
    w = [ratio ** i for i in range(max(n_waves, 1))]
    total = sum(w)
    return [x / total for x in w]


def _bytes_per_flop(shape: tuple[int, int], steps: int) -> float:
    return shape[0] * shape[1] / ns_cost(shape, steps)


def assign_waves(shapes: list[tuple[int, int]], owners: list[int], world_size: int, n_waves: int,
                 steps: int = 5, ratio: float = 0.7) -> list[int]:
    """Wave index of each matrix: every rank orders its own matrices by
    decreasing bytes per FLOP and cuts them at the cumulative FLOP shares of
    ``wave_fractions(n_waves, ratio)``. Deterministic, so every rank computes
    every rank's waves."""
    waves = [0] * len(shapes)
    if n_waves <= 1:
        return waves
    bounds = []
    acc = 0.0
    for f in wave_fractions(n_waves, ratio)[:-1]:
        acc += f
        bounds.append(acc)
    for r in range(world_size):
        mine = sorted((i for i, o in enumerate(owners) if o == r),
                      key=lambda i: (-_bytes_per_flop(shapes[i], steps), -ns_cost(shapes[i], steps), i))
        total = sum(ns_cost(shapes[i], steps) for i in mine)
        done, w = 0.0, 0
        for i in mine:
            # a matrix joins the wave its cost midpoint falls into
            mid = (done + ns_cost(shapes[i], steps) / 2) / total if total > 0 else 0.0
            while w < len(bounds) and mid > bounds[w]:
                w += 1
            waves[i] = w
            done += ns_cost(shapes[i], steps)
    return waves


def load_balance(shapes: list[tuple[int, int]], owners: list[int], world_size: int, steps: int = 5) -> dict:
    """Per-rank Newton-Schulz FLOPs and the max/mean imbalance of a plan."""
    loads = [0.0] * world_size
    for s, r in zip(shapes, owners):
        loads[r] += ns_cost(s, steps)
    mean = sum(loads) / max(world_size, 1)
    return {"loads": loads, "max_over_mean": (max(loads) / mean) if mean > 0 else 1.0}


class FlatParamBuckets:
    """Re-points owned-by-rank parameters into flat buffers, one per (dtype,
    wave), and all-gathers the owners' buckets into every rank."""

    def __init__(self, params: list[torch.Tensor], owners: list[int], world_size: int, rank: int,
                 process_group=None, waves: list[int] | None = None):
        self.world_size = world_size
        self.rank = rank
        self.group = process_group
        waves = waves if waves is not None else [0] * len(params)
        self.n_waves = max(waves, default=0) + 1
        # (flat buffer, bucket elements, wave)
        self.buffers: list[tuple[torch.Tensor, int, int]] = []
        by_key: dict[tuple, list[int]] = {}
        for i, p in enumerate(params):
            by_key.setdefault((waves[i], str(p.dtype)), []).append(i)
        for (wave, _), idxs in sorted(by_key.items()):
            sizes = [0] * world_size
            for i in idxs:
                sizes[owners[i]] += params[i].numel()
            bucket = max(sizes)
            bucket = (bucket + 127) // 128 * 128  # keep every bucket 256-byte aligned
            dtype, device = params[idxs[0]].dtype, params[idxs[0]].device
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
            self.buffers.append((flat, bucket, wave))

    def sync(self, wave: int | None = None, async_op: bool = False, group=None) -> list:
        """All-gather every owner's bucket into all ranks (in place), for one
        wave or all of them. With ``async_op`` (CUDA only) the collectives
        are queued behind the work already on the current stream and their
        handles returned; ``wait()`` on each makes the current stream wait
        for it."""
        handles = []
        group = group if group is not None else self.group
        for flat, bucket, w in self.buffers:
            if bucket == 0 or (wave is not None and w != wave):
                continue
            mine = flat[self.rank * bucket:(self.rank + 1) * bucket]
            if flat.device.type == "cuda":
                h = dist.all_gather_into_tensor(flat, mine, group=group, async_op=async_op)
                if async_op:
                    handles.append(h)
            else:
                # gloo has no in-place all_gather_into_tensor: gather a list and copy back.
                parts = [torch.empty_like(mine) for _ in range(self.world_size)]
                dist.all_gather(parts, mine.clone(), group=self.group)
                for r, part in enumerate(parts):
                    if r != self.rank:
                        flat[r * bucket:(r + 1) * bucket].copy_(part)
        return handles

    def nbytes_received(self) -> int:
        """Bytes each rank receives per sync."""
        return sum(b * flat.element_size() * (self.world_size - 1) for flat, b, _ in self.buffers)


class FlatAdamShards:
    """AdamW parameters replicated on every rank (DDP), re-pointed once into
    one flat buffer per dtype and split into equal contiguous ranges, one per
    rank (ZeRO-1 style). AdamW is elementwise, so a rank updates its range of
    every parameter it overlaps, whole tensors or not: the reference runs the
    full AdamW on every rank (muon_adamw.py:333-343), and a single embedding
    (e.g. 151936 x 2048) dominates the group, so owners of whole tensors
    would not balance. One ``all_gather_into_tensor`` per dtype then gives
    every rank every range.

    Layout per dtype: parameters back to back, each starting on a multiple of
    ``ALIGN`` elements; the buffer is ``world_size`` ranges of ``range_numel``
    elements (a multiple of ``ALIGN``), so every range and every sub-range a
    rank updates starts 128-byte aligned or better."""

    ALIGN = 64

    def __init__(self, params: list[torch.Tensor], world_size: int, rank: int, process_group=None):
        self.world_size = world_size
        self.rank = rank
        self.group = process_group
        # (flat buffer, range elements, [(param index, flat offset)])
        self.buffers: list[tuple[torch.Tensor, int, list[tuple[int, int]]]] = []
        by_dtype: dict[str, list[int]] = {}
        for i, p in enumerate(params):
            by_dtype.setdefault(str(p.dtype), []).append(i)
        for _, idxs in sorted(by_dtype.items()):
            placed, total = [], 0
            for i in idxs:
                placed.append((i, total))
                total += (params[i].numel() + self.ALIGN - 1) // self.ALIGN * self.ALIGN
            per_rank = (total + world_size - 1) // world_size
            per_rank = (per_rank + self.ALIGN - 1) // self.ALIGN * self.ALIGN
            if per_rank == 0:
                continue
            dtype, device = params[idxs[0]].dtype, params[idxs[0]].device
            flat = torch.zeros(per_rank * world_size, dtype=dtype, device=device)
            for i, off in placed:
                p = params[i]
                view = flat[off:off + p.numel()].view(p.shape)
                view.copy_(p.data)
                p.data = view
            self.buffers.append((flat, per_rank, placed))

    def ranges(self, params: list[torch.Tensor]) -> list[tuple[int, int, int, int]]:
        """Every (param index, owner rank, start, length) piece: the
        intersection of each parameter with each rank's range, in element
        offsets within the flattened parameter."""
        out = []
        for _, per_rank, placed in self.buffers:
            for i, off in placed:
                n = params[i].numel()
                r0, r1 = off // per_rank, (off + max(n, 1) - 1) // per_rank
                for r in range(r0, min(r1, self.world_size - 1) + 1):
                    lo, hi = max(off, r * per_rank), min(off + n, (r + 1) * per_rank)
                    if hi > lo:
                        out.append((i, r, lo - off, hi - lo))
        return out

    def owned(self, params: list[torch.Tensor]) -> list[tuple[int, int, int]]:
        """This rank's pieces: (param index, start, length)."""
        return [(i, s, n) for i, r, s, n in self.ranges(params) if r == self.rank]

    def sync(self, async_op: bool = False, group=None) -> list:
        """All-gather every rank's range into all ranks (in place); with
        ``async_op`` (CUDA only) the handles are returned, as in
        ``FlatParamBuckets.sync``."""
        handles = []
        group = group if group is not None else self.group
        for flat, per_rank, _ in self.buffers:
            mine = flat[self.rank * per_rank:(self.rank + 1) * per_rank]
            if flat.device.type == "cuda":
                h = dist.all_gather_into_tensor(flat, mine, group=group, async_op=async_op)
                if async_op:
                    handles.append(h)
            else:
                parts = [torch.empty_like(mine) for _ in range(self.world_size)]
                dist.all_gather(parts, mine.clone(), group=self.group)
                for r, part in enumerate(parts):
                    if r != self.rank:
                        flat[r * per_rank:(r + 1) * per_rank].copy_(part)
        return handles

    def nbytes_received(self) -> int:
        """Bytes each rank receives per sync."""
        return sum(b * flat.element_size() * (self.world_size - 1) for flat, b, _ in self.buffers)
