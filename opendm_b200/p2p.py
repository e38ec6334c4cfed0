"""Parameter all-gather over NVLink copy engines for the sharded Muon step.

The sharded step (``opendm_b200.sharding``) leaves each rank with the updated
parameters of the matrices it owns; every rank needs all of them. NCCL's
all-gather does this with kernels that need free SMs, which the persistent
Newton-Schulz kernels hold. Here the flat parameter buffers live in
peer-mapped (symmetric) memory instead, and each rank pulls every peer's
bucket with ``cudaMemcpyAsync`` (copy engines) on one stream per peer, so
the transfer of wave w overlaps the Newton-Schulz of wave w + 1 at full SM
count. Ordering across GPUs uses flags in the same kind of memory
(``muon_flags_set`` / ``muon_flags_wait`` in ``libopendm_muon.so``):

* after rank r's update of wave w: r raises flag (w, r) on every peer;
* peer k's copy stream for r waits for that flag, then copies r's bucket;
* at the end of the step every rank waits for its copies, raises its barrier
  flag on every peer and waits for all peers' barrier flags, so no rank
  rewrites its bucket (next step) while a peer still reads it.

Flag values are the step count (wrap-around compared); every wait is bounded
and records 0x106 in the engine's device error word on expiry.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _native as N

WAIT_TIMEOUT_US = 60_000_000  # a peer may still be building its first-step plans


def available() -> bool:
    """True when torch's symmetric memory can map peers' buffers here."""
    try:
        import torch.distributed._symmetric_memory  # noqa: F401
    except Exception:
        return False
    return torch.cuda.is_available()


class P2PFlatBuckets:
    """Flat (dtype, wave) parameter buckets in peer-mapped memory, laid out
    like ``FlatParamBuckets`` ([rank 0 bucket | rank 1 bucket | ...]), with a
    copy-engine all-gather split by wave."""

    def __init__(self, params: list[torch.Tensor], owners: list[int], world_size: int, rank: int,
                 process_group, waves: list[int], err_word: torch.Tensor):
        import torch.distributed._symmetric_memory as symm_mem

        self.world_size, self.rank = world_size, rank
        self.group = process_group if process_group is not None else dist.group.WORLD
        self.err = err_word
        self.lib = N.lib()
        self.n_waves = max(waves, default=0) + 1
        device = params[0].device
        self.device = device
        # (flat, bucket elements, wave, peer views, symmetric-memory handle)
        self.buffers: list[tuple[torch.Tensor, int, int, list, object]] = []
        by_key: dict[tuple, list[int]] = {}
        for i, p in enumerate(params):
            by_key.setdefault((waves[i], str(p.dtype)), []).append(i)
        for (wave, _), idxs in sorted(by_key.items()):
            sizes = [0] * world_size
            for i in idxs:
                sizes[owners[i]] += params[i].numel()
            bucket = (max(sizes) + 127) // 128 * 128
            if bucket == 0:
                continue
            dtype = params[idxs[0]].dtype
            flat = symm_mem.empty(bucket * world_size, dtype=dtype, device=device)
            flat.zero_()
            hdl = symm_mem.rendezvous(flat, self.group)
            offsets = [r * bucket for r in range(world_size)]
            for i in idxs:
                p, r, n = params[i], owners[i], params[i].numel()
                view = flat[offsets[r]:offsets[r] + n].view(p.shape)
                view.copy_(p.data)
                p.data = view
                offsets[r] += n
            peers = [None if k == rank else
                     hdl.get_buffer(k, (bucket * world_size,), dtype)[k * bucket:(k + 1) * bucket]
                     for k in range(world_size)]
            self.buffers.append((flat, bucket, wave, peers, hdl))
        # flags[channel][src]: channel w < n_waves = wave w ready, channel n_waves = step done
        self.n_channels = self.n_waves + 1
        self.flags = symm_mem.empty(self.n_channels * world_size, dtype=torch.int32, device=device)
        self.flags.zero_()
        self.flag_hdl = symm_mem.rendezvous(self.flags, self.group)
        self.flag_base = [int(p) for p in self.flag_hdl.buffer_ptrs]
        self.streams = [None if k == rank else torch.cuda.Stream(device) for k in range(world_size)]
        self.step = 0
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)  # every rank's flags are zero before anyone signals

    # ------------------------------------------------------------ helpers
    def _flag(self, owner_rank: int, channel: int, src: int) -> int:
        return self.flag_base[owner_rank] + 4 * (channel * self.world_size + src)

    def _list(self, ptrs: list[int]) -> N.FlagList:
        fl = N.FlagList()
        for i, p in enumerate(ptrs):
            fl.ptr[i] = p
        fl.n = len(ptrs)
        return fl

    def _set(self, ptrs, stream) -> None:
        N.check(self.lib.muon_flags_set(ctypes.byref(self._list(ptrs)), self.step & 0xFFFFFFFF,
                                        ctypes.c_void_p(stream.cuda_stream)), "muon_flags_set")

    def _wait(self, ptrs, stream) -> None:
        N.check(self.lib.muon_flags_wait(ctypes.byref(self._list(ptrs)), self.step & 0xFFFFFFFF, WAIT_TIMEOUT_US,
                                         ctypes.c_void_p(self.err.data_ptr()), ctypes.c_void_p(stream.cuda_stream)),
                "muon_flags_wait")

    # ------------------------------------------------------------- a step
    def begin(self) -> None:
        """Start a step: the copy streams follow everything already queued on
        the current stream (e.g. the forward pass reading the parameters)."""
        self.step += 1
        cur = torch.cuda.current_stream(self.device)
        for s in self.streams:
            if s is not None:
                s.wait_stream(cur)

    def wave_done(self, wave: int) -> None:
        """This rank's updates of `wave` are queued on the current stream:
        signal the peers and queue the pulls of their buckets."""
        cur = torch.cuda.current_stream(self.device)
        peers = [k for k in range(self.world_size) if k != self.rank]
        self._set([self._flag(k, wave, self.rank) for k in peers], cur)
        for k in peers:
            s = self.streams[k]
            self._wait([self._flag(self.rank, wave, k)], s)
            with torch.cuda.stream(s):
                for flat, bucket, w, views, _ in self.buffers:
                    if w == wave:
                        flat[k * bucket:(k + 1) * bucket].copy_(views[k], non_blocking=True)

    def finish(self) -> None:
        """Join the copies and hold every rank until all ranks have theirs."""
        cur = torch.cuda.current_stream(self.device)
        for s in self.streams:
            if s is not None:
                cur.wait_stream(s)
        peers = [k for k in range(self.world_size) if k != self.rank]
        done = self.n_waves
        self._set([self._flag(k, done, self.rank) for k in peers], cur)
        self._wait([self._flag(self.rank, done, k) for k in peers], cur)

    def sync(self) -> None:
        """A whole all-gather (all waves), outside a step."""
        self.begin()
        for w in range(self.n_waves):
            self.wave_done(w)
        self.finish()

    def nbytes_received(self) -> int:
        return sum(b * flat.element_size() * (self.world_size - 1) for flat, b, *_ in self.buffers)
