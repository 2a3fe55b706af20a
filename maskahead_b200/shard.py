"""Multi-GPU partitioning of the select + attend hot path: one process per GPU.

Selection, retention and attention are independent per (sequence, KV head): the eviction
state, the read set and the retained set are per KV head and shared by its query-head
group (eviction.py:206-212). Two partitionings follow (the reference itself runs only
independent replicas, one process per GPU: scripts/gpu_queue.sh:1-49):

* by sequences -- a serving batch of independent sequences. Each rank takes a contiguous
  range of sequences whose total prefix length is within one sequence of 1/world of the
  job's; no data-path collective.
* by KV heads -- one long sequence. Each rank holds H/world KV heads with their G query
  heads each (query head h*G + g belongs to KV head h) and runs the whole path for them;
  after every layer step the per-rank head outputs [B, Hq/world, T, D] are gathered into
  [B, Hq, T, D] on every rank, the only exchange: PeerHeadGather does it with this
  library's own kernel (peer stores over NVLink into IPC-mapped receive regions,
  ma_head_gather), HeadGather with an NCCL all-gather.

The functions take plain sizes and work with any torch.distributed backend (NCCL on the
GPU box, gloo in the CPU tests).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

__all__ = ["SequenceShard", "HeadShard", "sequence_shard", "head_shard", "HeadGather", "PeerHeadGather"]


@dataclass(frozen=True)
class SequenceShard:
    lo: int          # first sequence of the rank
    hi: int          # one past its last
    lens: list       # their prefix lengths


@dataclass(frozen=True)
class HeadShard:
    h0: int          # first KV head of the rank
    H: int           # KV heads of the rank
    hq0: int         # first query head (h0 * G)
    Hq: int          # query heads of the rank (H * G)


def sequence_shard(lens, world: int, rank: int) -> SequenceShard:
    """Contiguous range of sequences for `rank`: the cut between ranks r-1 and r is the
    prefix sum of lengths nearest to r/world of the total, so every rank's share is
    within one sequence of its ideal."""
    lens = [int(x) for x in lens]
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside [0, {world})")
    total = sum(lens)
    prefix = [0]
    for n in lens:
        prefix.append(prefix[-1] + n)
    bounds = [0]
    for r in range(1, world):
        goal = total * r / world
        bounds.append(min(range(bounds[-1], len(lens) + 1), key=lambda j: abs(prefix[j] - goal)))
    bounds.append(len(lens))
    lo, hi = bounds[rank], bounds[rank + 1]
    return SequenceShard(lo, hi, lens[lo:hi])


def head_shard(H: int, Hq: int, world: int, rank: int) -> HeadShard:
    """The KV heads of `rank` (an equal slice; H must divide by world) with their query
    heads."""
    if H % world or Hq % H:
        raise ValueError(f"{H} KV heads ({Hq} query heads) do not split over {world} ranks")
    h = H // world
    g = Hq // H
    return HeadShard(rank * h, h, rank * h * g, h * g)


class HeadGather:
    """All-gather of per-rank head outputs [B, Hq/world, T, D] into [B, Hq, T, D], the
    heads in global order (rank r holds query heads [r*Hq/world, (r+1)*Hq/world)).

    The receive buffer is allocated once per shape and reused, so a CUDA graph captured
    around the collective sees fixed addresses. The gathered heads are copied out of it
    into `out`, or into a new tensor when out is None (never a view of the buffer, which
    the next call overwrites)."""

    def __init__(self, world: int, group=None):
        self.world = world
        self.group = group
        self._bufs: dict[tuple, torch.Tensor] = {}

    def __call__(self, part: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        import torch.distributed as dist

        if self.world == 1:
            return part if out is None else out.copy_(part)
        b, hq, t, d = part.shape
        key = (part.device, part.dtype, b, hq, t, d)
        buf = self._bufs.get(key)
        if buf is None:
            buf = torch.empty((self.world, b, hq, t, d), device=part.device, dtype=part.dtype)
            self._bufs[key] = buf
        dist.all_gather_into_tensor(buf.view(self.world * b, hq, t, d), part.contiguous(), group=self.group)
        full = buf.permute(1, 0, 2, 3, 4)
        if out is None:
            out = torch.empty((b, self.world * hq, t, d), device=part.device, dtype=part.dtype)
        out.view(b, self.world, hq, t, d).copy_(full)
        return out


class PeerHeadGather:
    """The exchange of HeadGather by this library's own kernel (ma_head_gather): every rank
    stores its head outputs straight into every rank's receive region over NVLink -- its
    own device allocation, mapped into the peers through a CUDA IPC handle -- and waits
    (bounded) for every rank's flag of the call before copying the region out.

    One instance per process group, one rank per GPU; every rank makes the same calls in
    the same order, as with a collective. The first call of a shape allocates the region
    and exchanges the handles (torch.distributed, so it must run outside CUDA-graph
    capture); later calls, captured or not, launch two kernels. The attention can run the
    same exchange inside its own launch (splitk_attention(..., head_gather=(this,
    gathered)): its merge stores the rows, no further launch). A wait that gave up is
    reported by maskahead_b200.device_status()."""

    def __init__(self, world: int, rank: int, group=None):
        self.world, self.rank, self.group = world, rank, group
        self._regions: dict[tuple, tuple] = {}

    def _region(self, dev: torch.device, b: int, hq: int, t: int):
        import torch.distributed as dist

        from . import _lib

        key = (dev.index, b, hq, t)
        reg = self._regions.get(key)
        if reg is not None:
            return reg
        lib = _lib.lib()
        ptr = ctypes.c_void_p()
        _lib.check("ma_peer_alloc", lib.ma_peer_alloc(lib.ma_head_gather_region_bytes(b, hq, t), ctypes.byref(ptr)))
        torch.cuda.synchronize(dev)   # the zeroed region before any peer can write it
        hb = lib.ma_ipc_handle_bytes()
        handle = (ctypes.c_char * hb)()
        _lib.check("ma_ipc_get_handle", lib.ma_ipc_get_handle(ptr, handle))
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=self.group)
        bases, opened = [], []
        for p, h in enumerate(handles):
            if p == self.rank:
                bases.append(ptr.value)
                continue
            q = ctypes.c_void_p()
            _lib.check("ma_ipc_open_handle", lib.ma_ipc_open_handle((ctypes.c_char * hb).from_buffer_copy(h),
                                                                    ctypes.byref(q)))
            bases.append(q.value)
            opened.append(q.value)
        # the call counter and error word of this region (zeroed; ma_workspace_status reads it)
        ws = torch.zeros(lib.ma_head_gather_workspace() + 256, dtype=torch.uint8, device=dev)
        _lib.STATUS_EXTRA.append((dev.index, ws))
        dist.barrier(group=self.group)   # every rank mapped every region
        reg = (ptr, (ctypes.c_void_p * self.world)(*bases), opened, ws)
        self._regions[key] = reg
        return reg

    def region(self, dev: torch.device, b: int, hq: int, t: int):
        """(regions, workspace) of the exchange of [b, hq, t, 128] rows, for an attention
        launch that runs the exchange itself (splitk_attention's head_gather): the peers'
        regions as mapped here (a ctypes array) and this rank's counters. The first call
        of a shape allocates and maps (outside CUDA-graph capture, like __call__'s)."""
        _ptr, bases, _opened, ws = self._region(dev, b, hq, t)
        return bases, ws

    def __call__(self, part: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        from . import _lib

        if self.world == 1:
            return part if out is None else out.copy_(part)
        b, hl, t, d = part.shape
        if part.dtype != torch.bfloat16 or part.stride(-1) != 1:
            raise ValueError("part must be a bfloat16 [B, Hl, T, D] tensor with a contiguous last dimension")
        dev = part.device
        _ptr, bases, _opened, ws = self._region(dev, b, hl * self.world, t)
        if out is None:
            out = torch.empty((b, hl * self.world, t, d), device=dev, dtype=part.dtype)
        lib = _lib.lib()
        _lib.check("ma_head_gather", lib.ma_head_gather(
            part.data_ptr(), _lib.i64(*part.stride()[:3]), b, hl, t, d, self.world, self.rank, bases, out.data_ptr(),
            _lib.i64(*out.stride()[:3]), ws.data_ptr(), ws.numel(), _lib.stream_handle(dev)))
        return out

    def close(self) -> None:
        """Unmap the peers' regions and free this rank's (after a barrier: no rank may still
        write into them)."""
        import torch.distributed as dist

        from . import _lib

        if not self._regions:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        lib = _lib.lib()
        for ptr, _bases, opened, ws in self._regions.values():
            for q in opened:
                lib.ma_ipc_close_handle(q)
            lib.ma_peer_free(ptr)
            _lib.STATUS_EXTRA[:] = [(i, w) for i, w in _lib.STATUS_EXTRA if w is not ws]
        self._regions.clear()
