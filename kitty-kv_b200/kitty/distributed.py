"""Multi-GPU partitioning of the decode path (one process per GPU, torch.distributed).

The path shards without exchanging KV data:

* **by KV head** (tensor parallel): rank r owns KV heads
  ``[r*H/N, (r+1)*H/N)`` with their query heads and a pool holding only those
  heads' pages; after the local decode one all-gather assembles the per-head
  outputs.  The local output is laid out head-major, ``(Hq_local, B, D)``, so
  the gathered buffer is a plain concatenation.  ``gather_head_outputs`` runs it
  as an NCCL all-gather, ``PeerGather`` as direct NVLink stores into every rank's
  exchange region (the library's ``kitty_tp_allgather``);
* **by sequence**: sequences are assigned to ranks by longest-processing-time
  first on their algorithmic bytes, each rank holds its sequences' pages, and
  no collective is needed for the decode itself (``gather_sequence_outputs``
  reassembles the batch when a caller wants it on every rank).

The reference has no multi-GPU code (it asserts batch 1, ``kitty/attention.py:100``);
these helpers are the B200 build's own.
"""

from __future__ import annotations

import ctypes
import heapq
from typing import List, Sequence, Tuple

import torch
import torch.distributed as dist


def kv_head_range(num_kv_heads: int, world: int, rank: int) -> Tuple[int, int]:
    """KV heads owned by ``rank`` when sharding by head (requires H % world == 0)."""
    if num_kv_heads % world != 0:
        raise ValueError(f"{num_kv_heads} KV heads do not split evenly over {world} ranks")
    per = num_kv_heads // world
    return rank * per, (rank + 1) * per


def q_head_range(num_q_heads: int, num_kv_heads: int, world: int, rank: int) -> Tuple[int, int]:
    """Query heads that read the KV heads of ``rank`` (GQA groups are contiguous)."""
    h0, h1 = kv_head_range(num_kv_heads, world, rank)
    g = num_q_heads // num_kv_heads
    return h0 * g, h1 * g


def lpt_assign(costs: Sequence[float], world: int) -> List[List[int]]:
    """Longest-processing-time-first assignment of items to ``world`` bins.

    Items are taken in decreasing cost order (ties by index) and each goes to the
    currently least-loaded bin (ties by bin index).  Returns the item indices per
    bin, each list in increasing index order."""
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0.0, r) for r in range(world)]
    bins: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        bins[r].append(i)
        heapq.heappush(heap, (load + float(costs[i]), r))
    return [sorted(b) for b in bins]


def sequence_costs(num_pages: Sequence[int], sink_lens: Sequence[int], tail_lens: Sequence[int],
                   num_kv_heads: int, page_head_bytes: int, head_dim: int) -> List[float]:
    """Algorithmic bytes one decode step reads for each sequence."""
    return [num_kv_heads * (n * page_head_bytes + (s + t) * head_dim * 4)
            for n, s, t in zip(num_pages, sink_lens, tail_lens)]


def gather_head_outputs(out_local: torch.Tensor, group=None, full: torch.Tensor = None) -> torch.Tensor:
    """All-gather per-rank head-major outputs ``(Hq_local, B, D)`` into the head-major
    buffer ``full`` ``(Hq, B, D)`` (allocated when not given; pass one to keep the call
    free of allocation, e.g. inside a CUDA graph) and return it viewed as ``(B, Hq, D)``.

    Rank r's heads land at ``[r*Hq_local, (r+1)*Hq_local)``.  The returned tensor is
    ``full.permute(1, 0, 2)``: a strided view (strides ``(D, B*D, 1)``), not a
    contiguous tensor; call ``.contiguous()`` where a dense ``(B, Hq, D)`` is needed.
    The decode entry points accept it as ``out`` directly (they take any head and
    sequence strides), and a rank's own decode can write its ``(Hq_local, B, D)``
    slice head-major the same way, so no copy is needed on either side."""
    world = dist.get_world_size(group)
    hq_local, B, D = out_local.shape
    if full is None:
        full = torch.empty(world * hq_local, B, D, dtype=out_local.dtype, device=out_local.device)
    elif tuple(full.shape) != (world * hq_local, B, D) or not full.is_contiguous():
        raise RuntimeError("full must be a contiguous (world * Hq_local, B, D) tensor")
    dist.all_gather_into_tensor(full, out_local.contiguous(), group=group)
    return full.permute(1, 0, 2)


class PeerGather:
    """The all-gather of ``gather_head_outputs`` over NVLink peer memory instead of a
    library collective (``kitty_tp_allgather`` in the C ABI).

    Construction is collective (every rank of ``group`` builds one with the same
    shapes): each rank allocates an exchange region through the library, the CUDA IPC
    handles are exchanged with ``all_gather_object`` and every peer's region is mapped
    into this process.  Each call then stores this rank's ``(Hq_local, B, D)`` slice
    straight into every rank's region and waits (bounded) until all slices of the call
    have arrived, copying the assembled ``(Hq, B, D)`` into ``full``: two kernels on the
    current stream, no host synchronisation, capturable in a CUDA graph.  Every rank
    must make the same sequence of calls.  ``close()`` (collective) unmaps and frees."""

    def __init__(self, hq_local: int, batch: int, head_dim: int, dtype=torch.float16, device=None, group=None):
        from .kernels import _lib
        self._lib = _lib
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _lib.TP_MAX_RANKS:
            raise ValueError(f"peer gather supports at most {_lib.TP_MAX_RANKS} ranks, got {self.world}")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.shape_local = (hq_local, batch, head_dim)
        self.dtype = dtype
        elem = torch.empty(0, dtype=dtype).element_size()
        self.local_bytes = hq_local * batch * head_dim * elem
        if self.local_bytes % 16:
            raise ValueError("the per-rank slice must be a multiple of 16 bytes")
        self.data_bytes = self.world * self.local_bytes
        lib = _lib.load()
        self._region = None
        self._opened = []
        with torch.cuda.device(self.device):
            region = _lib.c_ptr()
            _lib.check(lib.kitty_tp_region_alloc(self.data_bytes, ctypes.byref(region)), "kitty_tp_region_alloc")
            self._region = region.value
            handle = ctypes.create_string_buffer(64)
            _lib.check(lib.kitty_tp_ipc_handle(self._region, handle), "kitty_tp_ipc_handle")
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=group)
            self.args = _lib.TpGatherArgs()
            self.args.world, self.args.rank = self.world, self.rank
            self.args.data_bytes = self.data_bytes
            self.args.src_bytes = self.local_bytes
            self.args.dst_offset = self.rank * self.local_bytes
            error = ""
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.args.region[r] = self._region
                    continue
                p = _lib.c_ptr()
                if lib.kitty_tp_ipc_open(ctypes.create_string_buffer(h, 64), ctypes.byref(p)) != 0:
                    error = f"rank {self.rank}: mapping rank {r}'s region failed: {lib.kitty_last_error().decode()}"
                    break
                self._opened.append(p.value)
                self.args.region[r] = p.value
        # every rank learns whether every mapping succeeded (so all of them raise
        # together instead of some waiting for the others), and no rank stores before
        # every region is mapped everywhere
        errors = [None] * self.world
        dist.all_gather_object(errors, error, group=group)
        failed = [e for e in errors if e]
        if failed:
            self.close(collective=False)
            raise RuntimeError("peer-memory exchange unavailable: " + "; ".join(failed))

    def __call__(self, out_local: torch.Tensor, full: torch.Tensor = None) -> torch.Tensor:
        """Same contract as ``gather_head_outputs``: returns ``full.permute(1, 0, 2)``."""
        if tuple(out_local.shape) != self.shape_local or out_local.dtype != self.dtype or not out_local.is_contiguous():
            raise RuntimeError(f"out_local must be a contiguous {self.shape_local} {self.dtype} tensor")
        hq_local, B, D = self.shape_local
        if full is None:
            full = torch.empty(self.world * hq_local, B, D, dtype=self.dtype, device=out_local.device)
        elif tuple(full.shape) != (self.world * hq_local, B, D) or not full.is_contiguous() or full.dtype != self.dtype:
            raise RuntimeError("full must be a contiguous (world * Hq_local, B, D) tensor of the slice's dtype")
        self.args.src = out_local.data_ptr()
        self.args.dst = full.data_ptr()
        self._lib.check(self._lib.load().kitty_tp_allgather(ctypes.byref(self.args),
                                                            self._lib.stream_ptr(out_local.device)),
                        "kitty_tp_allgather")
        return full.permute(1, 0, 2)

    def close(self, collective: bool = True) -> None:
        """Collective (unless ``collective`` is False, for a construction that failed on
        every rank alike): after every rank's calls have completed, unmap the peers'
        regions and free this rank's own."""
        if self._region is None:
            return
        lib = self._lib.load()
        torch.cuda.synchronize(self.device)
        if collective:
            dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                self._lib.check(lib.kitty_tp_ipc_close(p), "kitty_tp_ipc_close")
            self._opened = []
            self._lib.check(lib.kitty_tp_region_free(self._region), "kitty_tp_region_free")
        self._region = None


def gather_sequence_outputs(out_local: torch.Tensor, assignment: List[List[int]], group=None) -> torch.Tensor:
    """Reassemble ``(B, Hq, D)`` from per-rank outputs of their assigned sequences
    (rows in the order of ``assignment[rank]``); pads to the largest share."""
    world = dist.get_world_size(group)
    rows = max(len(a) for a in assignment)
    _, Hq, D = out_local.shape
    pad = torch.zeros(rows, Hq, D, dtype=out_local.dtype, device=out_local.device)
    pad[:out_local.shape[0]] = out_local
    full = torch.empty(world * rows, Hq, D, dtype=out_local.dtype, device=out_local.device)
    dist.all_gather_into_tensor(full, pad, group=group)
    B = sum(len(a) for a in assignment)
    out = torch.empty(B, Hq, D, dtype=out_local.dtype, device=out_local.device)
    for r, seqs in enumerate(assignment):
        if seqs:
            out[torch.tensor(seqs, device=out.device)] = full[r * rows:r * rows + len(seqs)]
    return out
