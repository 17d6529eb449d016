"""Multi-GPU partitioning of the decode path (one process per GPU, torch.distributed).

The path shards without exchanging KV data:

* **by KV head** (tensor parallel): rank r owns KV heads
  ``[r*H/N, (r+1)*H/N)`` with their query heads and a pool holding only those
  heads' pages; after the local decode one all-gather assembles the per-head
  outputs.  The local output is laid out head-major, ``(Hq_local, B, D)``, so
  the gathered buffer is a plain concatenation;
* **by sequence**: sequences are assigned to ranks by longest-processing-time
  first on their algorithmic bytes, each rank holds its sequences' pages, and
  no collective is needed for the decode itself (``gather_sequence_outputs``
  reassembles the batch when a caller wants it on every rank).

The reference has no multi-GPU code (it asserts batch 1, ``kitty/attention.py:100``);
these helpers are the B200 build's own.
"""

from __future__ import annotations

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
