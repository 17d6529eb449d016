"""PageCentricKVLayoutManager - HBM page pools, free list and page table.

Same pools (shapes, dtypes, order), accessors and allocation policy as the
reference (``kitty/layout.py:75-316``):

    key_baseline   (P, H, D, G/4)  uint8   low 2 bits of every channel
    key_boost      (P, H, K, G/4)  uint8   high 2 bits of the K boosted channels
    key_metadata   (P, H, 2, D)    fp16    row 0 scale, row 1 zero-point
    value_pool     (P, H, G, D/4)  uint8   per-token INT2 codes
    value_metadata (P, H, G, 2)    fp16    per-token (scale, zero-point)

These pools are the operands of the CUDA kernels, so their layout is the
contract.  Allocation keeps the reference's "lowest free index first" policy
(``layout.py:186-191``) but uses a min-heap instead of a ``nonzero`` scan of a
device mask, and page lists are also available as int32 device block tables
for the batched decode kernel.
"""

from __future__ import annotations

import heapq
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from .config import KittyConfig


@dataclass
class Page:
    """A quantised page (G tokens of all KV heads of one layer)."""
    physical_idx: int
    layer_id: int
    head_id: int
    seq_id: int
    start_token: int
    num_tokens: int = 0
    group: int = 0

    @property
    def is_full(self) -> bool:
        return self.num_tokens == self.group

    def __repr__(self) -> str:
        return (f"Page(phys={self.physical_idx}, layer={self.layer_id}, head={self.head_id}, "
                f"seq={self.seq_id}, tokens=[{self.start_token}..{self.start_token + self.num_tokens}))")


def torch_dtype(name: str) -> torch.dtype:
    return torch.float16 if name == "float16" else torch.bfloat16


class PageCentricKVLayoutManager:
    """Pre-allocated page pools plus the allocator and the logical page table.

    boost_idx_uint8: (num_layers, num_kv_heads, head_dim) uint8 from the
    sensitivity profiler (moved to ``config.device``).
    """

    def __init__(self, config: KittyConfig, boost_idx_uint8: torch.Tensor,
                 num_pages: Optional[int] = None) -> None:
        self.config = config
        dev = torch.device(config.device)
        self.boost_idx_uint8 = boost_idx_uint8.to(dev)
        G, D, K, H = config.q_buffer_size, config.head_dim, config.d_boost, config.num_kv_heads
        P = config.max_pages if num_pages is None else int(num_pages)
        self.num_pages_total = P
        self._torch_dtype = torch_dtype(config.dtype)
        self.key_baseline = torch.zeros(P, H, D, G // 4, dtype=torch.uint8, device=dev)
        self.key_boost = torch.zeros(P, H, K, G // 4, dtype=torch.uint8, device=dev)
        self.key_metadata = torch.zeros(P, H, 2, D, dtype=self._torch_dtype, device=dev)
        self.value_pool = torch.zeros(P, H, G, D // 4, dtype=torch.uint8, device=dev)
        self.value_metadata = torch.zeros(P, H, G, 2, dtype=self._torch_dtype, device=dev)
        self._free_heap: List[int] = list(range(P))
        self._num_free = P
        self._page_table: Dict[Tuple[int, int, int], int] = {}
        self._pages: Dict[int, Page] = {}

    # ------------------------------------------------------------ allocation

    def allocate_page(self, seq_id: int, layer_id: int, page_number: int) -> Page:
        """Take the lowest free physical page; raise RuntimeError when exhausted."""
        if self._num_free == 0:
            raise RuntimeError(
                "KV Cache page pool exhausted! "
                f"All {self.num_pages_total} pages are in use. "
                "Increase config.max_pages or reduce max_seq_len/max_batch_size.")
        phys = heapq.heappop(self._free_heap)
        self._num_free -= 1
        page = Page(physical_idx=phys, layer_id=layer_id, head_id=-1, seq_id=seq_id,
                    start_token=page_number * self.config.q_buffer_size, group=self.config.q_buffer_size)
        self._page_table[(seq_id, layer_id, page_number)] = phys
        self._pages[phys] = page
        return page

    def free_page(self, seq_id: int, layer_id: int, page_number: int) -> None:
        phys = self._page_table.pop((seq_id, layer_id, page_number), None)
        if phys is None:
            return
        self._pages.pop(phys, None)
        heapq.heappush(self._free_heap, phys)
        self._num_free += 1

    def free_sequence(self, seq_id: int) -> None:
        for key in [k for k in self._page_table if k[0] == seq_id]:
            self.free_page(*key)

    def get_physical_idx(self, seq_id: int, layer_id: int, page_number: int) -> int:
        key = (seq_id, layer_id, page_number)
        if key not in self._page_table:
            raise KeyError(f"Page {key} not found in page table.")
        return self._page_table[key]

    # ------------------------------------------------------------ accessors

    def key_baseline_page(self, phys_idx: int) -> torch.Tensor:
        return self.key_baseline[phys_idx]

    def key_boost_page(self, phys_idx: int) -> torch.Tensor:
        return self.key_boost[phys_idx]

    def key_meta_page(self, phys_idx: int) -> torch.Tensor:
        return self.key_metadata[phys_idx]

    def value_page(self, phys_idx: int) -> torch.Tensor:
        return self.value_pool[phys_idx]

    def value_meta_page(self, phys_idx: int) -> torch.Tensor:
        return self.value_metadata[phys_idx]

    # ------------------------------------------------------------ page lists

    def get_page_list(self, seq_id: int, layer_id: int) -> List[int]:
        """Physical pages of (seq, layer) in logical order (stops at the first gap)."""
        pages = []
        n = 0
        while (seq_id, layer_id, n) in self._page_table:
            pages.append(self._page_table[(seq_id, layer_id, n)])
            n += 1
        return pages

    def block_table(self, seq_ids: Sequence[int], layer_id: int, device=None,
                    width: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """(B, width) int32 block table and (B,) int32 page counts for the batched
        decode kernel, built from the page lists of ``seq_ids``."""
        lists = [self.get_page_list(s, layer_id) for s in seq_ids]
        w = max([len(x) for x in lists] + [1]) if width is None else int(width)
        bt = torch.zeros(len(lists), w, dtype=torch.int32)
        for i, pl in enumerate(lists):
            if len(pl) > w:
                raise RuntimeError(f"sequence {seq_ids[i]} has {len(pl)} pages, block table width is {w}")
            if pl:
                bt[i, :len(pl)] = torch.tensor(pl, dtype=torch.int32)
        n = torch.tensor([len(x) for x in lists], dtype=torch.int32)
        dev = torch.device(self.config.device) if device is None else torch.device(device)
        return bt.to(dev), n.to(dev)

    # ------------------------------------------------------------ stats

    def memory_stats(self) -> Dict[str, float]:
        def mb(t: torch.Tensor) -> float:
            return t.numel() * t.element_size() / (1024 ** 2)
        pools = [self.key_baseline, self.key_boost, self.key_metadata, self.value_pool, self.value_metadata]
        return {
            "key_baseline_MB": mb(self.key_baseline),
            "key_boost_MB": mb(self.key_boost),
            "key_metadata_MB": mb(self.key_metadata),
            "value_pool_MB": mb(self.value_pool),
            "value_metadata_MB": mb(self.value_metadata),
            "total_MB": sum(mb(t) for t in pools),
            "pages_free": self._num_free,
            "pages_used": self.num_pages_total - self._num_free,
            "pages_total": self.num_pages_total,
        }

    def __repr__(self) -> str:
        s = self.memory_stats()
        return (f"PageCentricKVLayoutManager(\n"
                f"  key_baseline:  {tuple(self.key_baseline.shape)}  uint8\n"
                f"  key_boost:     {tuple(self.key_boost.shape)}  uint8\n"
                f"  key_metadata:  {tuple(self.key_metadata.shape)}  {self.key_metadata.dtype}\n"
                f"  value_pool:    {tuple(self.value_pool.shape)}  uint8\n"
                f"  value_metadata:{tuple(self.value_metadata.shape)}  {self.value_metadata.dtype}\n"
                f"  Pages: {s['pages_used']}/{s['pages_total']} used  ({s['total_MB']:.1f} MB total)\n)")
