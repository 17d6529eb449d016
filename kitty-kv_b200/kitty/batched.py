"""BatchedKVCache - the Kitty cache of many sequences, resident in device memory.

A decode step appends one token to each of n sequences with ONE library call
(``kitty_cache_append``: four launches, no host synchronisation, CUDA-graph
capturable) and attends over them with one more (``kitty_paged_decode`` with a
sequence map).  Per sequence it runs the state machine of the reference's
``KittyInferencePipeline.push_token`` (``kitty/pipeline.py:115-181``): the first
``sink_size`` tokens stay unquantised (float16 or bfloat16, ``config.dtype``) in the
sinks, later tokens fill a G-token buffer, and a full buffer is quantised into a
freshly allocated page.  The values of a
page are those of the same G tokens (the pipeline's ``align_values=True``
mode), so decode pairs every key with its own value.  Pages come from a
device-side free stack shared by all layers; it replaces the host free mask of
``PageCentricKVLayoutManager.allocate_page / free_sequence``
(``kitty/layout.py:161-220``).

Errors found on the device (pool exhausted, block table full, a sequence id
repeated in one step) drop the affected token, leave its sequence unchanged and
raise a sticky flag; :meth:`check_errors` reads it (and synchronises).
"""

from __future__ import annotations

import math
from typing import Dict, Optional

import torch

from .config import KittyConfig
from .kernels import _lib
from .kernels.attention import paged_attention_batched
from .layout import torch_dtype


class BatchedKVCache:
    """Device-resident Kitty cache of ``max_seqs`` sequence slots x ``num_layers`` layers.

    boost_idx_uint8: (num_layers, H, D) or (H, D) uint8 (the profiler's output).
    num_pages: pool size shared by all layers (default: every slot can reach
    ``config.max_seq_len`` tokens in every layer).
    """

    def __init__(self, config: KittyConfig, boost_idx_uint8: torch.Tensor, max_seqs: int,
                 num_pages: Optional[int] = None, max_pages_per_seq: Optional[int] = None,
                 device: Optional[torch.device] = None) -> None:
        self.config = config
        dev = torch.device(device if device is not None else config.device)
        if dev.type != "cuda":
            raise RuntimeError("BatchedKVCache lives in CUDA memory (there is no CPU path)")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        L, H, D = config.num_layers, config.num_kv_heads, config.head_dim
        S, G, K = config.sink_size, config.q_buffer_size, config.d_boost
        if max_pages_per_seq is None:
            max_pages_per_seq = max(1, -(-max(config.max_seq_len - S, 0) // G))
        if num_pages is None:
            num_pages = max_seqs * max_pages_per_seq * L
        self.device, self.max_seqs = dev, int(max_seqs)
        self.max_pages_per_seq, self.num_pages = int(max_pages_per_seq), int(num_pages)
        bidx = boost_idx_uint8.to(dev, torch.uint8)
        if bidx.dim() == 2:
            bidx = bidx.unsqueeze(0).expand(L, H, D)
        if tuple(bidx.shape) != (L, H, D):
            raise RuntimeError(f"boost_idx must be ({L}, {H}, {D}) or ({H}, {D}) uint8")
        self.boost_idx = bidx.contiguous()
        f16, i32 = torch_dtype(config.dtype), torch.int32      # float16 or bfloat16 buffers / metadata
        self.dtype = f16
        P, B, M = self.num_pages, self.max_seqs, self.max_pages_per_seq
        # pools (the layout manager's shapes, kitty/layout.py:128-147)
        self.key_baseline = torch.zeros(P, H, D, G // 4, dtype=torch.uint8, device=dev)
        self.key_boost = torch.zeros(P, H, K, G // 4, dtype=torch.uint8, device=dev)
        self.key_metadata = torch.zeros(P, H, 2, D, dtype=f16, device=dev)
        self.value_pool = torch.zeros(P, H, G, D // 4, dtype=torch.uint8, device=dev)
        self.value_metadata = torch.zeros(P, H, G, 2, dtype=f16, device=dev)
        # per-layer, per-slot state
        self.sink_k = torch.zeros(L, B, H, S, D, dtype=f16, device=dev)
        self.sink_v = torch.zeros(L, B, H, S, D, dtype=f16, device=dev)
        self.tail_k = torch.zeros(L, B, H, G, D, dtype=f16, device=dev)
        self.tail_v = torch.zeros(L, B, H, G, D, dtype=f16, device=dev)
        self.sink_len = torch.zeros(L, B, dtype=i32, device=dev)
        self.tail_len = torch.zeros(L, B, dtype=i32, device=dev)
        self.page_count = torch.zeros(L, B, dtype=i32, device=dev)
        self.block_table = torch.zeros(L, B, M, dtype=i32, device=dev)
        self._claim = torch.zeros(L, B, dtype=i32, device=dev)
        self._job_off = torch.zeros(L, B, dtype=torch.int64, device=dev)
        self._job_page = torch.zeros(L, B, dtype=i32, device=dev)
        self._job_slot = torch.zeros(L, B, dtype=i32, device=dev)
        # shared free-page stack
        self.free_pages = torch.zeros(max(P, 1), dtype=i32, device=dev)
        self.free_top = torch.zeros(1, dtype=i32, device=dev)
        self._states = [self._make_state(l) for l in range(L)]
        self.reset()

    # ------------------------------------------------------------------ state

    def _make_state(self, l: int) -> _lib.CacheState:
        c = self.config
        st = _lib.CacheState()
        st.max_seqs, st.num_heads, st.head_dim, st.group = self.max_seqs, c.num_kv_heads, c.head_dim, c.q_buffer_size
        st.sink_size, st.d_boost, st.sentinel = c.sink_size, c.d_boost, c.sentinel
        st.max_pages_per_seq, st.pool_pages = self.max_pages_per_seq, self.num_pages
        st.boost_idx, st.bidx_s_head = self.boost_idx[l].data_ptr(), self.boost_idx.stride(1)
        st.sink_k, st.sink_v = self.sink_k[l].data_ptr(), self.sink_v[l].data_ptr()
        st.tail_k, st.tail_v = self.tail_k[l].data_ptr(), self.tail_v[l].data_ptr()
        st.sink_len, st.tail_len = self.sink_len[l].data_ptr(), self.tail_len[l].data_ptr()
        st.num_pages, st.claim = self.page_count[l].data_ptr(), self._claim[l].data_ptr()
        st.block_table = self.block_table[l].data_ptr()
        st.free_pages, st.free_top = self.free_pages.data_ptr(), self.free_top.data_ptr()
        st.key_low, st.key_high = self.key_baseline.data_ptr(), self.key_boost.data_ptr()
        st.key_meta = self.key_metadata.data_ptr()
        st.val_codes, st.val_meta = self.value_pool.data_ptr(), self.value_metadata.data_ptr()
        st.job_off, st.job_page = self._job_off[l].data_ptr(), self._job_page[l].data_ptr()
        st.job_slot = self._job_slot[l].data_ptr()
        st.dtype = _lib.dtype_code(self.dtype)
        return st

    def state(self, layer_id: int) -> _lib.CacheState:
        """The C-ABI view (``KittyCacheState``) of one layer."""
        return self._states[layer_id]

    def _stream(self) -> int:
        return _lib.stream_ptr(self.device)

    def _ids(self, seq_ids) -> torch.Tensor:
        if not isinstance(seq_ids, torch.Tensor):
            seq_ids = torch.tensor(list(seq_ids), dtype=torch.int32)
        if seq_ids.dtype != torch.int32:
            seq_ids = seq_ids.to(torch.int32)
        if seq_ids.device != self.device:
            seq_ids = seq_ids.to(self.device, non_blocking=True)
        return seq_ids.contiguous().view(-1)

    # ------------------------------------------------------------------ API

    def reset(self) -> None:
        """Empty every slot of every layer; all pages back on the free stack."""
        lib = _lib.load()
        for st in self._states:
            _lib.check(lib.kitty_cache_reset(st, self._stream()), "kitty_cache_reset")

    def append(self, layer_id: int, seq_ids, key: torch.Tensor, value: torch.Tensor) -> None:
        """Append token row i of key / value ((n, H, D), the cache's dtype) to slot seq_ids[i] of
        ``layer_id``; slots whose buffer fills are quantised into new pages."""
        ids = self._ids(seq_ids)
        n = ids.numel()
        H, D = self.config.num_kv_heads, self.config.head_dim
        for t, name in ((key, "key"), (value, "value")):
            if t.dtype != self.dtype or t.device != self.device or tuple(t.shape) != (n, H, D):
                raise RuntimeError(f"{name} must be ({n}, {H}, {D}) {self.dtype} on {self.device}")
        if key.stride(2) != 1:
            key = key.contiguous()
        if value.stride(2) != 1:
            value = value.contiguous()
        lib = _lib.load()
        _lib.check(lib.kitty_cache_append(self._states[layer_id], n, ids.data_ptr(), key.data_ptr(),
                                          key.stride(0), key.stride(1), value.data_ptr(), value.stride(0),
                                          value.stride(1), self._stream()), "kitty_cache_append")

    def prefill(self, layer_id: int, seq_ids, key: torch.Tensor, value: torch.Tensor, lengths) -> None:
        """Append lengths[i] tokens to slot seq_ids[i] of ``layer_id`` in one call: the
        tokens of the i-th sequence are the next lengths[i] rows of key / value
        ((sum(lengths), H, D), the cache's dtype, sequences one after another).  Same result as
        appending them one at a time; full groups of G tokens are quantised straight
        from ``key`` / ``value``.  ``lengths``: host integers (they size the launch)."""
        lens = [int(x) for x in (lengths.tolist() if isinstance(lengths, torch.Tensor) else lengths)]
        ids = self._ids(seq_ids)
        n = ids.numel()
        if len(lens) != n or min(lens, default=0) < 0:
            raise RuntimeError("lengths must hold one non-negative count per sequence id")
        H, D, G = self.config.num_kv_heads, self.config.head_dim, self.config.q_buffer_size
        N = sum(lens)
        for t, name in ((key, "key"), (value, "value")):
            if t.dtype != self.dtype or t.device != self.device or tuple(t.shape) != (N, H, D):
                raise RuntimeError(f"{name} must be ({N}, {H}, {D}) {self.dtype} on {self.device}")
        if key.stride(2) != 1 or key.stride() != value.stride():
            key, value = key.contiguous(), value.contiguous()
        starts = [0] * n
        for i in range(1, n):
            starts[i] = starts[i - 1] + lens[i - 1]
        dev = self.device
        host = torch.tensor(lens + [0] * (2 * n), dtype=torch.int64).pin_memory()
        host[n:2 * n] = torch.tensor(starts, dtype=torch.int64)
        meta = host.to(dev, non_blocking=True)
        lens_d = meta[:n].to(torch.int32)
        max_pages = sum(x // G for x in lens)
        page_off = torch.empty(max(max_pages, 1), dtype=torch.int64, device=dev)
        page_dst = torch.empty(max(max_pages, 1), dtype=torch.int32, device=dev)
        plan = torch.empty(6 * n, dtype=torch.int32, device=dev)
        a = _lib.PrefillArgs()
        a.n, a.seq_ids, a.lengths, a.row_start = n, ids.data_ptr(), lens_d.data_ptr(), meta[n:2 * n].data_ptr()
        a.key, a.value, a.s_tok, a.s_head = key.data_ptr(), value.data_ptr(), key.stride(0), key.stride(1)
        a.max_pages, a.page_off, a.page_dst, a.seq_plan = max_pages, page_off.data_ptr(), page_dst.data_ptr(), \
            plan.data_ptr()
        _lib.check(_lib.load().kitty_cache_prefill(self._states[layer_id], a, self._stream()), "kitty_cache_prefill")

    def release(self, seq_ids) -> None:
        """Empty the given slots in every layer and return their pages to the stack."""
        ids = self._ids(seq_ids)
        lib = _lib.load()
        for st in self._states:
            _lib.check(lib.kitty_cache_release(st, ids.numel(), ids.data_ptr(), self._stream()),
                       "kitty_cache_release")

    def decode(self, layer_id: int, q: torch.Tensor, seq_ids, out: Optional[torch.Tensor] = None,
               sm_scale: Optional[float] = None, num_splits: int = 0) -> torch.Tensor:
        """Decode attention of row i of q ((n, Hq, D)) over slot seq_ids[i]; float16 output."""
        ids = self._ids(seq_ids)
        l = layer_id
        return paged_attention_batched(
            q, self.block_table[l], self.page_count[l], self.key_baseline, self.key_boost,
            self.key_metadata, self.value_pool, self.value_metadata, self.boost_idx[l], self.config.d_boost,
            sink_k=self.sink_k[l] if self.config.sink_size else None,
            sink_v=self.sink_v[l] if self.config.sink_size else None,
            sink_len=self.sink_len[l] if self.config.sink_size else None,
            tail_k=self.tail_k[l], tail_v=self.tail_v[l], tail_len=self.tail_len[l], out=out,
            num_splits=num_splits, sm_scale=(1.0 / math.sqrt(self.config.head_dim)) if sm_scale is None
            else sm_scale, max_pages_per_seq=self.max_pages_per_seq, seq_map=ids)

    # ------------------------------------------------------------------ inspection (synchronising)

    def free_page_count(self) -> int:
        return int(self.free_top.item())

    def lengths(self, layer_id: int) -> Dict[str, torch.Tensor]:
        """Host copies of the per-slot counters of one layer."""
        return {"sink_len": self.sink_len[layer_id].cpu(), "tail_len": self.tail_len[layer_id].cpu(),
                "num_pages": self.page_count[layer_id].cpu()}

    def check_errors(self, clear: bool = True) -> None:
        """Raise if an append / release since the last check set a device error flag."""
        bits = _lib.device_error_flags(clear=clear)
        msgs = [m for b, m in _lib.CACHE_ERRORS.items() if bits & b]
        if bits & 1:
            msgs.append("a decode kernel timed out waiting for a copy")
        if msgs:
            raise RuntimeError("Kitty cache: " + "; ".join(msgs))
