"""KittyInferencePipeline - the fp16 buffer state machine around the page pools.

Same buffers, counters and public methods as the reference
(``kitty/pipeline.py:49-326``): attention sinks (S tokens, fp16 forever), the
Key Q-buffer (G tokens, quantised into a page when full), the Value local
window (the R most recent values) and the Value Q-buffer (values evicted from
the window).  A flush now runs two CUDA launches per layer (all KV heads of
the page at once) instead of a Python loop of per-head kernels with host
round-trips.

Two deliberate differences, both documented in the repository's design notes:

* Counters are kept per layer.  The reference advances shared counters only
  when layer 0 pushes and flushes every layer from inside layer 0's push
  (``pipeline.py:146-148,171-181``), which shifts the buffer positions of
  layers >= 1; with ``num_layers == 1`` both behave identically.
* ``align_values=True`` (default) quantises each value page from the values of
  the same G tokens as its key page and exposes the matching fp16 value tail,
  so decode attention pairs every key with its own value at every step.  The
  reference quantises the Value Q-buffer instead (value pages lag key pages
  by R tokens and page 0 holds zeros when R == G) and its decode raises a
  broadcast error whenever the key tail and the value window differ in
  length.  ``align_values=False`` reproduces the reference's page bytes exactly
  (checked against recorded reference output for ``num_layers == 1``).
"""

from __future__ import annotations

from collections import defaultdict
from typing import Dict, List, Tuple

import torch

from .config import KittyConfig
from .kernels import _lib
from .kernels.quantize_key import quantize_key_pages
from .kernels.quantize_value import quantize_value_pages
from .layout import PageCentricKVLayoutManager, torch_dtype


class KittyInferencePipeline:
    """Runtime KV-cache buffer state machine (all layers, all KV heads).

    boost_idx_uint8: (num_layers, num_kv_heads, head_dim) uint8.
    """

    def __init__(self, config: KittyConfig, layout: PageCentricKVLayoutManager,
                 boost_idx_uint8: torch.Tensor, align_values: bool = True) -> None:
        self.config = config
        self.layout = layout
        self.boost_idx_uint8 = boost_idx_uint8
        self.align_values = align_values
        L, H, D = config.num_layers, config.num_kv_heads, config.head_dim
        S, G, R = config.sink_size, config.q_buffer_size, config.local_value_window
        dev = torch.device(config.device)
        self._dtype = torch_dtype(config.dtype)
        self.sink_k = torch.zeros(L, H, S, D, dtype=self._dtype, device=dev)
        self.sink_v = torch.zeros(L, H, S, D, dtype=self._dtype, device=dev)
        self.key_qbuf = torch.zeros(L, H, G, D, dtype=self._dtype, device=dev)
        self.val_local = torch.zeros(L, H, R, D, dtype=self._dtype, device=dev)
        self.val_qbuf = torch.zeros(L, H, G, D, dtype=self._dtype, device=dev)
        # values of the tokens currently in the Key Q-buffer (align_values mode)
        self.val_tail = torch.zeros(L, H, G, D, dtype=self._dtype, device=dev) if align_values else None
        self._sink_fill = [0] * L
        self._kq = [0] * L
        self._vl = [0] * L
        self._vq = [0] * L
        self._page_counter: Dict[Tuple[int, int], int] = defaultdict(int)
        self._bidx_dev = None

    # reference attributes (shared counters there; layer 0's here)
    @property
    def sink_fill(self) -> int:
        return self._sink_fill[0]

    @property
    def key_qbuf_len(self) -> int:
        return self._kq[0]

    @property
    def val_local_len(self) -> int:
        return self._vl[0]

    @property
    def val_qbuf_len(self) -> int:
        return self._vq[0]

    def layer_state(self, layer_id: int) -> Dict[str, int]:
        return {"sink_fill": self._sink_fill[layer_id], "key_qbuf_len": self._kq[layer_id],
                "val_local_len": self._vl[layer_id], "val_qbuf_len": self._vq[layer_id]}

    # ------------------------------------------------------------------ push

    def push_token(self, layer_id: int, key: torch.Tensor, value: torch.Tensor, seq_id: int = 0) -> None:
        """Append one (num_kv_heads, head_dim) key/value token to ``layer_id``."""
        cfg = self.config
        S, G, R = cfg.sink_size, cfg.q_buffer_size, cfg.local_value_window
        l = layer_id
        key = key.to(self._dtype).to(self.sink_k.device)
        value = value.to(self._dtype).to(self.sink_v.device)

        if self._sink_fill[l] < S:
            pos = self._sink_fill[l]
            self.sink_k[l, :, pos, :] = key
            self.sink_v[l, :, pos, :] = value
            self._sink_fill[l] += 1
            return

        kq = self._kq[l]
        self.key_qbuf[l, :, kq, :] = key
        if self.val_tail is not None:
            self.val_tail[l, :, kq, :] = value

        if self._vl[l] < R:
            self.val_local[l, :, self._vl[l], :] = value
            self._vl[l] += 1
        else:
            if R > 0:
                oldest = self.val_local[l, :, 0, :].clone()
                self.val_local[l, :, :R - 1, :] = self.val_local[l, :, 1:R, :].clone()
                self.val_local[l, :, R - 1, :] = value
            else:
                oldest = value
            self.val_qbuf[l, :, self._vq[l], :] = oldest
            self._vq[l] += 1

        self._kq[l] += 1
        if self._kq[l] == G:
            self._flush(l, seq_id)

    def push_tokens(self, layer_id: int, keys: torch.Tensor, values: torch.Tensor, seq_id: int = 0) -> None:
        """Append T tokens at once: keys / values (num_kv_heads, T, head_dim).

        Same end state as T calls of :meth:`push_token` (buffers, counters, value
        window, pages and their bytes).  With ``align_values=True`` every full group
        of G tokens is quantised straight from ``keys`` / ``values`` in one launch per
        tensor (the reference pushes a prefill token by token,
        ``kitty/attention.py:169-177``); ``align_values=False`` keeps the per-token
        path, whose value pages depend on the window's evictions token by token.
        """
        keys = keys.to(self._dtype).to(self.sink_k.device)
        values = values.to(self._dtype).to(self.sink_v.device)
        T = keys.shape[1]
        if not self.align_values:
            for t in range(T):
                self.push_token(layer_id, keys[:, t], values[:, t], seq_id)
            return
        cfg = self.config
        S, G = cfg.sink_size, cfg.q_buffer_size
        l = layer_id
        t = min(max(S - self._sink_fill[l], 0), T)
        if t > 0:
            f = self._sink_fill[l]
            self.sink_k[l, :, f:f + t] = keys[:, :t]
            self.sink_v[l, :, f:f + t] = values[:, :t]
            self._sink_fill[l] += t
        if t == T:
            return
        self._window_push(l, values[:, t:])
        kq = self._kq[l]
        if kq > 0:
            pre = min(G - kq, T - t)
            self.key_qbuf[l, :, kq:kq + pre] = keys[:, t:t + pre]
            self.val_tail[l, :, kq:kq + pre] = values[:, t:t + pre]
            self._kq[l] += pre
            t += pre
            if self._kq[l] == G:
                self._flush_buffers(l, seq_id)
        m = (T - t) // G
        if m > 0:
            keys_c, values_c = keys.contiguous(), values.contiguous()
            dev = keys_c.device
            pages = []
            for _ in range(m):
                page_num = self._page_counter[(seq_id, l)]
                pages.append(self.layout.allocate_page(seq_id=seq_id, layer_id=l, page_number=page_num).physical_idx)
                self._page_counter[(seq_id, l)] += 1
            dst = torch.tensor(pages, dtype=torch.int32).to(dev, non_blocking=True)
            offs = (torch.arange(m, dtype=torch.int64) * G + t) * keys_c.stride(1)
            offs = offs.to(dev, non_blocking=True)
            H, D, K = cfg.num_kv_heads, cfg.head_dim, cfg.d_boost
            quantize_key_pages(keys_c, offs, (keys_c.stride(0), keys_c.stride(1), keys_c.stride(2)),
                               self._boost_idx_dev()[l], K, cfg.sentinel, dst, self.layout.key_baseline,
                               self.layout.key_boost, self.layout.key_metadata, H, D, G)
            quantize_value_pages(values_c, offs, (values_c.stride(0), values_c.stride(1), values_c.stride(2)), dst,
                                 self.layout.value_pool, self.layout.value_metadata, H, D, G)
            t += m * G
        rem = T - t
        if rem > 0:
            self.key_qbuf[l, :, :rem] = keys[:, t:]
            self.val_tail[l, :, :rem] = values[:, t:]
            self._kq[l] = rem

    def _window_push(self, l: int, new_values: torch.Tensor) -> None:
        """Value window (R most recent values) and Value Q-buffer after pushing the
        (H, n, D) values one by one, with the Q-buffer emptied whenever the Key
        Q-buffer reaches G tokens (push_token's bookkeeping, vectorised)."""
        G, R = self.config.q_buffer_size, self.config.local_value_window
        n = new_values.shape[1]
        vl0, vq0, kq0 = self._vl[l], self._vq[l], self._kq[l]
        W = torch.cat([self.val_local[l, :, :vl0], new_values], dim=1)   # oldest first
        first = max(1, R - vl0 + 1)             # push index (1-based) of the first eviction
        flushes = [p for p in range(1, n + 1) if (kq0 + p) % G == 0]
        start = flushes[-1] + 1 if flushes else 1
        lo = max(start, first)
        ev = W[:, lo - first:n - first + 1] if n >= lo else W[:, :0]      # values evicted after the last flush
        if flushes:
            self.val_qbuf[l].zero_()
            base = 0
        else:
            base = vq0
        if ev.shape[1]:
            self.val_qbuf[l, :, base:base + ev.shape[1]] = ev
        self._vq[l] = base + ev.shape[1]
        keep = min(R, vl0 + n)
        if keep:
            self.val_local[l, :, :keep] = W[:, W.shape[1] - keep:]
        self._vl[l] = keep

    def _trigger_quantization(self, triggering_layer_id: int, seq_id: int) -> None:
        """Flush the Q-buffers of ``triggering_layer_id`` into a new page."""
        self._flush(triggering_layer_id, seq_id)

    def _boost_idx_dev(self) -> torch.Tensor:
        if self._bidx_dev is None:
            self._bidx_dev = self.boost_idx_uint8.to(self.key_qbuf.device).contiguous()
        return self._bidx_dev

    def _flush(self, l: int, seq_id: int) -> None:
        self._flush_buffers(l, seq_id)
        self.val_qbuf[l].zero_()
        self._vq[l] = 0

    def _flush_buffers(self, l: int, seq_id: int) -> None:
        """Quantise the Key Q-buffer and its value page into a new page; empty the
        Key Q-buffer (and the aligned value tail)."""
        cfg = self.config
        G, H, D, K = cfg.q_buffer_size, cfg.num_kv_heads, cfg.head_dim, cfg.d_boost
        page_num = self._page_counter[(seq_id, l)]
        page = self.layout.allocate_page(seq_id=seq_id, layer_id=l, page_number=page_num)
        self._page_counter[(seq_id, l)] += 1
        dev = self.key_qbuf.device
        dst = torch.tensor([page.physical_idx], dtype=torch.int32).to(dev, non_blocking=True)
        zero_off = _lib.zeros_const(dev, torch.int64)
        kb = self.key_qbuf[l]
        quantize_key_pages(kb, zero_off, (kb.stride(0), kb.stride(1), kb.stride(2)), self._boost_idx_dev()[l],
                           K, cfg.sentinel, dst, self.layout.key_baseline, self.layout.key_boost,
                           self.layout.key_metadata, H, D, G)
        if self.val_tail is not None:
            vb, n_valid = self.val_tail[l], None
        else:
            vb = self.val_qbuf[l]
            n_valid = torch.tensor([self._vq[l]], dtype=torch.int32).to(dev, non_blocking=True)
        quantize_value_pages(vb, zero_off, (vb.stride(0), vb.stride(1), vb.stride(2)), dst,
                             self.layout.value_pool, self.layout.value_metadata, H, D, G, n_valid=n_valid)
        self.key_qbuf[l].zero_()
        self._kq[l] = 0
        if self.val_tail is not None:
            self.val_tail[l].zero_()

    # ------------------------------------------------------------------ query

    def get_attention_context(self, layer_id: int, seq_id: int = 0) -> dict:
        """fp16 regions and page list for decode attention of ``layer_id``.

        Keys as in the reference: ``sink_k``, ``sink_v``, ``key_qbuf``,
        ``val_local``, ``page_list``; plus ``value_tail`` (values of the
        ``key_qbuf`` tokens) when ``align_values`` is on.
        """
        l = layer_id
        s, q, r = self._sink_fill[l], self._kq[l], self._vl[l]
        ctx = {
            "sink_k": self.sink_k[l, :, :s, :],
            "sink_v": self.sink_v[l, :, :s, :],
            "key_qbuf": self.key_qbuf[l, :, :q, :],
            "val_local": self.val_local[l, :, :r, :],
            "page_list": self.layout.get_page_list(seq_id=seq_id, layer_id=l),
        }
        if self.val_tail is not None:
            ctx["value_tail"] = self.val_tail[l, :, :q, :]
        return ctx

    # ------------------------------------------------------------------ reset

    def reset_sequence(self, seq_id: int = 0) -> None:
        """Free the sequence's pages and clear every buffer and counter."""
        self.layout.free_sequence(seq_id)
        for k in [k for k in self._page_counter if k[0] == seq_id]:
            del self._page_counter[k]
        L = self.config.num_layers
        self._sink_fill, self._kq, self._vl, self._vq = [0] * L, [0] * L, [0] * L, [0] * L
        for t in (self.sink_k, self.sink_v, self.key_qbuf, self.val_local, self.val_qbuf, self.val_tail):
            if t is not None:
                t.zero_()

    def stats(self) -> dict:
        return {
            "sink_fill": self.sink_fill,
            "sink_capacity": self.config.sink_size,
            "key_qbuf_len": self.key_qbuf_len,
            "key_qbuf_capacity": self.config.q_buffer_size,
            "val_local_len": self.val_local_len,
            "val_local_capacity": self.config.local_value_window,
            "val_qbuf_len": self.val_qbuf_len,
            **self.layout.memory_stats(),
        }
