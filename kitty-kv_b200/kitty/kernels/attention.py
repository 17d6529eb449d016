"""Fused paged GQA decode attention on B200.

Drop-in for ``kitty/kernels/attention.py`` of the reference:

* :func:`paged_attention` / :func:`paged_attention_reference` - reference
  signature (``attention.py:292-309`` and ``:46-63``), batch 1, returning
  (Hq, D) float16.  Both run the CUDA kernel (the reference's "reference"
  version is its CPU path; here there is only the GPU path);
* :func:`paged_attention_batched` - the batched form the reference lacks
  (``kitty/attention.py:100`` asserts batch 1): per-sequence block tables,
  page counts, sink and tail lengths, one launch for the whole batch.

Semantics (``attention.py:136-189``): for query head qh and KV head
h = qh // (Hq/H), keys are [sinks ; pages in block-table order ; key tail] and
values [sinks ; value pages ; value tail]; out = softmax(q.k / sqrt(D)) . v,
accumulated in float32 and returned as float16 (also for a bfloat16 cache, as the
reference's ``.to(torch.float16)`` at ``attention.py:189`` does).
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple, Union

import torch

from . import _lib

_workspaces: Dict[Tuple[torch.device, int], torch.Tensor] = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """A per-(device, stream) scratch buffer grown on demand (calls on one stream
    are ordered, so they may share it)."""
    key = (device, torch.cuda.current_stream(device).cuda_stream)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def _strides4(t: Optional[torch.Tensor]) -> Tuple[int, int, int]:
    if t is None:
        return 0, 0, 0
    if t.stride(-1) != 1:
        raise RuntimeError("fp16 region tensors need unit channel stride")
    return t.stride(0), t.stride(1), t.stride(2)


def _as_len(x, name, B, dev) -> Tuple[Optional[torch.Tensor], int]:
    if x is None:
        return None, 0
    if isinstance(x, int):
        if x < 0:
            raise RuntimeError(f"{name} must be non-negative")
        return None, x
    if x.dtype != torch.int32 or x.numel() != B or x.device != dev:
        raise RuntimeError(f"{name} must be an int32 tensor with one entry per sequence on {dev}")
    return x, 0


def paged_attention_batched(q: torch.Tensor, block_table: torch.Tensor, num_pages: torch.Tensor,
                            key_baseline: torch.Tensor, key_boost: torch.Tensor, key_meta: torch.Tensor,
                            value_pool: torch.Tensor, value_meta: torch.Tensor, boost_idx: torch.Tensor,
                            D_boost: int, sink_k: Optional[torch.Tensor] = None,
                            sink_v: Optional[torch.Tensor] = None,
                            sink_len: Union[int, torch.Tensor, None] = None,
                            tail_k: Optional[torch.Tensor] = None, tail_v: Optional[torch.Tensor] = None,
                            tail_len: Union[int, torch.Tensor, None] = None,
                            out: Optional[torch.Tensor] = None, num_splits: int = 0,
                            sm_scale: Optional[float] = None,
                            max_pages_per_seq: Optional[int] = None,
                            seq_map: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Batched decode: q (B, Hq, D) fp16 -> (B, Hq, D) fp16.

    block_table (B, maxP) int32 physical pages (row b uses its first
    num_pages[b] entries); pools as in the layout manager; sink_k/v and
    tail_k/v (B, H, S|Q, D) fp16 with per-sequence lengths ``sink_len`` /
    ``tail_len`` (int or (B,) int32 tensor).  Key and value tails share one length.
    With ``seq_map`` ((B,) int32), row b of q / out reads row seq_map[b] of the
    block table, page counts, lengths and fp16 regions, which then have one row
    per cache slot (any number of rows) instead of one per batch row.
    """
    dev = _lib.require_cuda(q, block_table, num_pages, key_baseline, key_boost, key_meta, value_pool,
                            value_meta, boost_idx, sink_k, sink_v, tail_k, tail_v)
    if q.dim() != 3:
        raise RuntimeError("q must be (B, Hq, D)")
    B, Hq, D = q.shape
    P, H, D_pool, G4 = key_baseline.shape
    G = G4 * 4
    if D_pool != D:
        raise RuntimeError(f"head_dim mismatch: q has {D}, pools have {D_pool}")
    if key_boost.shape[2] != D_boost:
        raise RuntimeError(f"key_boost has {key_boost.shape[2]} rows, D_boost is {D_boost}")
    if Hq % H != 0:
        raise RuntimeError("num_q_heads must be a multiple of num_kv_heads")
    for t, n in ((key_baseline, "key_baseline"), (key_boost, "key_boost"), (key_meta, "key_meta"),
                 (value_pool, "value_pool"), (value_meta, "value_meta")):
        if not t.is_contiguous():
            raise RuntimeError(f"{n} must be contiguous")
    if key_meta.dtype != value_meta.dtype or key_meta.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("metadata pools must both be float16 or both bfloat16")
    h16 = key_meta.dtype      # the cache's 16-bit type: q, sinks and tails are read in it
    if tuple(value_pool.shape) != (P, H, G, D // 4) or tuple(key_meta.shape) != (P, H, 2, D):
        raise RuntimeError("pool shapes are inconsistent")
    if boost_idx.dtype != torch.uint8 or tuple(boost_idx.shape) != (H, D) or boost_idx.stride(1) != 1:
        raise RuntimeError("boost_idx must be (H, D) uint8 with unit channel stride")
    rows = B
    if seq_map is not None:
        if seq_map.dtype != torch.int32 or seq_map.numel() != B or seq_map.device != dev:
            raise RuntimeError("seq_map must be a (B,) int32 tensor on the pools' device")
        if not seq_map.is_contiguous():
            seq_map = seq_map.contiguous()
        rows = block_table.shape[0]
    if block_table.dtype != torch.int32 or block_table.dim() != 2 or block_table.shape[0] != rows:
        raise RuntimeError("block_table must be (B, maxP) int32 (one row per cache slot with seq_map)")
    if block_table.stride(1) != 1:
        raise RuntimeError("block_table rows need unit stride")
    if num_pages.dtype != torch.int32 or num_pages.numel() != rows:
        raise RuntimeError("num_pages must be (B,) int32 (one entry per cache slot with seq_map)")
    if q.dtype != h16:
        q = q.to(h16)
    if q.stride(-1) != 1:
        q = q.contiguous()
    for t, n in ((sink_k, "sink_k"), (sink_v, "sink_v"), (tail_k, "tail_k"), (tail_v, "tail_v")):
        if t is not None and (t.dtype != h16 or t.dim() != 4 or t.shape[1] != H or t.shape[3] != D):
            raise RuntimeError(f"{n} must be (B, H, T, D) {h16} (the metadata pools' dtype)")
    sink_t, sink_all = _as_len(sink_len, "sink_len", rows, dev)
    tail_t, tail_all = _as_len(tail_len, "tail_len", rows, dev)
    if sink_t is None and sink_all > 0 and (sink_k is None or sink_all > min(sink_k.shape[2], sink_v.shape[2])):
        raise RuntimeError("sink_len exceeds the sink tensors")
    if tail_t is None and tail_all > 0 and (tail_k is None or tail_all > min(tail_k.shape[2], tail_v.shape[2])):
        raise RuntimeError("tail_len exceeds the tail tensors")
    if out is None:
        out = torch.empty(B, Hq, D, dtype=torch.float16, device=dev)
    elif out.dtype != torch.float16 or tuple(out.shape) != (B, Hq, D) or out.stride(-1) != 1:
        raise RuntimeError("out must be (B, Hq, D) float16 with unit channel stride")
    maxp = block_table.shape[1] if max_pages_per_seq is None else int(max_pages_per_seq)

    a = _lib.DecodeArgs()
    a.batch, a.num_q_heads, a.num_kv_heads, a.head_dim, a.group, a.d_boost = B, Hq, H, D, G, int(D_boost)
    a.sm_scale = (1.0 / math.sqrt(D)) if sm_scale is None else float(sm_scale)
    a.q, a.q_s_seq, a.q_s_head = q.data_ptr(), q.stride(0), q.stride(1)
    a.out, a.out_s_seq, a.out_s_head = out.data_ptr(), out.stride(0), out.stride(1)
    a.block_table, a.bt_s_seq = block_table.data_ptr(), block_table.stride(0)
    a.num_pages, a.pool_pages = num_pages.data_ptr(), P
    a.key_low, a.key_high, a.key_meta = key_baseline.data_ptr(), key_boost.data_ptr(), key_meta.data_ptr()
    a.val_codes, a.val_meta = value_pool.data_ptr(), value_meta.data_ptr()
    a.boost_idx, a.bidx_s_head = boost_idx.data_ptr(), boost_idx.stride(0)
    a.sink_k = _lib.ptr(sink_k); a.sk_s_seq, a.sk_s_head, a.sk_s_tok = _strides4(sink_k)
    a.sink_v = _lib.ptr(sink_v); a.sv_s_seq, a.sv_s_head, a.sv_s_tok = _strides4(sink_v)
    a.sink_len, a.sink_len_all = _lib.ptr(sink_t), sink_all
    a.tail_k = _lib.ptr(tail_k); a.tk_s_seq, a.tk_s_head, a.tk_s_tok = _strides4(tail_k)
    a.tail_v = _lib.ptr(tail_v); a.tv_s_seq, a.tv_s_head, a.tv_s_tok = _strides4(tail_v)
    a.tail_len, a.tail_len_all = _lib.ptr(tail_t), tail_all
    a.max_pages_per_seq, a.num_splits = maxp, int(num_splits)
    a.seq_map = _lib.ptr(seq_map)
    a.dtype = _lib.dtype_code(h16)
    lib = _lib.load()
    nbytes = _lib.c_size(0)
    _lib.check(lib.kitty_paged_decode_workspace_size(a, nbytes, None), "kitty_paged_decode_workspace_size")
    if nbytes.value:
        ws = _workspace(dev, nbytes.value)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(lib.kitty_paged_decode(a, _lib.stream_ptr(dev)), "kitty_paged_decode")
    return out


_page_tables: Dict[torch.device, torch.Tensor] = {}


def _device_page_list(page_list: Sequence[int], device: torch.device, pool_pages: int) -> torch.Tensor:
    pages = [int(p) for p in page_list]
    for p in pages:
        if p < 0 or p >= pool_pages:
            raise IndexError(f"page index {p} out of range for a pool of {pool_pages} pages")
    host = torch.tensor(pages if pages else [0], dtype=torch.int32).pin_memory()
    return host.to(device, non_blocking=True).view(1, -1)


def paged_attention(q: torch.Tensor, page_list: List[int], key_baseline: torch.Tensor,
                    key_boost: torch.Tensor, key_meta: torch.Tensor, value_pool: torch.Tensor,
                    value_meta: torch.Tensor, boost_idx: torch.Tensor, D_boost: int,
                    sink_k: torch.Tensor, sink_v: torch.Tensor, qbuf_k: torch.Tensor,
                    qbuf_v: torch.Tensor, num_q_heads: int, num_kv_heads: int,
                    head_dim: int) -> torch.Tensor:
    """Decode attention for one sequence, reference signature; returns (Hq, D) float16."""
    dev = _lib.require_cuda(q, key_baseline)
    if q.shape != (num_q_heads, head_dim):
        raise RuntimeError(f"q must be ({num_q_heads}, {head_dim})")
    if key_baseline.shape[1] != num_kv_heads or key_baseline.shape[2] != head_dim:
        raise RuntimeError("pool shape does not match num_kv_heads / head_dim")
    if qbuf_k.shape[1] != qbuf_v.shape[1]:
        raise RuntimeError(
            f"key tail has {qbuf_k.shape[1]} tokens but value tail has {qbuf_v.shape[1]}; keys and "
            "values must cover the same tokens (the reference fails with a broadcast error here)")
    if sink_k.shape[1] != sink_v.shape[1]:
        raise RuntimeError("sink_k and sink_v lengths differ")
    bt = _device_page_list(page_list, dev, key_baseline.shape[0])
    n = len(page_list)
    num_pages = torch.full((1,), n, dtype=torch.int32, device=dev) if n else _lib.zeros_const(dev, torch.int32)
    s, t = sink_k.shape[1], qbuf_k.shape[1]
    out = paged_attention_batched(
        q.unsqueeze(0), bt, num_pages, key_baseline, key_boost, key_meta, value_pool, value_meta,
        boost_idx, D_boost,
        sink_k=sink_k.unsqueeze(0) if s else None, sink_v=sink_v.unsqueeze(0) if s else None, sink_len=s,
        tail_k=qbuf_k.unsqueeze(0) if t else None, tail_v=qbuf_v.unsqueeze(0) if t else None, tail_len=t,
        max_pages_per_seq=n)
    return out[0]


def paged_attention_reference(*args, **kwargs) -> torch.Tensor:
    """Same as :func:`paged_attention` (the reference's CPU path name; GPU here)."""
    return paged_attention(*args, **kwargs)
