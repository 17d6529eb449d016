"""CPU oracle for the Kitty quantized-KV hot path (numpy restatement).

TEST INFRASTRUCTURE ONLY.  This module is the checker that the CUDA kernels are
compared against.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py`` may import it; the ``kitty`` package never does,
and it must never be used as a fallback for the CUDA path.

Every function restates one function of the reference's PyTorch path
(bitxwolf/kitty-kv) with numpy, in the same float32 operation order, so that
integer outputs (packed 2-bit codes, high planes) are bit-exact and the fp16
metadata equals the reference's by value:

* ``quantize_key_page``    <- ``kitty/kernels/quantize_key.py:38-124``
* ``quantize_value_page``  <- ``kitty/kernels/quantize_value.py:38-90``
* ``dequantize_key_page``  <- ``kitty/kernels/dequantize_key.py:35-97``
* ``dequantize_value_page``<- ``kitty/kernels/quantize_value.py:97-133``
* ``paged_attention``      <- ``kitty/kernels/attention.py:46-189``
* ``boost_idx_from_scores``<- ``kitty/sensitivity.py:164-207``
* ``cache_regions`` / ``sequence_state`` <- ``kitty/pipeline.py:115-181`` (push_token's
  sink / Q-buffer / flush state machine, values aligned with their keys)

Parity of this restatement is pinned against golden vectors produced by the
reference itself (``tests/golden/make_golden.py`` imports the reference and
records its outputs); ``tests/test_oracle_golden.py`` checks the pin.

Float32 semantics reproduced from torch:

* ``clamp(min=1e-8)`` compares against float32(1e-8) and propagates NaN;
* ``torch.round`` is round-half-to-even (``np.rint``);
* division is IEEE float32 round-to-nearest;
* ``torch.maximum/minimum`` propagate NaN (``np.maximum/minimum`` do too);
* ``.to(float16)`` rounds to nearest even (``astype(np.float16)``);
* a bfloat16 cache (``dtype="bfloat16"``): inputs widen exactly (``.float()``),
  and the fp16 scale / zero-point the quantisers return are copied into bf16
  pool views (``kitty/kernels/quantize_key.py:261-269``), i.e. rounded to fp16
  and then to bf16 (nearest even, ``bf16_round``).  bf16 arrays are passed and
  returned here as float32 arrays holding bf16 values.
"""

from __future__ import annotations

import math
from typing import Iterable, List, Sequence, Tuple

import numpy as np

F32 = np.float32
_EPS_RANGE = F32(1e-8)


# ---------------------------------------------------------------------------
# 16-bit float types
# ---------------------------------------------------------------------------

def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bfloat16 (ties to even), returned as float32; NaN stays NaN."""
    x = np.ascontiguousarray(np.asarray(x, dtype=F32))
    b = x.view(np.uint32).astype(np.uint64)
    r = (((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(F32)
    return np.where(np.isnan(x), x, r).astype(F32)


def _h16(x, dtype: str) -> np.ndarray:
    """Exact float32 values of a 16-bit float input (fp16 arrays, or float32 arrays
    holding bf16 values)."""
    if dtype == "float16":
        return np.asarray(x, dtype=np.float16).astype(F32)
    if dtype == "bfloat16":
        return bf16_round(np.asarray(x, dtype=F32))
    raise ValueError(f"dtype must be float16 or bfloat16, got {dtype}")


def _meta(x: np.ndarray, dtype: str) -> np.ndarray:
    """A float32 scale / zero-point as stored in the cache: fp16, or fp16 then bf16."""
    h = np.asarray(x, dtype=F32).astype(np.float16)
    return h if dtype == "float16" else bf16_round(h.astype(F32))


# ---------------------------------------------------------------------------
# bit packing helpers (4 two-bit codes per byte, first element in bits 0-1)
# ---------------------------------------------------------------------------

def pack_2bit(codes: np.ndarray) -> np.ndarray:
    """Pack the last axis of ``codes`` (values 0..3) four per byte.

    Byte ``j`` holds elements ``4j, 4j+1, 4j+2, 4j+3`` at bit offsets
    0, 2, 4, 6 (``quantize_key.py:108-110``, ``quantize_value.py:84-86``).
    """
    c = (codes.astype(np.uint8) & 3).reshape(codes.shape[:-1] + (codes.shape[-1] // 4, 4))
    return (c[..., 0] | (c[..., 1] << 2) | (c[..., 2] << 4) | (c[..., 3] << 6)).astype(np.uint8)


def unpack_2bit(packed: np.ndarray) -> np.ndarray:
    """Inverse of :func:`pack_2bit` (``dequantize_key.py:70-74``)."""
    p = packed.astype(np.uint8)[..., None]
    shifts = np.array([0, 2, 4, 6], dtype=np.uint8)
    return ((p >> shifts) & 3).reshape(packed.shape[:-1] + (packed.shape[-1] * 4,))


def _clamp_range(r: np.ndarray) -> np.ndarray:
    # torch clamp(min=v): NaN stays NaN, values below v become v.
    return np.where(r < _EPS_RANGE, _EPS_RANGE, r).astype(F32)


# ---------------------------------------------------------------------------
# key quantisation (per channel, INT4 for boosted channels, INT2 otherwise)
# ---------------------------------------------------------------------------

def quantize_key_page(key: np.ndarray, boost_idx: np.ndarray, d_boost: int, sentinel: int, dtype: str = "float16",
                      meta_dtype: str = None) -> Tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
    """Restates ``quantize_key_page_torch`` (``quantize_key.py:38-124``).

    key: (D, G) float16, boost_idx: (D,) uint8.  Returns
    (low (D, G/4) u8, high (d_boost, G/4) u8, scale (D,) f16, zero (D,) f16)
    (bf16 values as float32 with ``dtype="bfloat16"``; ``meta_dtype="float16"`` gives
    the fp16 scale / zero-point the functional form returns for a bf16 input).
    """
    x = _h16(key, dtype)
    D, G = x.shape
    assert G % 4 == 0
    bidx = np.asarray(boost_idx).astype(np.int64)
    is_boosted = bidx < int(sentinel)                               # :73
    x_min = x.min(axis=1)                                           # :76
    x_max = x.max(axis=1)                                           # :77
    x_range = _clamp_range((x_max - x_min).astype(F32))             # :78
    max_q = np.where(is_boosted, F32(15.0), F32(3.0)).astype(F32)   # :81-82
    scale = (x_range / max_q).astype(F32)                           # :84
    zp = np.rint((-x_min / scale).astype(F32))                      # :86
    zp = np.minimum(np.maximum(zp, F32(0.0)), max_q).astype(F32)    # :87
    xq = (np.rint((x / scale[:, None]).astype(F32)) + zp[:, None]).astype(F32)   # :95
    xq = np.minimum(np.maximum(xq, F32(0.0)), max_q[:, None])       # :97-99
    codes = np.nan_to_num(xq, nan=0.0).astype(np.uint8)
    low = pack_2bit(codes & 3)                                      # :102,108-110
    high_codes = (codes >> 2) & 3                                   # :103
    high = np.zeros((d_boost, G // 4), dtype=np.uint8)              # :113
    packed_high = pack_2bit(high_codes)
    for c in np.nonzero(is_boosted)[0]:                             # :114-119
        r = int(bidx[c])
        if r < d_boost:
            high[r] |= packed_high[c]
    m = meta_dtype or dtype
    return low, high, _meta(scale, m), _meta(zp, m)


def dequantize_key_page(low: np.ndarray, high: np.ndarray, scale: np.ndarray,
                        zero: np.ndarray, boost_idx: np.ndarray, d_boost: int, dtype: str = "float16") -> np.ndarray:
    """Restates ``dequantize_key_page_torch`` (``dequantize_key.py:35-97``): (D, G) float32."""
    D, G4 = low.shape
    code = unpack_2bit(low).astype(np.int32)                        # :70-74
    bidx = np.asarray(boost_idx).astype(np.int64)
    hi = np.zeros_like(code)
    for c in range(D):                                              # :81-87
        if bidx[c] < d_boost:
            hi[c] = unpack_2bit(high[bidx[c]]).astype(np.int32)
    xq = (code | (hi << 2)).astype(F32)                             # :90
    s = _h16(scale, dtype)[:, None]
    z = _h16(zero, dtype)[:, None]
    return ((xq - z) * s).astype(F32)                               # :93-95


# ---------------------------------------------------------------------------
# value quantisation (per token INT2)
# ---------------------------------------------------------------------------

def quantize_value_page(value: np.ndarray, dtype: str = "float16",
                        meta_dtype: str = None) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Restates ``quantize_value_page_torch`` (``quantize_value.py:38-90``).

    value: (G, D) float16.  Returns (codes (G, D/4) u8, scale (G,) f16, zero (G,) f16).
    """
    v = _h16(value, dtype)
    v_min = v.min(axis=1)                                           # :62
    v_max = v.max(axis=1)                                           # :63
    v_range = _clamp_range((v_max - v_min).astype(F32))             # :64
    scale = (v_range / F32(3.0)).astype(F32)                        # :66
    zp = np.rint((-v_min / scale).astype(F32))                      # :68
    zp = np.minimum(np.maximum(zp, F32(0.0)), F32(3.0)).astype(F32)  # :69-72
    vq = (np.rint((v / scale[:, None]).astype(F32)) + zp[:, None]).astype(F32)   # :77
    vq = np.minimum(np.maximum(vq, F32(0.0)), F32(3.0))             # :78-81
    codes = np.nan_to_num(vq, nan=0.0).astype(np.uint8)
    m = meta_dtype or dtype
    return pack_2bit(codes), _meta(scale, m), _meta(zp, m)


def dequantize_value_page(packed: np.ndarray, scale: np.ndarray, zero: np.ndarray,
                          dtype: str = "float16") -> np.ndarray:
    """Restates ``dequantize_value_page_torch`` (``quantize_value.py:97-133``): (G, D) float32."""
    code = unpack_2bit(packed).astype(F32)
    s = _h16(scale, dtype)[:, None]
    z = _h16(zero, dtype)[:, None]
    return ((code - z) * s).astype(F32)


# ---------------------------------------------------------------------------
# vectorised batch forms (same arithmetic, many page-heads at once)
# ---------------------------------------------------------------------------

def quantize_key_pages(keys: np.ndarray, boost_idx: np.ndarray, d_boost: int,
                       sentinel: int, dtype: str = "float16") -> Tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
    """Batch of :func:`quantize_key_page` over leading axes.

    keys: (..., D, G) float16; boost_idx broadcastable to (..., D).
    Identical arithmetic to the single-page form (checked in the tests).
    """
    x = _h16(keys, dtype)
    lead = x.shape[:-2]
    D, G = x.shape[-2:]
    bidx = np.broadcast_to(np.asarray(boost_idx).astype(np.int64), lead + (D,))
    is_boosted = bidx < int(sentinel)
    x_min = x.min(axis=-1)
    x_max = x.max(axis=-1)
    x_range = _clamp_range((x_max - x_min).astype(F32))
    max_q = np.where(is_boosted, F32(15.0), F32(3.0)).astype(F32)
    scale = (x_range / max_q).astype(F32)
    zp = np.rint((-x_min / scale).astype(F32))
    zp = np.minimum(np.maximum(zp, F32(0.0)), max_q).astype(F32)
    xq = (np.rint((x / scale[..., None]).astype(F32)) + zp[..., None]).astype(F32)
    xq = np.minimum(np.maximum(xq, F32(0.0)), max_q[..., None])
    codes = np.nan_to_num(xq, nan=0.0).astype(np.uint8)
    low = pack_2bit(codes & 3)
    packed_high = pack_2bit((codes >> 2) & 3)                      # (..., D, G/4)
    high = np.zeros(lead + (d_boost, G // 4), dtype=np.uint8)
    writes = is_boosted & (bidx < d_boost)
    for c in range(D):
        sel = writes[..., c]
        if not sel.any():
            continue
        rows = bidx[..., c]
        # OR the channel's high plane into row boost_idx[c] where selected
        idx = np.nonzero(sel)
        high[idx + (rows[idx],)] |= packed_high[idx + (c,)]
    return low, high, _meta(scale, dtype), _meta(zp, dtype)


def quantize_value_pages(values: np.ndarray, dtype: str = "float16") -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Batch of :func:`quantize_value_page`; values: (..., G, D) float16."""
    v = _h16(values, dtype)
    v_min = v.min(axis=-1)
    v_max = v.max(axis=-1)
    v_range = _clamp_range((v_max - v_min).astype(F32))
    scale = (v_range / F32(3.0)).astype(F32)
    zp = np.rint((-v_min / scale).astype(F32))
    zp = np.minimum(np.maximum(zp, F32(0.0)), F32(3.0)).astype(F32)
    vq = (np.rint((v / scale[..., None]).astype(F32)) + zp[..., None]).astype(F32)
    vq = np.minimum(np.maximum(vq, F32(0.0)), F32(3.0))
    codes = np.nan_to_num(vq, nan=0.0).astype(np.uint8)
    return pack_2bit(codes), _meta(scale, dtype), _meta(zp, dtype)


def dequantize_key_pages(low: np.ndarray, high: np.ndarray, scale: np.ndarray,
                         zero: np.ndarray, boost_idx: np.ndarray, d_boost: int, dtype: str = "float16") -> np.ndarray:
    """Batch of :func:`dequantize_key_page`; low (..., D, G/4) -> (..., D, G) float32."""
    code = unpack_2bit(low).astype(np.int32)
    lead = low.shape[:-2]
    D = low.shape[-2]
    bidx = np.broadcast_to(np.asarray(boost_idx).astype(np.int64), lead + (D,))
    hi = np.zeros_like(code)
    if d_boost > 0:
        hi_all = unpack_2bit(high).astype(np.int32)                # (..., K, G)
        rows = np.where(bidx < d_boost, bidx, 0)
        gathered = np.take_along_axis(hi_all, rows[..., None], axis=-2)
        hi = np.where((bidx < d_boost)[..., None], gathered, 0)
    xq = (code | (hi << 2)).astype(F32)
    s = _h16(scale, dtype)[..., None]
    z = _h16(zero, dtype)[..., None]
    return ((xq - z) * s).astype(F32)


def dequantize_value_pages(packed: np.ndarray, scale: np.ndarray, zero: np.ndarray,
                           dtype: str = "float16") -> np.ndarray:
    """Batch of :func:`dequantize_value_page`; (..., G, D/4) -> (..., G, D) float32."""
    code = unpack_2bit(packed).astype(F32)
    s = _h16(scale, dtype)[..., None]
    z = _h16(zero, dtype)[..., None]
    return ((code - z) * s).astype(F32)


# ---------------------------------------------------------------------------
# paged decode attention
# ---------------------------------------------------------------------------

def paged_attention(q: np.ndarray, page_list: Sequence[int], key_baseline: np.ndarray,
                    key_boost: np.ndarray, key_meta: np.ndarray, value_pool: np.ndarray,
                    value_meta: np.ndarray, boost_idx: np.ndarray, d_boost: int,
                    sink_k: np.ndarray, sink_v: np.ndarray, qbuf_k: np.ndarray,
                    qbuf_v: np.ndarray, num_q_heads: int, num_kv_heads: int,
                    head_dim: int, dtype: str = "float16") -> np.ndarray:
    """Restates ``paged_attention_reference`` (``kitty/kernels/attention.py:46-189``).

    Per KV head the keys are [sinks ; dequantised pages in ``page_list`` order ;
    qbuf_k] and the values [sinks ; dequantised value pages ; qbuf_v]
    (``:136-168``); query head ``qh`` reads KV head ``qh // (Hq/H)`` (``:93,177``);
    scores are ``(q . k) / sqrt(D)`` in float32 followed by a softmax and a
    weighted sum (``:172-187``); the result is cast to float16 (``:189``).
    Returns (Hq, D) float16.
    """
    H, D = num_kv_heads, head_dim
    q_per_kv = num_q_heads // num_kv_heads
    pages = [int(p) for p in page_list]
    keys_h: List[np.ndarray] = []
    vals_h: List[np.ndarray] = []
    for h in range(H):
        kp, vp = [], []
        if sink_k.shape[1] > 0:
            kp.append(_h16(sink_k[h], dtype))
            vp.append(_h16(sink_v[h], dtype))
        if pages:
            pidx = np.asarray(pages, dtype=np.int64)
            kdq = dequantize_key_pages(key_baseline[pidx, h], key_boost[pidx, h],
                                       key_meta[pidx, h, 0], key_meta[pidx, h, 1],
                                       boost_idx[h], d_boost, dtype)   # (n, D, G)
            kp.append(np.swapaxes(kdq, 1, 2).reshape(-1, D))
            vdq = dequantize_value_pages(value_pool[pidx, h], value_meta[pidx, h, :, 0],
                                         value_meta[pidx, h, :, 1], dtype)   # (n, G, D)
            vp.append(vdq.reshape(-1, D))
        if qbuf_k.shape[1] > 0:                                        # :163
            kp.append(_h16(qbuf_k[h], dtype))
            vp.append(_h16(qbuf_v[h], dtype))
        keys_h.append(np.concatenate(kp, axis=0) if kp else np.zeros((0, D), F32))
        vals_h.append(np.concatenate(vp, axis=0) if vp else np.zeros((0, D), F32))
    scale_factor = F32(1.0 / math.sqrt(D))
    qf = _h16(q, dtype)
    out = np.zeros((num_q_heads, D), dtype=F32)
    for qh in range(num_q_heads):
        K = keys_h[qh // q_per_kv]
        V = vals_h[qh // q_per_kv]
        if K.shape[0] == 0:
            continue
        if K.shape[0] != V.shape[0]:
            raise ValueError("key and value token counts differ (reference broadcast error)")
        scores = (K @ qf[qh]).astype(F32) * scale_factor
        m = scores.max()
        e = np.exp((scores - m).astype(F32)).astype(F32)
        w = (e / e.sum(dtype=F32)).astype(F32)
        out[qh] = (w[:, None] * V).sum(axis=0, dtype=F32)
    return out.astype(np.float16)


def paged_attention_batched(q: np.ndarray, block_table: np.ndarray, num_pages: np.ndarray,
                            pools: Tuple[np.ndarray, ...], boost_idx: np.ndarray, d_boost: int,
                            sink_k: np.ndarray, sink_v: np.ndarray, sink_len: np.ndarray,
                            tail_k: np.ndarray, tail_v: np.ndarray, tail_len: np.ndarray,
                            dtype: str = "float16") -> np.ndarray:
    """Per-sequence application of :func:`paged_attention` (the reference is batch 1,
    ``kitty/attention.py:100``; a batch is B independent calls).

    q (B, Hq, D); block_table (B, maxP) int; sink_k/v (B, H, S, D); tail_k/v (B, H, Q, D).
    """
    key_low, key_high, key_meta, val_codes, val_meta = pools
    B, Hq, D = q.shape
    H = sink_k.shape[1]
    out = np.zeros((B, Hq, D), dtype=np.float16)
    for b in range(B):
        n = int(num_pages[b]); s = int(sink_len[b]); t = int(tail_len[b])
        out[b] = paged_attention(q[b], block_table[b, :n], key_low, key_high, key_meta,
                                 val_codes, val_meta, boost_idx, d_boost,
                                 sink_k[b, :, :s], sink_v[b, :, :s], tail_k[b, :, :t],
                                 tail_v[b, :, :t], Hq, H, D, dtype)
    return out


# ---------------------------------------------------------------------------
# per-sequence cache state after a token history (push_token state machine)
# ---------------------------------------------------------------------------

def cache_regions(n_tokens: int, sink_size: int, group: int) -> Tuple[int, int, int]:
    """(sink_len, num_pages, tail_len) after ``n_tokens`` pushes: the first S tokens
    fill the sinks (``kitty/pipeline.py:138-145``), every later token goes to the
    Key Q-buffer (``:148``) and a buffer reaching G tokens becomes one page and is
    emptied (``:171-181``)."""
    s = min(n_tokens, sink_size)
    rest = n_tokens - s
    return s, rest // group, rest % group


def sequence_state(keys: np.ndarray, values: np.ndarray, sink_size: int, group: int,
                   boost_idx: np.ndarray, d_boost: int, sentinel: int, dtype: str = "float16") -> dict:
    """Expected cache contents of one sequence whose tokens are keys / values (T, H, D)
    float16: fp16 sinks and tail, and for each page the quantised key planes (of the
    (H, D, G) block of its G keys) and value planes (of its G values, the values of
    the same tokens - the pipeline's aligned-values mode)."""
    if dtype == "float16":
        keys = np.asarray(keys, np.float16)
        values = np.asarray(values, np.float16)
    else:
        keys, values = _h16(keys, dtype), _h16(values, dtype)
    s, n, t = cache_regions(keys.shape[0], sink_size, group)
    out = {"sink_k": keys[:s].transpose(1, 0, 2), "sink_v": values[:s].transpose(1, 0, 2),
           "tail_k": keys[s + n * group:].transpose(1, 0, 2), "tail_v": values[s + n * group:].transpose(1, 0, 2),
           "pages": []}
    for j in range(n):
        kb = keys[s + j * group: s + (j + 1) * group]          # (G, H, D)
        vb = values[s + j * group: s + (j + 1) * group]
        low, high, scale, zero = quantize_key_pages(kb.transpose(1, 2, 0), boost_idx, d_boost, sentinel, dtype)
        codes, vscale, vzero = quantize_value_pages(vb.transpose(1, 0, 2), dtype)
        out["pages"].append({"key_low": low, "key_high": high, "key_scale": scale, "key_zero": zero,
                             "val_codes": codes, "val_scale": vscale, "val_zero": vzero})
    return out


# ---------------------------------------------------------------------------
# sensitivity: boost index from channel scores
# ---------------------------------------------------------------------------

def boost_idx_from_scores(scores: np.ndarray, d_boost: int, sentinel: int) -> np.ndarray:
    """Restates ``KittySensitivityProfiler.compute`` (``kitty/sensitivity.py:164-207``):
    the channel with the r-th largest score gets index r (r < K), all others the sentinel.
    scores: (..., D) float32 -> (..., D) uint8."""
    s = np.asarray(scores, dtype=F32)
    order = np.argsort(-s, axis=-1, kind="stable")
    out = np.full(s.shape, sentinel, dtype=np.uint8)
    for rank in range(d_boost):
        np.put_along_axis(out, order[..., rank:rank + 1], np.uint8(rank), axis=-1)
    return out
