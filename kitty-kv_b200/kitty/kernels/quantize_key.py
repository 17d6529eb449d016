"""Key page quantisation on B200 (per-channel INT2/INT4, dense-sparse layout).

Drop-in for ``kitty/kernels/quantize_key.py`` of the reference:

* :func:`quantize_key_page` - same signature as the reference launcher
  (``quantize_key.py:217-226``): quantises one (D, G) key block into
  caller-provided output views;
* :func:`quantize_key_page_torch` - same signature and return value as the
  reference's functional form (``quantize_key.py:38-43``), computed by the CUDA
  kernel (CUDA tensors only; there is no CPU implementation here);
* :func:`quantize_key_pages` - batched form over (job, head) page-heads writing
  straight into the layout manager's pools (used by the pipeline flush and the
  bulk prefill path).

The CUDA kernel reproduces the reference's float32 arithmetic exactly, so the
packed planes are bit-identical and scale / zero-point equal by value.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib


def _check_h16(t: torch.Tensor, name: str) -> int:
    """KITTY_DTYPE_* of a float16 / bfloat16 tensor (other dtypes raise)."""
    if t.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError(f"{name} must be float16 or bfloat16 (got {t.dtype})")
    return _lib.dtype_code(t.dtype)


def quantize_key_pages(key_src: torch.Tensor, src_offsets: torch.Tensor, src_strides: Tuple[int, int, int],
                       boost_idx: torch.Tensor, d_boost: int, sentinel: int, dst_pages: torch.Tensor,
                       key_low: torch.Tensor, key_high: torch.Tensor, key_meta: torch.Tensor,
                       num_heads: int, head_dim: int, group: int) -> None:
    """Quantise ``len(dst_pages)`` x ``num_heads`` page-heads into the pools.

    Job j, head h reads token t, channel c at
    ``key_src.flatten()[src_offsets[j] + h*s_head + t*s_tok + c*s_ch]`` where
    ``(s_head, s_tok, s_ch) = src_strides`` (elements), and writes page-head
    ``(dst_pages[j], h)`` of the pools ``key_low (P,H,D,G/4)``,
    ``key_high (P,H,K,G/4)``, ``key_meta (P,H,2,D)``.
    """
    dev = _lib.require_cuda(key_src, src_offsets, boost_idx, dst_pages, key_low, key_high, key_meta)
    _check_h16(key_src, "key")
    _check_h16(key_meta, "key_meta")
    code = _lib.quant_dtype_code(key_src.dtype, key_meta.dtype)
    if src_offsets.dtype != torch.int64 or dst_pages.dtype != torch.int32:
        raise RuntimeError("src_offsets must be int64 and dst_pages int32")
    if boost_idx.dtype != torch.uint8 or boost_idx.dim() != 2 or boost_idx.stride(1) != 1:
        raise RuntimeError("boost_idx must be a (H, D) uint8 tensor with unit channel stride")
    for t, name in ((key_low, "key_low"), (key_high, "key_high"), (key_meta, "key_meta")):
        if not t.is_contiguous():
            raise RuntimeError(f"{name} pool must be contiguous")
    n = dst_pages.numel()
    if src_offsets.numel() != n:
        raise RuntimeError("src_offsets and dst_pages must have one entry per job")
    s_head, s_tok, s_ch = (int(x) for x in src_strides)
    a = _lib.KeyQuantArgs()
    a.key = key_src.data_ptr(); a.key_off = src_offsets.data_ptr()
    a.key_s_head, a.key_s_tok, a.key_s_ch = s_head, s_tok, s_ch
    a.boost_idx = boost_idx.data_ptr(); a.bidx_s_head = boost_idx.stride(0)
    a.dst_page = dst_pages.data_ptr()
    a.key_low = key_low.data_ptr(); a.key_high = key_high.data_ptr()
    a.key_scale = key_meta.data_ptr(); a.key_zero = key_meta.data_ptr() + 2 * head_dim
    a.low_s_page, a.low_s_head = key_low.stride(0), key_low.stride(1)
    a.high_s_page, a.high_s_head = key_high.stride(0), key_high.stride(1)
    a.meta_s_page, a.meta_s_head = key_meta.stride(0), key_meta.stride(1)
    a.n_jobs, a.num_heads, a.head_dim, a.group = n, num_heads, head_dim, group
    a.d_boost, a.sentinel = int(d_boost), int(sentinel)
    a.dtype = code
    lib = _lib.load()
    _lib.check(lib.kitty_quantize_key_pages(a, _lib.stream_ptr(dev)), "kitty_quantize_key_pages")


def _launch_single(key: torch.Tensor, boost_idx: torch.Tensor, d_boost: int, sentinel: int,
                   low: torch.Tensor, high: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor) -> None:
    """One (D, G) block into contiguous outputs (low (D,G/4), high (K,G/4), scale (D,), zero (D,))."""
    dev = _lib.require_cuda(key, boost_idx, low, high, scale, zero)
    D, G = key.shape
    a = _lib.KeyQuantArgs()
    a.key = key.data_ptr(); a.key_off = _lib.zeros_const(dev, torch.int64).data_ptr()
    a.key_s_head, a.key_s_tok, a.key_s_ch = 0, key.stride(1), key.stride(0)
    a.boost_idx = boost_idx.data_ptr(); a.bidx_s_head = 0
    a.dst_page = _lib.zeros_const(dev, torch.int32).data_ptr()
    a.key_low = low.data_ptr(); a.key_high = high.data_ptr() if high.numel() else low.data_ptr()
    a.key_scale = scale.data_ptr(); a.key_zero = zero.data_ptr()
    a.n_jobs, a.num_heads, a.head_dim, a.group = 1, 1, D, G
    a.d_boost, a.sentinel = int(d_boost), int(sentinel)
    a.dtype = _lib.quant_dtype_code(key.dtype, scale.dtype)
    lib = _lib.load()
    _lib.check(lib.kitty_quantize_key_pages(a, _lib.stream_ptr(dev)), "kitty_quantize_key_pages")


def _validate_single(key, boost_idx, D_boost):
    if key.dim() != 2:
        raise RuntimeError(f"key must be (D, G), got shape {tuple(key.shape)}")
    D, G = key.shape
    if G % 4 != 0:
        raise AssertionError("G must be divisible by 4 for uint8 packing")
    _check_h16(key, "key")
    if boost_idx.shape != (D,) or boost_idx.dtype != torch.uint8:
        raise RuntimeError("boost_idx must be a (D,) uint8 tensor")
    if boost_idx.stride(0) != 1:
        boost_idx = boost_idx.contiguous()
    return D, G, boost_idx


def quantize_key_page_torch(key: torch.Tensor, boost_idx: torch.Tensor, D_boost: int,
                            sentinel: int) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Functional form: returns (tensor_2bits (D,G/4) u8, tensor_high_2bits (K,G/4) u8,
    scale (D,) f16, zero_point (D,) f16) - reference ``quantize_key.py:38-124``."""
    D, G, boost_idx = _validate_single(key, boost_idx, D_boost)
    dev = _lib.require_cuda(key, boost_idx)
    low = torch.empty(D, G // 4, dtype=torch.uint8, device=dev)
    high = torch.empty(D_boost, G // 4, dtype=torch.uint8, device=dev)
    meta = torch.empty(2, D, dtype=torch.float16, device=dev)   # the reference returns fp16
    _launch_single(key, boost_idx, D_boost, sentinel, low, high, meta[0], meta[1])
    return low, high, meta[0], meta[1]


def quantize_key_page(key: torch.Tensor, boost_idx: torch.Tensor, D_boost: int, sentinel: int,
                      out_baseline: torch.Tensor, out_boost: torch.Tensor, out_scale: torch.Tensor,
                      out_zero: torch.Tensor) -> None:
    """Quantise one key page into pre-allocated outputs (views into the pool).

    Same signature as the reference launcher (``quantize_key.py:217-226``).
    Contiguous outputs are written in place by the kernel; any other view is
    filled through a temporary and ``copy_``.
    """
    D, G, boost_idx = _validate_single(key, boost_idx, D_boost)
    _lib.require_cuda(key, boost_idx, out_baseline, out_boost, out_scale, out_zero)
    if tuple(out_baseline.shape) != (D, G // 4) or tuple(out_boost.shape) != (D_boost, G // 4):
        raise RuntimeError("out_baseline must be (D, G/4) and out_boost (D_boost, G/4)")
    if out_scale.numel() != D or out_zero.numel() != D:
        raise RuntimeError("out_scale / out_zero must have D elements")
    direct = (out_baseline.is_contiguous() and out_boost.is_contiguous() and out_scale.is_contiguous()
              and out_zero.is_contiguous() and out_scale.dtype == out_zero.dtype
              and out_scale.dtype in (torch.float16, torch.bfloat16)
              and (out_scale.dtype == key.dtype or out_scale.dtype == torch.float16))
    if direct:
        _launch_single(key, boost_idx, D_boost, sentinel, out_baseline, out_boost, out_scale, out_zero)
        return
    low, high, scale, zero = quantize_key_page_torch(key, boost_idx, D_boost, sentinel)
    out_baseline.copy_(low); out_boost.copy_(high); out_scale.copy_(scale); out_zero.copy_(zero)
