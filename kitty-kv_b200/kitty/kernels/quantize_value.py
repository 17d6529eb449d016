"""Value page quantisation on B200 (per-token INT2).

Drop-in for ``kitty/kernels/quantize_value.py`` of the reference:

* :func:`quantize_value_page` - reference launcher signature
  (``quantize_value.py:197-202``); the scale / zero outputs may be the
  stride-2 views ``value_metadata[p, h, :, 0]`` / ``[..., 1]`` the pipeline passes;
* :func:`quantize_value_page_torch` - functional form (``:38-90``);
* :func:`dequantize_value_page_torch` - ``(code - zp) * scale`` in float32
  (``:97-133``), computed on the GPU with torch elementwise ops on the unpacked
  codes (a reference/debug helper; the decode kernel dequantises in registers);
* :func:`quantize_value_pages` - batched form writing into the pools.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib


def quantize_value_pages(value_src: torch.Tensor, src_offsets: torch.Tensor, src_strides: Tuple[int, int, int],
                         dst_pages: torch.Tensor, val_codes: torch.Tensor, val_meta: torch.Tensor,
                         num_heads: int, head_dim: int, group: int,
                         n_valid: Optional[torch.Tensor] = None) -> None:
    """Quantise ``len(dst_pages)`` x ``num_heads`` value page-heads into the pools
    ``val_codes (P,H,G,D/4)`` and ``val_meta (P,H,G,2)``.  Tokens at or beyond
    ``n_valid[j]`` read as zero (the reference pads a partial buffer with zeros,
    ``kitty/pipeline.py:238-243``)."""
    dev = _lib.require_cuda(value_src, src_offsets, dst_pages, val_codes, val_meta, n_valid)
    code = _lib.quant_dtype_code(value_src.dtype, val_meta.dtype)
    if src_offsets.dtype != torch.int64 or dst_pages.dtype != torch.int32:
        raise RuntimeError("src_offsets must be int64 and dst_pages int32")
    if n_valid is not None and (n_valid.dtype != torch.int32 or n_valid.numel() != dst_pages.numel()):
        raise RuntimeError("n_valid must be int32 with one entry per job")
    if not (val_codes.is_contiguous() and val_meta.is_contiguous()):
        raise RuntimeError("value pools must be contiguous")
    s_head, s_tok, s_ch = (int(x) for x in src_strides)
    a = _lib.ValueQuantArgs()
    a.value = value_src.data_ptr(); a.value_off = src_offsets.data_ptr()
    a.val_s_head, a.val_s_tok, a.val_s_ch = s_head, s_tok, s_ch
    a.n_valid = _lib.ptr(n_valid); a.dst_page = dst_pages.data_ptr()
    a.val_codes = val_codes.data_ptr()
    a.val_scale = val_meta.data_ptr(); a.val_zero = val_meta.data_ptr() + 2
    a.codes_s_page, a.codes_s_head = val_codes.stride(0), val_codes.stride(1)
    a.meta_s_page, a.meta_s_head, a.meta_s_tok = val_meta.stride(0), val_meta.stride(1), val_meta.stride(2)
    a.n_jobs, a.num_heads, a.head_dim, a.group = dst_pages.numel(), num_heads, head_dim, group
    a.dtype = code
    lib = _lib.load()
    _lib.check(lib.kitty_quantize_value_pages(a, _lib.stream_ptr(dev)), "kitty_quantize_value_pages")


def _launch_single(value: torch.Tensor, codes: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor) -> None:
    dev = _lib.require_cuda(value, codes, scale, zero)
    G, D = value.shape
    a = _lib.ValueQuantArgs()
    a.value = value.data_ptr(); a.value_off = _lib.zeros_const(dev, torch.int64).data_ptr()
    a.val_s_head, a.val_s_tok, a.val_s_ch = 0, value.stride(0), value.stride(1)
    a.n_valid = 0; a.dst_page = _lib.zeros_const(dev, torch.int32).data_ptr()
    a.val_codes = codes.data_ptr(); a.val_scale = scale.data_ptr(); a.val_zero = zero.data_ptr()
    a.meta_s_tok = scale.stride(0)
    a.n_jobs, a.num_heads, a.head_dim, a.group = 1, 1, D, G
    a.dtype = _lib.quant_dtype_code(value.dtype, scale.dtype)
    lib = _lib.load()
    _lib.check(lib.kitty_quantize_value_pages(a, _lib.stream_ptr(dev)), "kitty_quantize_value_pages")


def _validate(value):
    if value.dim() != 2:
        raise RuntimeError(f"value must be (G, D), got {tuple(value.shape)}")
    G, D = value.shape
    if D % 4 != 0:
        raise AssertionError("head_dim D must be divisible by 4 for packing")
    if value.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError(f"value must be float16 or bfloat16 (got {value.dtype})")
    return G, D


def quantize_value_page_torch(value: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Functional form: (packed (G,D/4) u8, scale (G,) f16, zero_point (G,) f16)."""
    G, D = _validate(value)
    dev = _lib.require_cuda(value)
    codes = torch.empty(G, D // 4, dtype=torch.uint8, device=dev)
    meta = torch.empty(2, G, dtype=torch.float16, device=dev)   # the reference returns fp16
    _launch_single(value, codes, meta[0], meta[1])
    return codes, meta[0], meta[1]


def quantize_value_page(value: torch.Tensor, out_packed: torch.Tensor, out_scale: torch.Tensor,
                        out_zero: torch.Tensor) -> None:
    """Quantise one value page into pre-allocated outputs (reference ``:197-227``)."""
    G, D = _validate(value)
    _lib.require_cuda(value, out_packed, out_scale, out_zero)
    if tuple(out_packed.shape) != (G, D // 4) or out_scale.numel() != G or out_zero.numel() != G:
        raise RuntimeError("out_packed must be (G, D/4); out_scale/out_zero must have G elements")
    same_stride = out_scale.dim() == 1 and out_zero.dim() == 1 and out_scale.stride(0) == out_zero.stride(0)
    if (out_packed.is_contiguous() and same_stride and out_scale.dtype == out_zero.dtype
            and (out_scale.dtype == value.dtype or out_scale.dtype == torch.float16)):
        _launch_single(value, out_packed, out_scale, out_zero)
        return
    codes, scale, zero = quantize_value_page_torch(value)
    out_packed.copy_(codes); out_scale.copy_(scale); out_zero.copy_(zero)


def dequantize_value_page_torch(packed: torch.Tensor, scale: torch.Tensor, zero_point: torch.Tensor) -> torch.Tensor:
    """(code - zp) * scale in float32, shape (G, D) (reference ``quantize_value.py:97-133``),
    by the CUDA value dequantiser (``kitty_dequantize_value_pages``, float32 output).
    ``scale`` / ``zero_point`` are (G,) float16 or bfloat16, any stride (the stride-2
    views of the value metadata pool included)."""
    dev = _lib.require_cuda(packed, scale, zero_point)
    if packed.dtype != torch.uint8 or packed.dim() != 2:
        raise RuntimeError("packed must be a (G, D/4) uint8 tensor")
    G, D4 = packed.shape
    if scale.numel() != G or zero_point.numel() != G or scale.dim() != 1 or zero_point.dim() != 1:
        raise RuntimeError(f"scale and zero_point must be ({G},) vectors")
    if scale.dtype != zero_point.dtype:
        raise RuntimeError("scale and zero_point must have the same dtype")
    if scale.stride(0) != zero_point.stride(0):
        scale, zero_point = scale.contiguous(), zero_point.contiguous()
    if not packed.is_contiguous():
        packed = packed.contiguous()
    out = torch.empty(G, D4 * 4, dtype=torch.float32, device=dev)
    a = _lib.ValueDequantArgs()
    a.val_codes = packed.data_ptr()
    a.val_scale, a.val_zero = scale.data_ptr(), zero_point.data_ptr()
    a.codes_s_page = a.codes_s_head = a.meta_s_page = a.meta_s_head = 0
    a.meta_s_tok = scale.stride(0)
    z32 = _lib.zeros_const(dev, torch.int32)
    a.src_page = z32.data_ptr(); a.head = z32.data_ptr()
    a.out, a.out_off = out.data_ptr(), _lib.zeros_const(dev, torch.int64).data_ptr()
    a.out_s_tok, a.out_s_ch = out.stride(0), out.stride(1)
    a.n_jobs, a.head_dim, a.group = 1, D4 * 4, G
    a.dtype = _lib.dequant_dtype_code(scale.dtype, torch.float32)
    _lib.check(_lib.load().kitty_dequantize_value_pages(a, _lib.stream_ptr(dev)), "kitty_dequantize_value_pages")
    return out
