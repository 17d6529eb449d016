"""Key page dequantisation on B200.

Drop-in for ``kitty/kernels/dequantize_key.py`` of the reference: code =
low | (high << 2) for channels whose boost index is below D_boost, value =
(code - zp) * scale in float32 (``dequantize_key.py:35-97``).  The decode
kernel never materialises dequantised keys; this is the standalone form the
reference exposes (and benchmarks).
"""

from __future__ import annotations

import torch

from . import _lib


def _launch(tensor_2bits, tensor_high_2bits, scale, zero_point, boost_idx, D_boost, out) -> None:
    dev = _lib.require_cuda(tensor_2bits, tensor_high_2bits, scale, zero_point, boost_idx, out)
    D, G4 = tensor_2bits.shape
    for t, n in ((tensor_2bits, "tensor_2bits"), (tensor_high_2bits, "tensor_high_2bits")):
        if not t.is_contiguous():
            raise RuntimeError(f"{n} must be contiguous")
    if scale.dtype != zero_point.dtype or scale.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("scale and zero_point must both be float16 or both bfloat16")
    if scale.stride(0) != 1 or zero_point.stride(0) != 1 or boost_idx.stride(0) != 1:
        raise RuntimeError("scale, zero_point and boost_idx need unit stride")
    a = _lib.KeyDequantArgs()
    a.key_low = tensor_2bits.data_ptr()
    a.key_high = tensor_high_2bits.data_ptr() if tensor_high_2bits.numel() else tensor_2bits.data_ptr()
    a.key_scale = scale.data_ptr(); a.key_zero = zero_point.data_ptr()
    z32 = _lib.zeros_const(dev, torch.int32)
    a.src_page = z32.data_ptr(); a.head = z32.data_ptr()
    a.boost_idx = boost_idx.data_ptr(); a.bidx_s_head = 0
    a.out = out.data_ptr(); a.out_off = _lib.zeros_const(dev, torch.int64).data_ptr()
    a.out_s_ch, a.out_s_tok = out.stride(0), out.stride(1)
    a.n_jobs, a.num_heads, a.head_dim, a.group, a.d_boost = 1, 1, D, G4 * 4, int(D_boost)
    a.dtype = _lib.dequant_dtype_code(scale.dtype, out.dtype)
    lib = _lib.load()
    _lib.check(lib.kitty_dequantize_key_pages(a, _lib.stream_ptr(dev)), "kitty_dequantize_key_pages")


def dequantize_key_page(tensor_2bits: torch.Tensor, tensor_high_2bits: torch.Tensor, scale: torch.Tensor,
                        zero_point: torch.Tensor, boost_idx: torch.Tensor, D_boost: int,
                        out: torch.Tensor) -> None:
    """Dequantise one key page into a pre-allocated (D, G) float16 (or, with bfloat16
    metadata, bfloat16) tensor (reference signature ``dequantize_key.py:169-177``)."""
    D, G4 = tensor_2bits.shape
    if tuple(out.shape) != (D, G4 * 4):
        raise RuntimeError(f"out must be ({D}, {G4 * 4})")
    _launch(tensor_2bits, tensor_high_2bits, scale, zero_point, boost_idx, D_boost, out)


def dequantize_key_page_torch(tensor_2bits: torch.Tensor, tensor_high_2bits: torch.Tensor, scale: torch.Tensor,
                              zero_point: torch.Tensor, boost_idx: torch.Tensor, D_boost: int) -> torch.Tensor:
    """Functional form returning the float32 (D, G) block, as the reference does
    (``dequantize_key.py:35-97``), by the CUDA key dequantiser with float32 output."""
    D, G4 = tensor_2bits.shape
    dev = _lib.require_cuda(tensor_2bits, tensor_high_2bits, scale, zero_point, boost_idx)
    out = torch.empty(D, G4 * 4, dtype=torch.float32, device=dev)
    _launch(tensor_2bits, tensor_high_2bits, scale.contiguous(), zero_point.contiguous(), boost_idx.contiguous(),
            D_boost, out)
    return out
