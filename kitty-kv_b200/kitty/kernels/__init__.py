"""Kitty quantisation / decode kernels - B200 (sm_100a) CUDA implementations.

Same names as the reference's ``kitty/kernels/__init__.py:19-29`` plus the
batched forms.  All of them run the hand-written CUDA kernels of
``libkitty_b200.so`` on CUDA tensors; there is no Triton and no CPU fallback
(CPU tensors raise ``RuntimeError``).  The library is loaded on first use.
"""

from .quantize_key import quantize_key_page, quantize_key_page_torch, quantize_key_pages
from .dequantize_key import dequantize_key_page, dequantize_key_page_torch
from .quantize_value import (
    quantize_value_page,
    quantize_value_page_torch,
    quantize_value_pages,
    dequantize_value_page_torch,
)
from .attention import paged_attention, paged_attention_reference, paged_attention_batched

__all__ = [
    "quantize_key_page",
    "quantize_key_page_torch",
    "dequantize_key_page",
    "dequantize_key_page_torch",
    "quantize_value_page",
    "quantize_value_page_torch",
    "dequantize_value_page_torch",
    "paged_attention",
    "paged_attention_reference",
    # batched extensions
    "quantize_key_pages",
    "quantize_value_pages",
    "paged_attention_batched",
]
