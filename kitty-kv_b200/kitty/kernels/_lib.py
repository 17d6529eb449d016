"""ctypes binding of ``libkitty_b200.so`` (the C ABI in ``include/kitty_b200.h``).

The library is loaded on first use.  There is no fallback: if it is missing,
was built for another ABI version, or a tensor is not on a CUDA device, the
call raises ``RuntimeError``.  Every entry point is launched on the current
torch CUDA stream of the tensors' device.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path
from typing import Dict, Optional, Tuple

import torch

ABI_VERSION = 5
LIB_NAME = "libkitty_b200.so"
_LIB_PATH = Path(os.environ.get("KITTY_B200_LIB", Path(__file__).resolve().parent.parent / LIB_NAME))

c_i32, c_i64, c_ptr, c_f32, c_size = ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p, ctypes.c_float, ctypes.c_size_t

KITTY_OK = 0
DTYPE_F16, DTYPE_BF16 = 0, 1
ERROR_NAMES = {1: "invalid argument", 2: "unsupported", 3: "CUDA error", 4: "workspace"}


class KeyQuantArgs(ctypes.Structure):
    _fields_ = [("key", c_ptr), ("key_off", c_ptr), ("key_s_head", c_i64), ("key_s_tok", c_i64),
                ("key_s_ch", c_i64), ("boost_idx", c_ptr), ("bidx_s_head", c_i64), ("dst_page", c_ptr),
                ("key_low", c_ptr), ("key_high", c_ptr), ("key_scale", c_ptr), ("key_zero", c_ptr),
                ("low_s_page", c_i64), ("low_s_head", c_i64), ("high_s_page", c_i64), ("high_s_head", c_i64),
                ("meta_s_page", c_i64), ("meta_s_head", c_i64), ("n_jobs", c_i32), ("num_heads", c_i32),
                ("head_dim", c_i32), ("group", c_i32), ("d_boost", c_i32), ("sentinel", c_i32), ("dtype", c_i32)]


class ValueQuantArgs(ctypes.Structure):
    _fields_ = [("value", c_ptr), ("value_off", c_ptr), ("val_s_head", c_i64), ("val_s_tok", c_i64),
                ("val_s_ch", c_i64), ("n_valid", c_ptr), ("dst_page", c_ptr), ("val_codes", c_ptr),
                ("val_scale", c_ptr), ("val_zero", c_ptr), ("codes_s_page", c_i64), ("codes_s_head", c_i64),
                ("meta_s_page", c_i64), ("meta_s_head", c_i64), ("meta_s_tok", c_i64), ("n_jobs", c_i32),
                ("num_heads", c_i32), ("head_dim", c_i32), ("group", c_i32), ("dtype", c_i32)]


class KeyDequantArgs(ctypes.Structure):
    _fields_ = [("key_low", c_ptr), ("key_high", c_ptr), ("key_scale", c_ptr), ("key_zero", c_ptr),
                ("low_s_page", c_i64), ("low_s_head", c_i64), ("high_s_page", c_i64), ("high_s_head", c_i64),
                ("meta_s_page", c_i64), ("meta_s_head", c_i64), ("src_page", c_ptr), ("head", c_ptr),
                ("boost_idx", c_ptr), ("bidx_s_head", c_i64), ("out", c_ptr), ("out_off", c_ptr),
                ("out_s_ch", c_i64), ("out_s_tok", c_i64), ("n_jobs", c_i32), ("num_heads", c_i32),
                ("head_dim", c_i32), ("group", c_i32), ("d_boost", c_i32), ("dtype", c_i32)]


class ValueDequantArgs(ctypes.Structure):
    _fields_ = [("val_codes", c_ptr), ("val_scale", c_ptr), ("val_zero", c_ptr), ("codes_s_page", c_i64),
                ("codes_s_head", c_i64), ("meta_s_page", c_i64), ("meta_s_head", c_i64), ("meta_s_tok", c_i64),
                ("src_page", c_ptr), ("head", c_ptr), ("out", c_ptr), ("out_off", c_ptr), ("out_s_tok", c_i64),
                ("out_s_ch", c_i64), ("n_jobs", c_i32), ("head_dim", c_i32), ("group", c_i32), ("dtype", c_i32)]


class DecodeArgs(ctypes.Structure):
    _fields_ = [("batch", c_i32), ("num_q_heads", c_i32), ("num_kv_heads", c_i32), ("head_dim", c_i32),
                ("group", c_i32), ("d_boost", c_i32), ("sm_scale", c_f32),
                ("q", c_ptr), ("q_s_seq", c_i64), ("q_s_head", c_i64),
                ("out", c_ptr), ("out_s_seq", c_i64), ("out_s_head", c_i64),
                ("block_table", c_ptr), ("bt_s_seq", c_i64), ("num_pages", c_ptr), ("pool_pages", c_i64),
                ("key_low", c_ptr), ("key_high", c_ptr), ("key_meta", c_ptr), ("val_codes", c_ptr),
                ("val_meta", c_ptr), ("boost_idx", c_ptr), ("bidx_s_head", c_i64),
                ("sink_k", c_ptr), ("sk_s_seq", c_i64), ("sk_s_head", c_i64), ("sk_s_tok", c_i64),
                ("sink_v", c_ptr), ("sv_s_seq", c_i64), ("sv_s_head", c_i64), ("sv_s_tok", c_i64),
                ("sink_len", c_ptr), ("sink_len_all", c_i32),
                ("tail_k", c_ptr), ("tk_s_seq", c_i64), ("tk_s_head", c_i64), ("tk_s_tok", c_i64),
                ("tail_v", c_ptr), ("tv_s_seq", c_i64), ("tv_s_head", c_i64), ("tv_s_tok", c_i64),
                ("tail_len", c_ptr), ("tail_len_all", c_i32),
                ("max_pages_per_seq", c_i32), ("num_splits", c_i32),
                ("workspace", c_ptr), ("workspace_bytes", c_size), ("seq_map", c_ptr), ("dtype", c_i32)]


class CacheState(ctypes.Structure):
    _fields_ = [("max_seqs", c_i32), ("num_heads", c_i32), ("head_dim", c_i32), ("group", c_i32),
                ("sink_size", c_i32), ("d_boost", c_i32), ("sentinel", c_i32), ("max_pages_per_seq", c_i32),
                ("pool_pages", c_i64), ("boost_idx", c_ptr), ("bidx_s_head", c_i64),
                ("sink_k", c_ptr), ("sink_v", c_ptr), ("tail_k", c_ptr), ("tail_v", c_ptr),
                ("sink_len", c_ptr), ("tail_len", c_ptr), ("num_pages", c_ptr), ("claim", c_ptr),
                ("block_table", c_ptr), ("free_pages", c_ptr), ("free_top", c_ptr),
                ("key_low", c_ptr), ("key_high", c_ptr), ("key_meta", c_ptr), ("val_codes", c_ptr),
                ("val_meta", c_ptr), ("job_off", c_ptr), ("job_page", c_ptr), ("job_slot", c_ptr), ("dtype", c_i32)]


class PrefillArgs(ctypes.Structure):
    _fields_ = [("n", c_i32), ("seq_ids", c_ptr), ("lengths", c_ptr), ("row_start", c_ptr),
                ("key", c_ptr), ("value", c_ptr), ("s_tok", c_i64), ("s_head", c_i64), ("max_pages", c_i32),
                ("page_off", c_ptr), ("page_dst", c_ptr), ("seq_plan", c_ptr)]


TP_MAX_RANKS = 8


class TpGatherArgs(ctypes.Structure):
    _fields_ = [("world", c_i32), ("rank", c_i32), ("region", c_ptr * TP_MAX_RANKS), ("data_bytes", ctypes.c_uint64),
                ("src", c_ptr), ("src_bytes", ctypes.c_uint64), ("dst_offset", ctypes.c_uint64), ("dst", c_ptr)]


# Every symbol the header declares, with its ctypes signature.
SIGNATURES = {
    "kitty_abi_version": (ctypes.c_int, []),
    "kitty_last_error": (ctypes.c_char_p, []),
    "kitty_args_size": (c_size, [ctypes.c_int]),
    "kitty_quantize_key_pages": (ctypes.c_int, [ctypes.POINTER(KeyQuantArgs), c_ptr]),
    "kitty_quantize_value_pages": (ctypes.c_int, [ctypes.POINTER(ValueQuantArgs), c_ptr]),
    "kitty_dequantize_key_pages": (ctypes.c_int, [ctypes.POINTER(KeyDequantArgs), c_ptr]),
    "kitty_dequantize_value_pages": (ctypes.c_int, [ctypes.POINTER(ValueDequantArgs), c_ptr]),
    "kitty_paged_decode_workspace_size": (ctypes.c_int, [ctypes.POINTER(DecodeArgs), ctypes.POINTER(c_size),
                                                         ctypes.POINTER(c_i32)]),
    "kitty_paged_decode": (ctypes.c_int, [ctypes.POINTER(DecodeArgs), c_ptr]),
    "kitty_device_error_flags": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int]),
    "kitty_paged_decode_noalloc": (ctypes.c_int, [ctypes.POINTER(DecodeArgs), c_ptr]),
    "kitty_decode_force_variant": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    "kitty_cache_reset": (ctypes.c_int, [ctypes.POINTER(CacheState), c_ptr]),
    "kitty_cache_append": (ctypes.c_int, [ctypes.POINTER(CacheState), c_i32, c_ptr, c_ptr, c_i64, c_i64,
                                          c_ptr, c_i64, c_i64, c_ptr]),
    "kitty_cache_prefill": (ctypes.c_int, [ctypes.POINTER(CacheState), ctypes.POINTER(PrefillArgs), c_ptr]),
    "kitty_cache_release": (ctypes.c_int, [ctypes.POINTER(CacheState), c_i32, c_ptr, c_ptr]),
    "kitty_tp_region_bytes": (c_size, [ctypes.c_uint64]),
    "kitty_tp_region_alloc": (ctypes.c_int, [ctypes.c_uint64, ctypes.POINTER(c_ptr)]),
    "kitty_tp_region_free": (ctypes.c_int, [c_ptr]),
    "kitty_tp_ipc_handle": (ctypes.c_int, [c_ptr, c_ptr]),
    "kitty_tp_ipc_open": (ctypes.c_int, [c_ptr, ctypes.POINTER(c_ptr)]),
    "kitty_tp_ipc_close": (ctypes.c_int, [c_ptr]),
    "kitty_tp_allgather": (ctypes.c_int, [ctypes.POINTER(TpGatherArgs), c_ptr]),
}
STRUCTS = {0: KeyQuantArgs, 1: ValueQuantArgs, 2: KeyDequantArgs, 3: DecodeArgs, 4: CacheState, 5: PrefillArgs,
           6: ValueDequantArgs, 7: TpGatherArgs}

_lib: Optional[ctypes.CDLL] = None
_lock = threading.Lock()


def library_path() -> Path:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load the library (once), bind every signature and check the ABI."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not _LIB_PATH.exists():
            raise RuntimeError(
                f"Kitty CUDA library not found at {_LIB_PATH}. Build it with "
                "`python kitty-kv_b200/build.py` (there is no CPU fallback).")
        lib = ctypes.CDLL(str(_LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.kitty_abi_version() != ABI_VERSION:
            raise RuntimeError(f"{_LIB_PATH} has ABI version {lib.kitty_abi_version()}, expected {ABI_VERSION}")
        for kind, st in STRUCTS.items():
            if lib.kitty_args_size(kind) != ctypes.sizeof(st):
                raise RuntimeError(f"struct layout mismatch for {st.__name__}: library "
                                   f"{lib.kitty_args_size(kind)} bytes, binding {ctypes.sizeof(st)}")
        _lib = lib
        return lib


def check(rc: int, what: str) -> None:
    if rc != KITTY_OK:
        msg = load().kitty_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed ({ERROR_NAMES.get(rc, rc)}): {msg}")


def device_error_flags(clear: bool = True) -> int:
    """Sticky device-side error bits (bit 0: a decode wait timed out; bits 1-5: cache
    append / prefill / release, ``CACHE_ERRORS``); synchronises."""
    v = ctypes.c_uint32(0)
    check(load().kitty_device_error_flags(ctypes.byref(v), int(clear)), "kitty_device_error_flags")
    return v.value


CACHE_ERRORS = {1 << 1: "no free page", 1 << 2: "block table full",
                1 << 3: "sequence id out of range or repeated in a batch", 1 << 4: "free-page stack overflow",
                1 << 5: "prefill page budget (max_pages) too small"}

DECODE_VARIANTS = {"auto": -1, "simt": 0, "int8": 2, "tc": 3}


def force_decode_variant(name: str) -> str:
    """Pin the decode kernel family ("auto", "simt", "int8" or "tc") for later decode
    calls of this process; returns the previous setting.  Shapes the pinned family
    does not support fall back to the library's choice."""
    prev = ctypes.c_int(-1)
    check(load().kitty_decode_force_variant(DECODE_VARIANTS[name], ctypes.byref(prev)), "kitty_decode_force_variant")
    return {v: k for k, v in DECODE_VARIANTS.items()}[prev.value]


def dtype_code(dtype: torch.dtype) -> int:
    """KITTY_DTYPE_* of a 16-bit float torch dtype; other dtypes raise."""
    if dtype == torch.float16:
        return DTYPE_F16
    if dtype == torch.bfloat16:
        return DTYPE_BF16
    raise RuntimeError(f"expected a float16 or bfloat16 tensor, got {dtype}")


DTYPE_BF16_F16META = 3
DTYPE_F16_F32OUT, DTYPE_BF16_F32OUT = 4, 5


def dequant_dtype_code(meta: torch.dtype, out: torch.dtype) -> int:
    """KITTY_DTYPE_* of a dequantiser call: metadata of a 16-bit type and an output of
    the same type or float32."""
    code = dtype_code(meta)
    if out == meta:
        return code
    if out == torch.float32:
        return DTYPE_F16_F32OUT if code == DTYPE_F16 else DTYPE_BF16_F32OUT
    raise RuntimeError(f"output dtype {out} does not go with {meta} metadata (same type or float32)")


def quant_dtype_code(src: torch.dtype, meta: torch.dtype) -> int:
    """KITTY_DTYPE_* of a quantiser call: the source's type, metadata of the same
    type, or fp16 metadata for a bf16 source (the reference's functional forms)."""
    code = dtype_code(src)
    if meta == src:
        return code
    if src == torch.bfloat16 and meta == torch.float16:
        return DTYPE_BF16_F16META
    raise RuntimeError(f"metadata dtype {meta} does not go with a {src} source")


def require_cuda(*tensors: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("Kitty B200 kernels need CUDA tensors (there is no CPU path); "
                               f"got a tensor on {t.device}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    if dev is None:
        raise RuntimeError("no CUDA tensor given")
    return dev


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: Optional[torch.Tensor]) -> int:
    return 0 if t is None else t.data_ptr()


# Small per-device constant tensors reused by single-page calls (no per-call allocation).
_consts: Dict[Tuple[torch.device, str], torch.Tensor] = {}


def zeros_const(device: torch.device, dtype: torch.dtype, n: int = 1) -> torch.Tensor:
    key = (device, f"{dtype}:{n}")
    t = _consts.get(key)
    if t is None:
        t = torch.zeros(n, dtype=dtype, device=device)
        _consts[key] = t
    return t
