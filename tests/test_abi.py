"""The C-ABI library loads (no GPU needed for loading) and exports exactly the
functions ``include/kitty_b200.h`` declares, with matching ABI version and
argument-struct layouts.  No compute entry point is called here."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from kitty.kernels import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "kitty_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\**(kitty_\w+)\s*\(", text, flags=re.M)))


def test_library_built():
    assert _lib.library_path().exists(), "run `python kitty-kv_b200/build.py` (or __graft_entry__.build())"


def test_exports_every_declared_symbol():
    names = declared_functions()
    assert len(names) >= 8
    lib = ctypes.CDLL(str(_lib.library_path()))
    for n in names:
        assert hasattr(lib, n), f"{n} declared in the header but not exported"
    assert set(names) == set(_lib.SIGNATURES), "binding and header disagree"
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.library_path())], capture_output=True, text=True)
    if out.returncode == 0:
        exported = set(re.findall(r"\sT\s(kitty_\w+)$", out.stdout, flags=re.M))
        assert exported == set(names), f"extra or missing exports: {exported ^ set(names)}"


def test_abi_version_and_struct_layouts():
    lib = _lib.load()
    assert lib.kitty_abi_version() == _lib.ABI_VERSION
    for kind, st in _lib.STRUCTS.items():
        assert lib.kitty_args_size(kind) == ctypes.sizeof(st), st.__name__
    assert lib.kitty_args_size(99) == 0
    assert lib.kitty_last_error() == b""


def test_null_args_are_rejected_without_a_gpu():
    lib = _lib.load()
    assert lib.kitty_quantize_key_pages(None, None) == 1
    assert b"NULL" in lib.kitty_last_error()
    a = _lib.DecodeArgs()
    a.batch, a.num_q_heads, a.num_kv_heads, a.head_dim, a.group = 1, 3, 2, 16, 8
    assert lib.kitty_paged_decode(a, None) == 1          # 3 q heads over 2 kv heads
    assert b"multiple" in lib.kitty_last_error()


def test_tp_allgather_argument_checks_without_a_gpu():
    """kitty_tp_allgather rejects bad rank counts, missing or unaligned regions and
    slices that do not fit, before touching the device."""
    lib = _lib.load()
    assert lib.kitty_tp_region_bytes(1 << 20) == 2 * (1 << 20) + 256
    assert lib.kitty_tp_region_bytes(1000) == 2 * 1024 + 256     # buffers rounded to 256 bytes

    def args(**kw):
        a = _lib.TpGatherArgs()
        a.world, a.rank, a.data_bytes, a.src_bytes, a.dst_offset = 2, 0, 4096, 2048, 0
        a.src, a.dst = 0x1000, 0x2000
        a.region[0], a.region[1] = 0x10000, 0x20000
        for k, v in kw.items():
            setattr(a, k, v)
        return a

    cases = [dict(world=0), dict(world=9), dict(rank=2), dict(rank=-1), dict(src=0), dict(dst=0x2004),
             dict(data_bytes=4100), dict(src_bytes=0), dict(dst_offset=3072), dict(dst_offset=8)]
    for kw in cases:
        assert lib.kitty_tp_allgather(args(**kw), None) == 1, kw
        assert lib.kitty_last_error() != b""
    a = args()
    a.region[1] = 0x20010                                    # not 256-byte aligned
    assert lib.kitty_tp_allgather(a, None) == 1
    a.region[1] = 0
    assert lib.kitty_tp_allgather(a, None) == 1
    assert lib.kitty_tp_region_alloc(0, ctypes.byref(_lib.c_ptr())) == 1
    assert lib.kitty_tp_ipc_handle(None, None) == 1


C_PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "kitty_b200.h"
/* every declared entry point is referenced, so the link checks the exports; only the
   calls that need no GPU are made */
typedef int (*any_fn)(void);
int main(void) {
  any_fn fns[] = {
    (any_fn)kitty_quantize_key_pages, (any_fn)kitty_quantize_value_pages, (any_fn)kitty_dequantize_key_pages,
    (any_fn)kitty_dequantize_value_pages,
    (any_fn)kitty_paged_decode_workspace_size, (any_fn)kitty_paged_decode, (any_fn)kitty_paged_decode_noalloc,
    (any_fn)kitty_device_error_flags, (any_fn)kitty_decode_force_variant, (any_fn)kitty_cache_reset,
    (any_fn)kitty_cache_append, (any_fn)kitty_cache_prefill, (any_fn)kitty_cache_release,
    (any_fn)kitty_tp_region_bytes, (any_fn)kitty_tp_region_alloc, (any_fn)kitty_tp_region_free,
    (any_fn)kitty_tp_ipc_handle, (any_fn)kitty_tp_ipc_open, (any_fn)kitty_tp_ipc_close, (any_fn)kitty_tp_allgather};
  if (kitty_abi_version() != KITTY_ABI_VERSION) return 1;
  if (kitty_args_size(0) != sizeof(KittyKeyQuantArgs) || kitty_args_size(1) != sizeof(KittyValueQuantArgs) ||
      kitty_args_size(2) != sizeof(KittyKeyDequantArgs) || kitty_args_size(3) != sizeof(KittyDecodeArgs) ||
      kitty_args_size(4) != sizeof(KittyCacheState) || kitty_args_size(5) != sizeof(KittyPrefillArgs) ||
      kitty_args_size(6) != sizeof(KittyValueDequantArgs) || kitty_args_size(7) != sizeof(KittyTpGatherArgs))
    return 2;
  KittyDecodeArgs a;
  memset(&a, 0, sizeof(a));
  a.batch = 1; a.num_q_heads = 3; a.num_kv_heads = 2; a.head_dim = 16; a.group = 8;
  if (kitty_paged_decode(&a, NULL) != KITTY_ERR_INVALID_ARGUMENT) return 3;
  if (strlen(kitty_last_error()) == 0) return 4;
  if (kitty_cache_append(NULL, 0, NULL, NULL, 0, 0, NULL, 0, 0, NULL) != KITTY_ERR_INVALID_ARGUMENT) return 5;
  if (kitty_tp_region_bytes(1024) != 2 * 1024 + 256) return 6;
  if (kitty_tp_allgather(NULL, NULL) != KITTY_ERR_INVALID_ARGUMENT) return 7;
  KittyTpGatherArgs t;
  memset(&t, 0, sizeof(t));
  t.world = 9;
  if (kitty_tp_allgather(&t, NULL) != KITTY_ERR_INVALID_ARGUMENT) return 8;
  printf("%d entry points\n", (int)(sizeof(fns) / sizeof(fns[0])));
  return 0;
}
"""


def test_header_compiles_as_c_and_links(tmp_path):
    """A plain C program (gcc, C99) includes the header, references every entry point,
    links against the library and checks the struct sizes against it (no GPU call)."""
    import shutil
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    src = tmp_path / "abi_check.c"
    src.write_text(C_PROGRAM)
    exe = tmp_path / "abi_check"
    lib = _lib.library_path()
    cmd = ["gcc", "-std=c99", "-Wall", "-Werror", "-Wno-cast-function-type", "-I", str(HEADER.parent), str(src),
           "-o", str(exe), str(lib), f"-Wl,-rpath,{lib.parent}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, (out.returncode, out.stdout, out.stderr)
    assert out.stdout.strip() == f"{len(declared_functions()) - 3} entry points"
