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
