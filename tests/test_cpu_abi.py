"""CPU-only checks of the boundary: libdi.so loads and exports every symbol include/di.h declares, the
Python binding's signature table covers the same set, and compute entry points refuse cleanly without a
GPU (no CPU fallback)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "di.h").read_text()
    return sorted(set(re.findall(r"^DI_API\s+[\w\s\*]+?\b(di_\w+)\s*\(", text, flags=re.M)))


def test_header_parses():
    syms = declared_symbols()
    assert "di_init" in syms and "di_attention" in syms and len(syms) > 30


def test_library_exports_every_declared_symbol(dib):
    L = ctypes.CDLL(str(dib.LIB_PATH))
    missing = [s for s in declared_symbols() if not hasattr(L, s)]
    assert not missing, f"declared but not exported: {missing}"


def test_binding_table_matches_header(dib):
    assert sorted(dib.SIGNATURES) == declared_symbols()


def test_no_gpu_refuses_cleanly(dib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    h = ctypes.c_void_p()
    rc = dib.lib().di_init(0, ctypes.byref(h))
    assert rc != 0 and not h.value


def test_ops_reject_cpu_tensors(dib):
    import torch
    with pytest.raises(dib.DIError):
        dib.ptr(torch.zeros(4))
