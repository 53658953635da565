"""CPU: the C-ABI library builds, loads, and exports every entry point that
include/uf_b200.h declares (no compute call needs a GPU here)."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "uf_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ufb_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for name in ("ufb_conv2d", "ufb_add", "ufb_mul", "ufb_lut", "ufb_bytes", "ufb_wsilu4", "ufb_warp"):
        assert name in syms


def test_library_exports_every_declared_symbol(ufb):
    lib = ufb.library()
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_version_and_errors_without_gpu(ufb):
    lib = ufb.library()
    assert lib.ufb_version() >= 100
    # argument validation happens before any CUDA call
    rc = lib.ufb_add(1, None, 0, None, None)
    assert rc == -1
    assert b"2 to 4" in lib.ufb_last_error()
    rc = lib.ufb_conv2d(None, 1, 1, 1, 1, None, 1, 1, 1, None, 0, 1, 1, 0, 0, 1, None, None)
    assert rc == -1


def test_package_raises_without_fallback(ufb):
    import torch
    x = torch.zeros((1, 4, 2, 2), dtype=torch.int16)
    try:
        ufb.conv2d(x, torch.zeros((4, 4, 1, 1), dtype=torch.int16))
    except ufb.UfbError as e:
        assert "CUDA" in str(e)
    else:
        raise AssertionError("CPU tensors must be rejected, never computed on the host")
