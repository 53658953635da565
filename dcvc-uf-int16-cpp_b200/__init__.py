"""Python view of the B200 INT16 engine (libufb200.so, C ABI in include/uf_b200.h).

The functions below mirror the reference's ``uf::int16`` CUDA dispatch
(``src/int16_ops.cpp:65-204`` over ``include/uf/cuda_ops.hpp:10-23``): they
take CUDA int16/uint8 torch tensors, allocate the result like the reference
does (``torch::empty`` on the input's device) and launch on the current torch
stream.  PyTorch is only the allocator and stream provider here; all
arithmetic runs in the library's own sm_100a kernels.  There is no fallback:
if the library is missing, every call raises.
"""
from __future__ import annotations

import ctypes as C
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libufb200.so")
ROOT = os.path.dirname(HERE)
HEADER = os.path.join(ROOT, "include", "uf_b200.h")

_LIB = None


class UfbError(RuntimeError):
    """Raised for a failing C-ABI call; ``code`` is the UFB_E* value."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def library():
    """Load libufb200.so (raises if it was not built)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise UfbError(-3, f"{LIB_PATH} is missing; build it with build.py")
        L = C.CDLL(LIB_PATH)
        vp, i16, i64 = C.c_void_p, C.c_int, C.c_int64
        L.ufb_last_error.restype = C.c_char_p
        L.ufb_version.restype = C.c_int
        conv_args = [vp, i16, i16, i16, i16, vp, i16, i16, i16, vp, i16, i16, i16, i16, i16, i16, vp, vp]
        for name in ("ufb_conv2d", "ufb_conv2d_generic", "ufb_conv2d_baseline"):
            getattr(L, name).argtypes = conv_args
        L.ufb_add.argtypes = [C.c_int, C.POINTER(C.c_void_p), i64, vp, vp]
        L.ufb_mul.argtypes = [vp, C.POINTER(C.c_int64), vp, C.POINTER(C.c_int64), vp, vp]
        L.ufb_lut.argtypes = [vp, i64, vp, C.c_int, vp, vp]
        L.ufb_bytes.argtypes = [vp, i64, vp, vp]
        L.ufb_wsilu4.argtypes = [vp, C.c_int, C.c_int, C.c_int, C.c_int, vp, vp, vp]
        L.ufb_warp.argtypes = [vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, vp, vp]
        L.ufb_device_status.argtypes = [C.c_int]
        _LIB = L
    return _LIB


def _check(rc: int):
    if rc != 0:
        raise UfbError(rc, library().ufb_last_error().decode())


def _stream(t: torch.Tensor):
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _cuda(t: torch.Tensor, dtype, what: str) -> torch.Tensor:
    if not (isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == dtype):
        raise UfbError(-1, f"{what}: CUDA {dtype} tensor required")
    return t.contiguous()


def device_status(device: int = 0) -> int:
    """Synchronise and return/clear the device's kernel pipeline status word."""
    rc = library().ufb_device_status(device)
    if rc < 0:
        _check(rc)
    return rc


def conv2d(x, weight, bias=None, stride_h=1, stride_w=1, pad_h=0, pad_w=0, groups=1, variant="auto"):
    """uf::int16::conv2d on CUDA (src/int16_ops.cpp:173-204 -> uf_conv)."""
    L = library()
    x = _cuda(x, torch.int16, "conv2d input")
    weight = _cuda(weight, torch.int16, "conv2d weight")
    if x.dim() != 4 or weight.dim() != 4:
        raise UfbError(-1, "Unsupported INT16 convolution arguments")
    n, ci, h, w = x.shape
    co, _, kh, kw = weight.shape
    if weight.shape[1] * groups != ci or co % groups:
        raise UfbError(-1, "invalid groups")
    bias_ptr, bits = None, 0
    if bias is not None:
        if bias.dtype not in (torch.int16, torch.int32) or bias.numel() != co or bias.dim() != 1:
            raise UfbError(-1, "invalid bias")
        bias = bias.contiguous()
        bias_ptr, bits = bias.data_ptr(), 16 if bias.dtype == torch.int16 else 32
    oh = (h + 2 * pad_h - kh) // stride_h + 1
    ow = (w + 2 * pad_w - kw) // stride_w + 1
    out = torch.empty((n, co, max(oh, 0), max(ow, 0)), dtype=torch.int16, device=x.device)
    fn = {"auto": L.ufb_conv2d, "generic": L.ufb_conv2d_generic, "baseline": L.ufb_conv2d_baseline}[variant]
    _check(fn(x.data_ptr(), n, ci, h, w, weight.data_ptr(), co, kh, kw, bias_ptr, bits, stride_h, stride_w, pad_h,
              pad_w, groups, out.data_ptr(), _stream(x)))
    return out


def add(values):
    """uf::int16::add (src/int16_ops.cpp:65-75 -> uf_add)."""
    vs = [_cuda(v, torch.int16, "add") for v in values]
    if any(v.shape != vs[0].shape for v in vs):
        raise UfbError(-1, "add shape/device mismatch")
    out = torch.empty_like(vs[0])
    arr = (C.c_void_p * len(vs))(*[v.data_ptr() for v in vs])
    _check(library().ufb_add(len(vs), arr, vs[0].numel(), out.data_ptr(), _stream(vs[0])))
    return out


def multiply(x, scale):
    """uf::int16::multiply (src/int16_ops.cpp:77-83 -> uf_mul)."""
    x = _cuda(x, torch.int16, "multiply")
    s = _cuda(scale, torch.int16, "multiply scale")
    xs = (C.c_int64 * 4)(*x.shape)
    ss = (C.c_int64 * 4)(*s.shape)
    out = torch.empty_like(x)
    _check(library().ufb_mul(x.data_ptr(), xs, s.data_ptr(), ss, out.data_ptr(), _stream(x)))
    return out


def lookup(x, table):
    """uf::int16::lookup (src/int16_ops.cpp:107-115 -> uf_lut)."""
    x = _cuda(x, torch.int16, "lookup")
    if table.dtype not in (torch.int16, torch.uint8) or table.numel() != 65536 or not table.is_cuda:
        raise UfbError(-1, "invalid lookup table")
    table = table.contiguous()
    out = torch.empty(x.shape, dtype=table.dtype, device=x.device)
    bits = 16 if table.dtype == torch.int16 else 8
    _check(library().ufb_lut(x.data_ptr(), x.numel(), table.data_ptr(), bits, out.data_ptr(), _stream(x)))
    return out


def from_bytes(x):
    """uf::int16::from_bytes (src/int16_ops.cpp:99-105 -> uf_bytes)."""
    x = _cuda(x, torch.uint8, "from_bytes")
    out = torch.empty(x.shape, dtype=torch.int16, device=x.device)
    _check(library().ufb_bytes(x.data_ptr(), x.numel(), out.data_ptr(), _stream(x)))
    return out


def wsilu4(x, table):
    """uf::int16::wsilu4 (src/int16_ops.cpp:117-130 -> uf_wsilu4)."""
    x = _cuda(x, torch.int16, "wsilu4")
    table = _cuda(table, torch.int16, "wsilu4 table")
    if x.dim() != 4 or x.shape[1] % 4 or table.numel() != 65536:
        raise UfbError(-1, "invalid WSiLU4 inputs")
    n, c4, h, w = x.shape
    out = torch.empty((n, c4 // 4, h, w), dtype=torch.int16, device=x.device)
    _check(library().ufb_wsilu4(x.data_ptr(), n, c4, h, w, table.data_ptr(), out.data_ptr(), _stream(x)))
    return out


def warp(feature, flow):
    """Fixed-point backward bilinear warp (Q9 flow, border clamp)."""
    feature = _cuda(feature, torch.int16, "warp feature")
    flow = _cuda(flow, torch.int16, "warp flow")
    n, c, h, w = feature.shape
    if flow.shape != (n, 2, h, w):
        raise UfbError(-1, "Invalid flow shape")
    out = torch.empty_like(feature)
    _check(library().ufb_warp(feature.data_ptr(), flow.data_ptr(), n, c, h, w, out.data_ptr(), _stream(feature)))
    return out
