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
        L.ufb_set_conv_max_ctas.argtypes = [C.c_int]
        L.ufb_set_conv_narrow.argtypes = [C.c_int]
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


def set_conv_max_ctas(n: int) -> None:
    """Testing aid: cap the persistent tensor-core and depthwise convolution
    grids at n CTAs (0: no cap)."""
    _check(library().ufb_set_conv_max_ctas(int(n)))


def set_conv_narrow(enable: bool) -> None:
    """Testing aid: enable or disable the narrow convolution recombination
    (identical outputs either way)."""
    _check(library().ufb_set_conv_narrow(1 if enable else 0))


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


# ---------------------------------------------------------------- engine ----
# Host-array wrappers of the model / codec / rANS entry points.  The engine owns
# its device memory and CUDA stream; these calls take and return numpy arrays.

import numpy as _np

_DTYPE_CODES = {_np.dtype(_np.int16): 0, _np.dtype(_np.uint8): 1, _np.dtype(_np.int32): 2,
                _np.dtype(_np.int8): 3, _np.dtype(_np.int64): 4}


def _engine_lib():
    L = library()
    if getattr(L, "_engine_ready", False):
        return L
    vp, ci, i64, sz = C.c_void_p, C.c_int, C.c_int64, C.c_size_t
    L.ufb_rans_create.restype = vp
    L.ufb_rans_create.argtypes = [vp, ci, ci, vp, vp, ci, ci, vp]
    L.ufb_rans_destroy.argtypes = [vp]
    L.ufb_rans_encode.restype = i64
    L.ufb_rans_encode.argtypes = [vp, ci, C.POINTER(vp), C.POINTER(sz), vp, sz, ci, ci, vp, sz]
    L.ufb_rans_decode.argtypes = [vp, vp, sz, sz, ci, ci, vp, ci, C.POINTER(vp), C.POINTER(sz), C.POINTER(vp)]
    L.ufb_model_create.restype = vp
    L.ufb_model_create.argtypes = [ci, C.c_char_p, ci, C.POINTER(C.c_char_p), C.POINTER(ci), C.POINTER(ci),
                                   C.POINTER(i64), C.POINTER(vp)]
    L.ufb_model_destroy.argtypes = [vp]
    L.ufb_model_run.argtypes = [vp, C.c_char_p, ci, C.POINTER(vp), C.POINTER(i64), C.c_char_p, ci, vp, i64,
                                C.POINTER(i64)]
    L.ufb_codec_create.restype = vp
    L.ufb_codec_create.argtypes = [vp, ci]
    L.ufb_codec_destroy.argtypes = [vp]
    L.ufb_codec_set_skip_threshold.argtypes = [vp, C.c_double]
    L.ufb_codec_clear_dpb.argtypes = [vp]
    L.ufb_codec_add_ref_frames.argtypes = [vp, vp, ci, ci]
    L.ufb_codec_decompress.argtypes = [vp, C.POINTER(vp), C.POINTER(sz), C.c_uint32, C.c_uint32, ci, ci, ci, vp, vp]
    L.ufb_codec_compress.argtypes = [vp, vp, ci, ci, ci, ci, ci, vp, sz, C.POINTER(sz), vp]
    L.ufb_codec_state.argtypes = [vp, ci, vp, i64, C.POINTER(i64)]
    L.ufb_codec_host_seconds.restype = C.c_double
    L.ufb_codec_host_seconds.argtypes = [vp]
    L.ufb_codec_set_reference_from.argtypes = [vp, vp]
    L.ufb_codec_set_stream.argtypes = [vp, vp]
    L.ufb_codec_profile.argtypes = [vp, ci]
    L.ufb_codec_stats.argtypes = [vp, ci, C.POINTER(i64), C.POINTER(i64), C.POINTER(C.c_double),
                                  C.POINTER(C.c_double)]
    L.ufb_codec_shape_table.argtypes = [vp, C.c_char_p, i64, C.POINTER(i64)]
    L._engine_ready = True
    return L


def _c(a, dtype):
    return _np.ascontiguousarray(a, dtype=dtype)


class Rans:
    """uf::EntropyEncoder / EntropyDecoder wire format (host)."""

    def __init__(self, tables: dict):
        L = self.L = _engine_lib()
        self._t = [_c(tables[k], _np.int32) for k in ("tables.z_cdf", "tables.z_lengths", "tables.y_cdf",
                                                       "tables.y_lengths")]
        zc, zl, yc, yl = self._t
        self.h = L.ufb_rans_create(zc.ctypes.data, zc.shape[0], zc.shape[1], zl.ctypes.data, yc.ctypes.data,
                                   yc.shape[0], yc.shape[1], yl.ctypes.data)
        if not self.h:
            raise UfbError(-1, L.ufb_last_error().decode())

    def __del__(self):
        if getattr(self, "h", None):
            self.L.ufb_rans_destroy(self.h)
            self.h = None

    def encode(self, y_parts, z, z_offset, z_channels) -> bytes:
        parts = [_c(p, _np.int16) for p in y_parts]
        z = _c(z, _np.int8)
        pp = (C.c_void_p * max(len(parts), 1))(*[p.ctypes.data for p in parts])
        pl = (C.c_size_t * max(len(parts), 1))(*[p.size for p in parts])
        n = self.L.ufb_rans_encode(self.h, len(parts), pp, pl, z.ctypes.data, z.size, z_offset, z_channels, None, 0)
        if n < 0:
            raise UfbError(int(n), self.L.ufb_last_error().decode())
        out = _np.empty(n, _np.uint8)
        self.L.ufb_rans_encode(self.h, len(parts), pp, pl, z.ctypes.data, z.size, z_offset, z_channels,
                               out.ctypes.data, n)
        return out.tobytes()

    def decode(self, payload: bytes, z_count, z_offset, z_channels, index_parts):
        data = _np.frombuffer(payload, _np.uint8).copy()
        z = _np.empty(z_count, _np.int8)
        idx = [_c(i, _np.uint8) for i in index_parts]
        ys = [_np.empty(i.size, _np.int8) for i in idx]
        ip = (C.c_void_p * max(len(idx), 1))(*[i.ctypes.data for i in idx])
        il = (C.c_size_t * max(len(idx), 1))(*[i.size for i in idx])
        yp = (C.c_void_p * max(len(ys), 1))(*[y.ctypes.data for y in ys])
        _check(self.L.ufb_rans_decode(self.h, data.ctypes.data, data.size, z_count, z_offset, z_channels,
                                      z.ctypes.data, len(idx), ip, il, yp))
        return z, ys


class Model:
    """A prepared model resident on one GPU (uf::Layers + tables)."""

    def __init__(self, variant: str, tensors: dict, device: int = 0):
        L = self.L = _engine_lib()
        names = sorted(tensors)
        arrays = [_np.ascontiguousarray(tensors[n]) for n in names]
        c_names = (C.c_char_p * len(names))(*[n.encode() for n in names])
        dtypes = (C.c_int * len(names))(*[_DTYPE_CODES[a.dtype] for a in arrays])
        ndims = (C.c_int * len(names))(*[a.ndim for a in arrays])
        flat = [int(s) for a in arrays for s in a.shape]
        shapes = (C.c_int64 * max(len(flat), 1))(*flat)
        data = (C.c_void_p * len(names))(*[a.ctypes.data for a in arrays])
        self.variant = variant
        self.h = L.ufb_model_create(device, variant.encode(), len(names), c_names, dtypes, ndims, shapes, data)
        if not self.h:
            raise UfbError(-1, L.ufb_last_error().decode())

    def __del__(self):
        if getattr(self, "h", None):
            self.L.ufb_model_destroy(self.h)
            self.h = None

    def run(self, module, *args, q_name=None, qp=0):
        vs = [_c(a, _np.int16) for a in args]
        arr = (C.c_void_p * len(vs))(*[v.ctypes.data for v in vs])
        shapes = (C.c_int64 * (4 * len(vs)))(*[int(s) for v in vs for s in v.shape])
        cap = 1 << 26
        out = _np.empty(cap, _np.int16)
        shape = (C.c_int64 * 4)()
        _check(self.L.ufb_model_run(self.h, module.encode(), len(vs), arr, shapes,
                                    q_name.encode() if q_name else None, qp, out.ctypes.data, cap, shape))
        return out[: int(_np.prod(list(shape)))].reshape(tuple(shape)).copy()


class Codec:
    """uf::IntegerModel for `batch` streams decoded together on the model's GPU."""

    def __init__(self, model: Model, batch: int = 1):
        L = self.L = _engine_lib()
        self.model, self.batch = model, batch
        self.h = L.ufb_codec_create(model.h, batch)
        if not self.h:
            raise UfbError(-1, L.ufb_last_error().decode())

    def __del__(self):
        if getattr(self, "h", None):
            self.L.ufb_codec_destroy(self.h)
            self.h = None

    def set_skip_threshold(self, t):
        _check(self.L.ufb_codec_set_skip_threshold(self.h, float(t)))

    def clear_dpb(self):
        _check(self.L.ufb_codec_clear_dpb(self.h))

    def add_ref_frames(self, frames):
        f = _c(frames, _np.int16)
        _check(self.L.ufb_codec_add_ref_frames(self.h, f.ctypes.data, f.shape[-2], f.shape[-1]))

    def decompress(self, payloads, width, height, qp, reset=False, frames=True, yuv=False, yuv_out=None):
        """Decode one packet per stream.  Returns (frames [B, F, 3, Hp, Wp] int16 or
        None, yuv [B, F, W*H*3/2] uint8 or None).  yuv_out, when given, is a
        C-contiguous uint8 array of that shape that receives the YUV bytes (for
        example page-locked memory reused across packets, which the copy from
        the GPU reaches at full bus speed); it is returned as the yuv result."""
        bufs = [_np.frombuffer(p, _np.uint8).copy() if len(p) else _np.zeros(1, _np.uint8) for p in payloads]
        ptrs = (C.c_void_p * self.batch)(*[b.ctypes.data for b in bufs])
        lens = (C.c_size_t * self.batch)(*[len(p) for p in payloads])
        F = 1 if self.model.variant == "image" else 8
        hp, wp = (height + 15) // 16 * 16, (width + 15) // 16 * 16
        fo = _np.empty((self.batch, F, 3, hp, wp), _np.int16) if frames else None
        yshape = (self.batch, F, width * height * 3 // 2)
        if yuv_out is not None:
            if (not isinstance(yuv_out, _np.ndarray) or yuv_out.dtype != _np.uint8 or yuv_out.shape != yshape or
                    not yuv_out.flags.c_contiguous):
                raise UfbError(-1, f"yuv_out must be a C-contiguous uint8 array of shape {yshape}")
            yuv = True
        yo = (yuv_out if yuv_out is not None else _np.empty(yshape, _np.uint8)) if yuv else None
        rc = self.L.ufb_codec_decompress(self.h, ptrs, lens, width, height, qp, 1, int(reset),
                                         fo.ctypes.data if frames else None, yo.ctypes.data if yuv else None)
        if rc < 0:
            _check(rc)
        return fo, yo

    def compress(self, frames_u8, qp, reset=False, frames=False):
        x = _c(frames_u8, _np.uint8)
        b, c, h, w = x.shape
        cap = max(4096, c * h * w * 2)
        out = _np.empty(self.batch * cap, _np.uint8)
        lens = (C.c_size_t * self.batch)()
        F = 1 if self.model.variant == "image" else 8
        hp, wp = (h + 15) // 16 * 16, (w + 15) // 16 * 16
        fo = _np.empty((self.batch, F, 3, hp, wp), _np.int16) if frames else None
        rc = self.L.ufb_codec_compress(self.h, x.ctypes.data, c, h, w, qp, int(reset), out.ctypes.data, cap, lens,
                                       fo.ctypes.data if frames else None)
        if rc < 0:
            _check(rc)
        return [out[i * cap: i * cap + lens[i]].tobytes() for i in range(self.batch)], fo

    def state(self, which):
        idx = {"reference": 0, "memory": 1, "context": 2}[which]
        cap = 1 << 26
        out = _np.empty(cap, _np.int16)
        shape = (C.c_int64 * 4)()
        rc = self.L.ufb_codec_state(self.h, idx, out.ctypes.data, cap, shape)
        if rc < 0:
            _check(rc)
        if rc == 1:
            return None
        return out[: int(_np.prod(list(shape)))].reshape(tuple(shape)).copy()

    def state_hash(self, which):
        """SHA-256 hex of a DPB state as NCHW int16 little-endian bytes (the
        reference's check-int16 tensor_hash), or None when undefined."""
        L = _stream_lib()
        idx = {"reference": 0, "memory": 1, "context": 2}[which]
        out = (C.c_uint8 * 32)()
        rc = L.ufb_codec_state_hash(self.h, idx, out)
        if rc < 0:
            _check(rc)
        return None if rc == 1 else bytes(out).hex()

    def host_seconds(self):
        return self.L.ufb_codec_host_seconds(self.h)

    def set_reference_from(self, image_codec: "Codec"):
        _check(self.L.ufb_codec_set_reference_from(self.h, image_codec.h))

    def set_stream(self, stream):
        """stream: a torch.cuda.Stream, a raw handle, or None for the codec's own."""
        handle = getattr(stream, "cuda_stream", stream)
        _check(self.L.ufb_codec_set_stream(self.h, C.c_void_p(handle) if handle else None))

    def profile(self, enable=True):
        _check(self.L.ufb_codec_profile(self.h, int(enable)))

    def stats(self, reset=False):
        a, b = C.c_int64(), C.c_int64()
        m, t = C.c_double(), C.c_double()
        _check(self.L.ufb_codec_stats(self.h, int(reset), C.byref(a), C.byref(b), C.byref(m), C.byref(t)))
        return {"launches": a.value, "conv_launches": b.value, "conv_int16_macs": m.value, "conv_ms": t.value}

    def shape_table(self):
        """Profiled convolution time per launch shape and epilogue since the last
        stats reset: {shape: (launches, int16 MACs, ms, algorithmic DRAM bytes)}
        (profiling must be on)."""
        n = C.c_int64()
        _check(self.L.ufb_codec_shape_table(self.h, None, 0, C.byref(n)))
        buf = C.create_string_buffer(n.value + 1)
        _check(self.L.ufb_codec_shape_table(self.h, buf, n.value + 1, C.byref(n)))
        table = {}
        for line in buf.value.decode().splitlines():
            shape, launches, macs, ms, hbm = line.split("\t")
            table[shape] = (int(launches), float(macs), float(ms), float(hbm))
        return table


# ---------------------------------------------------------------------------
# UF16 bitstream container, digests and whole-stream coding
# (uf::read_* / write_* / scan_bitstream, src/bitstream.cpp:173-360;
# uf::IntegerCodec::encode / decode_stream_impl, src/integer_codec.cpp:215-493).
# ---------------------------------------------------------------------------

NAL_SPS, NAL_INTRA, NAL_PREDICTED = 0, 1, 2
PREPARED_FORMAT = "dcvc-uf-prepared-v1"
ARITHMETIC = "uf-int16-q9-w13-acc64-rna-sat-v1"


class Uf16Nal(C.Structure):
    _fields_ = [("type", C.c_int), ("sps_id", C.c_int), ("width", C.c_uint32), ("height", C.c_uint32),
                ("qp", C.c_int), ("entropy_parallel", C.c_int), ("reset", C.c_int),
                ("payload_offset", C.c_uint64), ("payload_length", C.c_uint64)]


class Uf16Summary(C.Structure):
    _fields_ = [("integer", C.c_int), ("image_identity", C.c_uint8 * 32), ("video_identity", C.c_uint8 * 32),
                ("width", C.c_uint32), ("height", C.c_uint32), ("packets", C.c_uint64),
                ("intra_packets", C.c_uint64), ("predicted_packets", C.c_uint64), ("maximum_frames", C.c_uint64)]


FRAME_SINK = C.CFUNCTYPE(None, C.c_void_p, C.c_int, C.c_uint64, C.POINTER(C.c_uint8), C.c_size_t)


def _stream_lib():
    L = _engine_lib()
    if getattr(L, "_stream_ready", False):
        return L
    vp, ci, i64, sz, u32, u64 = C.c_void_p, C.c_int, C.c_int64, C.c_size_t, C.c_uint32, C.c_uint64
    for name, args in (("ufb_uf16_write_preamble", [vp, vp, vp, sz]),
                       ("ufb_uf16_write_sps", [ci, u32, u32, vp, sz]),
                       ("ufb_uf16_write_packet", [ci, ci, ci, ci, ci, vp, sz, vp, sz]),
                       ("ufb_uf16_write_uint", [u32, vp, sz])):
        getattr(L, name).restype = i64
        getattr(L, name).argtypes = args
    L.ufb_uf16_read_uint.argtypes = [vp, sz, C.POINTER(sz), C.POINTER(u32)]
    L.ufb_uf16_read_preamble.argtypes = [vp, sz, C.POINTER(sz), C.POINTER(ci), vp, vp]
    L.ufb_uf16_next.argtypes = [vp, sz, C.POINTER(sz), C.POINTER(Uf16Nal)]
    L.ufb_uf16_scan.argtypes = [vp, sz, C.c_char_p, i64, C.POINTER(Uf16Summary)]
    L.ufb_sha256.argtypes = [vp, sz, vp]
    L.ufb_prepared_identity.argtypes = [C.c_char_p, C.c_char_p, C.c_char_p, C.c_char_p, ci, C.POINTER(C.c_char_p),
                                        C.POINTER(ci), C.POINTER(ci), C.POINTER(i64), C.POINTER(vp), C.c_char_p]
    L.ufb_codec_state_hash.argtypes = [vp, ci, vp]
    L.ufb_set_interrupt.argtypes = [ci]
    L.ufb_set_interrupt.restype = None
    L.ufb_interrupt_requested.restype = ci
    L.ufb_stream_codec_create.restype = vp
    L.ufb_stream_codec_create.argtypes = [vp, vp, vp, vp]
    L.ufb_stream_codec_destroy.argtypes = [vp]
    L.ufb_stream_encode.argtypes = [vp, vp, u64, u32, u32, ci, ci, ci, ci, vp, sz, C.POINTER(sz), C.POINTER(u64)]
    L.ufb_stream_decode.argtypes = [vp, C.POINTER(vp), C.POINTER(sz), u64, u64, u32, u32, FRAME_SINK, vp, vp,
                                    C.POINTER(u64), C.POINTER(u64)]
    L._stream_ready = True
    return L


def _buf(data: bytes):
    """A ctypes view of bytes (kept alive by the caller's reference)."""
    a = _np.frombuffer(bytes(data), _np.uint8)
    return a, (a.ctypes.data if a.size else None)


def _written(n: int, out) -> bytes:
    if n < 0:
        _check(int(n))
    return bytes(out[:n])


def write_preamble(image_identity: bytes, video_identity: bytes = bytes(32)) -> bytes:
    """write_preamble of an integer (UF16) stream: 72 bytes."""
    L = _stream_lib()
    if len(image_identity) != 32 or len(video_identity) != 32:
        raise UfbError(-1, "identities are 32 bytes")
    out = (C.c_uint8 * 72)()
    return _written(L.ufb_uf16_write_preamble(bytes(image_identity), bytes(video_identity), out, 72), out)


def write_sps(sps_id: int, width: int, height: int) -> bytes:
    L = _stream_lib()
    out = (C.c_uint8 * 16)()
    return _written(L.ufb_uf16_write_sps(sps_id, width, height, out, 16), out)


def write_packet(nal_type: int, sps_id: int, qp: int, entropy_parallel: int, reset: bool, payload: bytes) -> bytes:
    L = _stream_lib()
    keep, p = _buf(payload)
    cap = len(payload) + 16
    out = (C.c_uint8 * cap)()
    return _written(L.ufb_uf16_write_packet(nal_type, sps_id, qp, entropy_parallel, int(bool(reset)), p,
                                            len(payload), out, cap), out)


def write_uint(value: int) -> bytes:
    L = _stream_lib()
    out = (C.c_uint8 * 8)()
    return _written(L.ufb_uf16_write_uint(value, out, 8), out)


def read_uint(data: bytes, pos: int = 0):
    """read_uint_adaptive: (value, next position)."""
    L = _stream_lib()
    keep, p = _buf(data)
    at, v = C.c_size_t(pos), C.c_uint32()
    _check(L.ufb_uf16_read_uint(p, len(data), C.byref(at), C.byref(v)))
    return v.value, at.value


def read_preamble(data: bytes, pos: int = 0):
    """read_preamble: ({"integer", "image_identity", "video_identity"}, next position)."""
    L = _stream_lib()
    keep, p = _buf(data)
    at, integer = C.c_size_t(pos), C.c_int()
    img, vid = (C.c_uint8 * 32)(), (C.c_uint8 * 32)()
    _check(L.ufb_uf16_read_preamble(p, len(data), C.byref(at), C.byref(integer), img, vid))
    out = {"integer": bool(integer.value), "image_identity": bytes(32), "video_identity": bytes(32)}
    if integer.value:
        out["image_identity"], out["video_identity"] = bytes(img), bytes(vid)
    return out, at.value


def iter_nals(data: bytes, pos: int = 0):
    """The NAL units from pos on, as dicts (packets carry their payload bytes)."""
    L = _stream_lib()
    keep, p = _buf(data)
    at, nal = C.c_size_t(pos), Uf16Nal()
    while True:
        rc = L.ufb_uf16_next(p, len(data), C.byref(at), C.byref(nal))
        if rc < 0:
            _check(rc)
        if rc == 0:
            return
        if nal.type == NAL_SPS:
            yield {"type": NAL_SPS, "sps_id": nal.sps_id, "width": nal.width, "height": nal.height}
        else:
            o, n = nal.payload_offset, nal.payload_length
            yield {"type": nal.type, "sps_id": nal.sps_id, "qp": nal.qp, "entropy_parallel": nal.entropy_parallel,
                   "reset": bool(nal.reset), "payload": bytes(data[o:o + n])}


def scan_bitstream(data: bytes, variant: str, expected_frames=None) -> dict:
    """scan_bitstream (src/bitstream.cpp:315-358) over a whole stream in memory."""
    L = _stream_lib()
    keep, p = _buf(data)
    s = Uf16Summary()
    _check(L.ufb_uf16_scan(p, len(data), variant.encode(), -1 if expected_frames is None else int(expected_frames),
                           C.byref(s)))
    return {"integer": bool(s.integer), "image_identity": bytes(s.image_identity),
            "video_identity": bytes(s.video_identity), "width": s.width, "height": s.height,
            "packets": s.packets, "intra_packets": s.intra_packets, "predicted_packets": s.predicted_packets,
            "maximum_frames": s.maximum_frames}


def set_interrupt(on: bool = True) -> None:
    """uf::ProcessInterrupt: while set, codec calls stop with UfbError code -6."""
    _stream_lib().ufb_set_interrupt(int(bool(on)))


def interrupt_requested() -> bool:
    return bool(_stream_lib().ufb_interrupt_requested())


def sha256(data) -> bytes:
    L = _stream_lib()
    a = _np.ascontiguousarray(_np.frombuffer(bytes(data), _np.uint8) if isinstance(data, (bytes, bytearray))
                              else data).view(_np.uint8)
    out = (C.c_uint8 * 32)()
    _check(L.ufb_sha256(a.ctypes.data if a.size else None, a.nbytes, out))
    return bytes(out)


def prepared_identity(tensors: dict, variant: str, source_sha256: str = "", format: str = PREPARED_FORMAT,
                      arithmetic: str = ARITHMETIC) -> str:
    """uf::prepared_identity (src/prepared.cpp:64-105): 64 hex digits."""
    L = _stream_lib()
    names = sorted(tensors)
    arrays = [_np.ascontiguousarray(tensors[n]) for n in names]
    c_names = (C.c_char_p * max(len(names), 1))(*[n.encode() for n in names])
    dtypes = (C.c_int * max(len(names), 1))(*[_DTYPE_CODES[a.dtype] for a in arrays])
    ndims = (C.c_int * max(len(names), 1))(*[a.ndim for a in arrays])
    flat = [int(s) for a in arrays for s in a.shape]
    shapes = (C.c_int64 * max(len(flat), 1))(*flat)
    data = (C.c_void_p * max(len(names), 1))(*[a.ctypes.data for a in arrays])
    out = C.create_string_buffer(65)
    _check(L.ufb_prepared_identity(format.encode(), arithmetic.encode(), variant.encode(), source_sha256.encode(),
                                   len(names), c_names, dtypes, ndims, shapes, data, out))
    return out.value.decode()


class StreamCodec:
    """uf::IntegerCodec over an image codec and an optional video codec of the
    same batch: B independent UF16 streams coded in lock step."""

    def __init__(self, image: Codec, video: "Codec | None", image_identity: bytes, video_identity: bytes = bytes(32)):
        L = self.L = _stream_lib()
        if video is not None and video.batch != image.batch:
            raise UfbError(-1, "image and video codec batches differ")
        self.image, self.video, self.batch = image, video, image.batch
        self._ids = (bytes(image_identity), bytes(video_identity))
        self.h = L.ufb_stream_codec_create(image.h, video.h if video is not None else None, self._ids[0],
                                           self._ids[1])
        if not self.h:
            raise UfbError(-1, L.ufb_last_error().decode())

    def __del__(self):
        if getattr(self, "h", None):
            self.L.ufb_stream_codec_destroy(self.h)
            self.h = None

    def encode(self, frames_u8, width, height, qp_i, qp_p, reset_interval=0, intra_period=-1):
        """frames_u8: uint8 YUV444 [B, T, 3, height, width].  Returns (list of B
        bitstreams, packet count)."""
        x = _c(frames_u8, _np.uint8)
        if x.ndim != 5 or x.shape[0] != self.batch or x.shape[2:] != (3, height, width):
            raise UfbError(-1, f"frames must be [{self.batch}, T, 3, {height}, {width}] uint8")
        cap = 4096 + 4 * x[0].size
        out = _np.empty(self.batch * cap, _np.uint8)
        lens = (C.c_size_t * self.batch)()
        packets = C.c_uint64()
        _check(self.L.ufb_stream_encode(self.h, x.ctypes.data, x.shape[1], width, height, qp_i, qp_p,
                                        reset_interval, intra_period, out.ctypes.data, cap, lens,
                                        C.byref(packets)))
        return [out[i * cap: i * cap + lens[i]].tobytes() for i in range(self.batch)], packets.value

    def decode(self, streams, total_frames, total_packets, width=0, height=0, sink=None):
        """Decode B streams; sink(stream, frame, yuv_bytes) receives every frame.
        Returns {"frames", "packets", "sha256": [hex digest per stream]}."""
        if len(streams) != self.batch:
            raise UfbError(-1, f"{self.batch} streams required")
        bufs = [_buf(s) for s in streams]
        ptrs = (C.c_void_p * self.batch)(*[p for _, p in bufs])
        lens = (C.c_size_t * self.batch)(*[len(s) for s in streams])
        digest = (C.c_uint8 * (32 * self.batch))()
        frames, packets = C.c_uint64(), C.c_uint64()
        errors = []

        def forward(_user, stream, frame, yuv, n):
            try:
                sink(stream, frame, C.string_at(yuv, n))
            except Exception as e:  # noqa: BLE001 -- re-raised after the C call returns
                errors.append(e)

        cb = FRAME_SINK(forward) if sink is not None else FRAME_SINK()
        rc = self.L.ufb_stream_decode(self.h, ptrs, lens, total_frames, total_packets, width, height, cb, None,
                                      digest, C.byref(frames), C.byref(packets))
        if errors:
            raise errors[0]
        _check(rc)
        d = bytes(digest)
        return {"frames": frames.value, "packets": packets.value,
                "sha256": [d[32 * b: 32 * b + 32].hex() for b in range(self.batch)]}
