"""TEST INFRASTRUCTURE ONLY: ctypes bindings for the two CPU checkers.

* ``C``   -- ``_build/libuforacle.so``: this repository's plain-C restatement of
  the reference INT16 arithmetic (``uf_oracle.c``).
* ``Ref`` -- ``_ref/libufref.so``: the reference's own CPU INT16 path
  (``src/int16_ops.cpp``, ``src/layers.cpp``, ``src/integer_model.cpp``,
  ``src/entropy.cpp``) and UF16 container (``src/bitstream.cpp``) compiled from
  its sources by ``Makefile`` target ``ref``, wrapped by ``ref_shim.cpp``.
* ``stream`` -- restatements in Python of the stream-level loops over the
  compiled reference models (``uf::IntegerCodec``) and of the prepared-model
  identity.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU arm may
import this package; the product library never links or calls it.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
C_LIB_PATH = os.path.join(HERE, "_build", "libuforacle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libufref.so")

_i16p = np.ctypeslib.ndpointer(np.int16, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")

DTYPE_CODES = {np.dtype(np.int16): 0, np.dtype(np.uint8): 1, np.dtype(np.int32): 2,
               np.dtype(np.int8): 3, np.dtype(np.int64): 4}


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def conv_out_hw(h, w, kh, kw, sh, sw, ph, pw):
    return (h + 2 * ph - kh) // sh + 1, (w + 2 * pw - kw) // sw + 1


class COracle:
    """The plain-C restatement (uf_oracle.c)."""

    def __init__(self, path: str = C_LIB_PATH):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run make -C oracle")
        L = self.lib = C.CDLL(path)
        L.ufo_divide_round.restype = C.c_int64
        L.ufo_divide_round.argtypes = [C.c_int64, C.c_int64]
        L.ufo_conv2d.argtypes = [_i16p, C.c_int64, C.c_int64, C.c_int64, C.c_int64, _i16p, C.c_int64,
                                 C.c_int64, C.c_int64, C.c_void_p, C.c_int, C.c_int64, C.c_int64,
                                 C.c_int64, C.c_int64, C.c_int64, _i16p]
        L.ufo_add.argtypes = [C.c_int, C.POINTER(C.c_void_p), C.c_int64, _i16p]
        L.ufo_multiply.argtypes = [_i16p, _i64p, _i16p, _i64p, _i16p]
        L.ufo_lookup_i16.argtypes = [_i16p, C.c_int64, _i16p, _i16p]
        L.ufo_lookup_u8.argtypes = [_i16p, C.c_int64, _u8p, _u8p]
        L.ufo_wsilu4.argtypes = [_i16p, C.c_int64, C.c_int64, C.c_int64, _i16p, _i16p]
        L.ufo_from_bytes.argtypes = [_u8p, C.c_int64, _i16p]
        L.ufo_symbols.argtypes = [_i16p, C.c_int64, _i8p]
        L.ufo_from_symbols.argtypes = [_i8p, C.c_int64, _i16p]
        L.ufo_reciprocal.argtypes = [_i16p, C.c_int64, _i16p]
        L.ufo_pixel_shuffle.argtypes = [_i16p, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int64,
                                        C.c_int, _i16p]
        L.ufo_raw_frame.argtypes = [_i16p, C.c_int64, C.c_int64, C.c_int64, C.c_int64, _u8p]
        L.ufo_warp.argtypes = [_i16p, _i16p, C.c_int64, C.c_int64, C.c_int64, C.c_int64, _i16p]
        L.ufo_warp_float.argtypes = [_i16p, _i16p, C.c_int64, C.c_int64, C.c_int64, C.c_int64, _f32p]

    def divide_round(self, v, d):
        return int(self.lib.ufo_divide_round(int(v), int(d)))

    def conv2d(self, x, w, bias=None, stride=1, padding=0, groups=1):
        x, w = _c(x, np.int16), _c(w, np.int16)
        n, ci, h, wd = x.shape
        co, _, kh, kw = w.shape
        oh, ow = conv_out_hw(h, wd, kh, kw, stride, stride, padding, padding)
        out = np.empty((n, co, oh, ow), np.int16)
        bits, bp = 0, None
        if bias is not None:
            bias = np.ascontiguousarray(bias)
            bits = 32 if bias.dtype == np.int32 else 16
            bias = _c(bias, np.int32 if bits == 32 else np.int16)
            bp = bias.ctypes.data
        rc = self.lib.ufo_conv2d(x, n, ci, h, wd, w, co, kh, kw, bp, bits, stride, stride, padding,
                                 padding, groups, out)
        if rc:
            raise ValueError(f"ufo_conv2d failed ({rc})")
        return out

    def add(self, *values):
        vs = [_c(v, np.int16) for v in values]
        arr = (C.c_void_p * len(vs))(*[v.ctypes.data for v in vs])
        out = np.empty_like(vs[0])
        self.lib.ufo_add(len(vs), arr, vs[0].size, out)
        return out

    def multiply(self, x, scale):
        x, s = _c(x, np.int16), _c(scale, np.int16)
        out = np.empty_like(x)
        if self.lib.ufo_multiply(x, _c(x.shape, np.int64), s, _c(s.shape, np.int64), out):
            raise ValueError("invalid broadcast")
        return out

    def lookup(self, x, table):
        x = _c(x, np.int16)
        if table.dtype == np.uint8:
            out = np.empty(x.shape, np.uint8)
            self.lib.ufo_lookup_u8(x, x.size, _c(table, np.uint8), out)
        else:
            out = np.empty(x.shape, np.int16)
            self.lib.ufo_lookup_i16(x, x.size, _c(table, np.int16), out)
        return out

    def wsilu4(self, x, table):
        x = _c(x, np.int16)
        n, c4, h, w = x.shape
        out = np.empty((n, c4 // 4, h, w), np.int16)
        if self.lib.ufo_wsilu4(x, n, c4, h * w, _c(table, np.int16), out):
            raise ValueError("channels not divisible by four")
        return out

    def from_bytes(self, x):
        x = _c(x, np.uint8)
        out = np.empty(x.shape, np.int16)
        self.lib.ufo_from_bytes(x, x.size, out)
        return out

    def symbols(self, x):
        x = _c(x, np.int16)
        out = np.empty(x.shape, np.int8)
        self.lib.ufo_symbols(x, x.size, out)
        return out

    def from_symbols(self, x):
        x = _c(x, np.int8)
        out = np.empty(x.shape, np.int16)
        self.lib.ufo_from_symbols(x, x.size, out)
        return out

    def reciprocal(self, x):
        x = _c(x, np.int16)
        out = np.empty(x.shape, np.int16)
        self.lib.ufo_reciprocal(x, x.size, out)
        return out

    def pixel_shuffle(self, x, f):
        x = _c(x, np.int16)
        n, c, h, w = x.shape
        out = np.empty((n, c // (f * f), h * f, w * f), np.int16)
        if self.lib.ufo_pixel_shuffle(x, n, c, h, w, f, 0, out):
            raise ValueError("bad shuffle")
        return out

    def pixel_unshuffle(self, x, f):
        x = _c(x, np.int16)
        n, c, h, w = x.shape
        out = np.empty((n, c * f * f, h // f, w // f), np.int16)
        if self.lib.ufo_pixel_shuffle(x, n, c, h, w, f, 1, out):
            raise ValueError("bad unshuffle")
        return out

    def raw_frame(self, frame, height, width):
        """frame: int16 [3, h, w] (or [1, 3, h, w]) -> YUV420 bytes."""
        f = _c(frame, np.int16).reshape(3, frame.shape[-2], frame.shape[-1])
        out = np.empty(height * width * 3 // 2, np.uint8)
        if self.lib.ufo_raw_frame(f, f.shape[1], f.shape[2], height, width, out):
            raise ValueError("bad raw frame geometry")
        return out

    def warp(self, feature, flow):
        feature, flow = _c(feature, np.int16), _c(flow, np.int16)
        n, c, h, w = feature.shape
        out = np.empty_like(feature)
        self.lib.ufo_warp(feature, flow, n, c, h, w, out)
        return out

    def warp_float(self, feature, flow):
        feature, flow = _c(feature, np.int16), _c(flow, np.int16)
        n, c, h, w = feature.shape
        out = np.empty(feature.shape, np.float32)
        self.lib.ufo_warp_float(feature, flow, n, c, h, w, out)
        return out


class RefError(RuntimeError):
    pass


class RefOracle:
    """The reference's own CPU INT16 path, compiled from its sources."""

    def __init__(self, path: str = REF_LIB_PATH):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run make -C oracle ref REF_ROOT=<reference>")
        L = self.lib = C.CDLL(path)
        L.ufref_last_error.restype = C.c_char_p
        L.ufref_conv2d.argtypes = [_i16p, _i64p, _i16p, _i64p, C.c_void_p, C.c_int, C.c_int64, C.c_int64,
                                   C.c_int64, C.c_int64, C.c_int64, _i16p, C.c_int64, _i64p]
        L.ufref_add.argtypes = [C.c_int, C.POINTER(C.c_void_p), C.c_int64, _i16p]
        L.ufref_multiply.argtypes = [_i16p, _i64p, _i16p, _i64p, _i16p]
        L.ufref_lookup.argtypes = [_i16p, C.c_int64, C.c_void_p, C.c_int, C.c_void_p]
        L.ufref_wsilu4.argtypes = [_i16p, _i64p, _i16p, _i16p]
        L.ufref_from_bytes.argtypes = [_u8p, C.c_int64, _i16p]
        L.ufref_divide_round.argtypes = [_i64p, C.c_int64, C.c_int64, _i64p]
        L.ufref_symbols.argtypes = [_i16p, C.c_int64, _i8p]
        L.ufref_reciprocal.argtypes = [_i16p, C.c_int64, _i16p]
        L.ufref_pixel_shuffle.argtypes = [_i16p, _i64p, C.c_int64, C.c_int, _i16p, _i64p]
        L.ufref_model_new.restype = C.c_void_p
        L.ufref_model_new.argtypes = [C.c_char_p, C.c_int, C.POINTER(C.c_char_p), C.POINTER(C.c_int),
                                      C.POINTER(C.c_int), C.POINTER(C.c_int64), C.POINTER(C.c_void_p)]
        L.ufref_model_free.argtypes = [C.c_void_p]
        L.ufref_model_set_skip.argtypes = [C.c_void_p, C.c_double]
        L.ufref_model_clear_dpb.argtypes = [C.c_void_p]
        L.ufref_model_add_ref.argtypes = [C.c_void_p, _i16p, _i64p]
        L.ufref_model_compress.argtypes = [C.c_void_p, _i16p, _i64p, C.c_int, C.c_int]
        L.ufref_model_decompress.argtypes = [C.c_void_p, _u8p, C.c_int64, C.c_uint32, C.c_uint32,
                                             C.c_int, C.c_int]
        L.ufref_model_payload.restype = C.c_int64
        L.ufref_model_payload.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
        L.ufref_model_frame_count.argtypes = [C.c_void_p]
        L.ufref_model_frame.argtypes = [C.c_void_p, C.c_int, _i16p, C.c_int64, _i64p]
        L.ufref_model_state.argtypes = [C.c_void_p, C.c_int, _i16p, C.c_int64, _i64p]
        L.ufref_layers_run.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.POINTER(C.c_void_p), _i64p,
                                       _i16p, C.c_int64, _i64p]
        L.ufref_layers_parameter.argtypes = [C.c_void_p, C.c_char_p, C.c_int64, _i16p, C.c_int64, _i64p]
        L.ufref_layers_reconstruct.argtypes = [C.c_void_p, _i16p, _i64p, C.c_int, C.c_int, _i16p,
                                               C.c_int64, _i64p]
        L.ufref_rans_new.restype = C.c_void_p
        L.ufref_rans_new.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p, C.c_int64,
                                     C.c_int64, C.c_void_p]
        L.ufref_rans_free.argtypes = [C.c_void_p]
        L.ufref_rans_reset.argtypes = [C.c_void_p]
        L.ufref_rans_encode_y.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
        L.ufref_rans_encode_z.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_int, C.c_int]
        L.ufref_rans_flush.restype = C.c_int64
        L.ufref_rans_flush.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
        L.ufref_rans_set_stream.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
        L.ufref_rans_decode_z.argtypes = [C.c_void_p, C.c_int64, C.c_int, C.c_int, C.c_void_p]
        L.ufref_rans_decode_y.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]
        for name, args in (("ufref_bs_write_uint", [C.c_uint32, C.c_void_p, C.c_int64]),
                           ("ufref_bs_write_preamble", [C.c_char_p, C.c_char_p, C.c_void_p, C.c_int64]),
                           ("ufref_bs_write_sps", [C.c_int, C.c_uint32, C.c_uint32, C.c_void_p, C.c_int64]),
                           ("ufref_bs_write_packet", [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_char_p,
                                                      C.c_int64, C.c_void_p, C.c_int64])):
            getattr(L, name).restype = C.c_int64
            getattr(L, name).argtypes = args
        L.ufref_bs_scan.argtypes = [C.c_char_p, C.c_int64, C.c_char_p, C.c_int64, _i64p, _u8p]
        table = [C.c_char_p, C.c_int, C.POINTER(C.c_char_p), C.POINTER(C.c_int), C.POINTER(C.c_int),
                 C.POINTER(C.c_int64), C.POINTER(C.c_void_p)]
        L.ufref_codec_new.restype = C.c_void_p
        L.ufref_codec_new.argtypes = [C.c_char_p, C.c_double, C.c_int] + table + table
        L.ufref_codec_free.argtypes = [C.c_void_p]
        L.ufref_codec_encode.argtypes = [C.c_void_p, _u8p, C.c_int64, C.c_uint32, C.c_uint32, C.c_int, C.c_int,
                                         C.c_int, C.c_int, C.c_char_p, _i64p]
        L.ufref_codec_decode.argtypes = [C.c_void_p, C.c_char_p, C.c_int64, C.c_int64, C.c_int64, C.c_char_p,
                                         C.c_void_p, C.c_int64, _i64p]
        L.ufref_raw_frame.restype = C.c_int64
        L.ufref_raw_frame.argtypes = [_i16p, _i64p, C.c_int64, C.c_int64, _u8p, C.c_int64]
        L.ufref_bs_parse.argtypes = [C.c_char_p, C.c_int64, _i64p, _i64p, C.c_int64, _i64p, _u8p, C.c_int64]

    def _check(self, rc):
        if rc < 0:
            raise RefError(self.lib.ufref_last_error().decode())
        return rc

    def set_threads(self, n):
        self._check(self.lib.ufref_set_threads(int(n)))

    def conv2d(self, x, w, bias=None, stride=1, padding=0, groups=1):
        x, w = _c(x, np.int16), _c(w, np.int16)
        oh, ow = conv_out_hw(x.shape[2], x.shape[3], w.shape[2], w.shape[3], stride, stride, padding, padding)
        out = np.empty((x.shape[0], w.shape[0], max(oh, 0), max(ow, 0)), np.int16)
        shape = np.zeros(4, np.int64)
        bp, code = None, 0
        if bias is not None:
            bias = np.ascontiguousarray(bias)
            code = DTYPE_CODES[bias.dtype]
            bp = bias.ctypes.data
        self._check(self.lib.ufref_conv2d(x, _c(x.shape, np.int64), w, _c(w.shape, np.int64), bp, code,
                                          stride, stride, padding, padding, groups, out, out.size, shape))
        return out

    def add(self, *values):
        vs = [_c(v, np.int16) for v in values]
        arr = (C.c_void_p * len(vs))(*[v.ctypes.data for v in vs])
        out = np.empty_like(vs[0])
        self._check(self.lib.ufref_add(len(vs), arr, vs[0].size, out))
        return out

    def multiply(self, x, scale):
        x, s = _c(x, np.int16), _c(scale, np.int16)
        out = np.empty_like(x)
        self._check(self.lib.ufref_multiply(x, _c(x.shape, np.int64), s, _c(s.shape, np.int64), out))
        return out

    def lookup(self, x, table):
        x = _c(x, np.int16)
        table = np.ascontiguousarray(table)
        out = np.empty(x.shape, table.dtype)
        self._check(self.lib.ufref_lookup(x, x.size, table.ctypes.data, DTYPE_CODES[table.dtype], out.ctypes.data))
        return out

    def wsilu4(self, x, table):
        x = _c(x, np.int16)
        out = np.empty((x.shape[0], x.shape[1] // 4) + x.shape[2:], np.int16)
        self._check(self.lib.ufref_wsilu4(x, _c(x.shape, np.int64), _c(table, np.int16), out))
        return out

    def from_bytes(self, x):
        x = _c(x, np.uint8)
        out = np.empty(x.shape, np.int16)
        self._check(self.lib.ufref_from_bytes(x, x.size, out))
        return out

    def divide_round(self, x, d):
        x = _c(x, np.int64)
        out = np.empty_like(x)
        self._check(self.lib.ufref_divide_round(x, x.size, d, out))
        return out

    def symbols(self, x):
        x = _c(x, np.int16)
        out = np.empty(x.shape, np.int8)
        self._check(self.lib.ufref_symbols(x, x.size, out))
        return out

    def reciprocal(self, x):
        x = _c(x, np.int16)
        out = np.empty(x.shape, np.int16)
        self._check(self.lib.ufref_reciprocal(x, x.size, out))
        return out

    def pixel_shuffle(self, x, f, unshuffle=False):
        x = _c(x, np.int16)
        out = np.empty(x.size, np.int16)
        shape = np.zeros(4, np.int64)
        self._check(self.lib.ufref_pixel_shuffle(x, _c(x.shape, np.int64), f, int(unshuffle), out, shape))
        return out.reshape(tuple(int(s) for s in shape))

    def model(self, variant, tensors):
        return RefModel(self, variant, tensors)

    # ---- UF16 container: uf::write_* / read_* / scan_bitstream (src/bitstream.cpp) ----

    def _written(self, n, out):
        self._check(n)
        return bytes(out[:n])

    def bs_write_uint(self, v):
        out = (C.c_uint8 * 8)()
        return self._written(self.lib.ufref_bs_write_uint(v, out, 8), out)

    def bs_write_preamble(self, image_identity, video_identity):
        out = (C.c_uint8 * 72)()
        return self._written(self.lib.ufref_bs_write_preamble(bytes(image_identity), bytes(video_identity), out, 72),
                             out)

    def bs_write_sps(self, sps_id, width, height):
        out = (C.c_uint8 * 16)()
        return self._written(self.lib.ufref_bs_write_sps(sps_id, width, height, out, 16), out)

    def bs_write_packet(self, nal_type, sps_id, qp, entropy_parallel, reset, payload):
        cap = len(payload) + 16
        out = (C.c_uint8 * cap)()
        return self._written(self.lib.ufref_bs_write_packet(nal_type, sps_id, qp, entropy_parallel, int(bool(reset)),
                                                            bytes(payload), len(payload), out, cap), out)

    def bs_scan(self, data, variant, expected_frames=None):
        summary, ids = np.zeros(7, np.int64), np.zeros(64, np.uint8)
        self._check(self.lib.ufref_bs_scan(bytes(data), len(data), variant.encode(),
                                           -1 if expected_frames is None else int(expected_frames), summary, ids))
        keys = ("integer", "width", "height", "packets", "intra_packets", "predicted_packets", "maximum_frames")
        out = {k: int(v) for k, v in zip(keys, summary)}
        out["integer"] = bool(out["integer"])
        out["image_identity"], out["video_identity"] = ids[:32].tobytes(), ids[32:].tobytes()
        return out

    def bs_parse(self, data, max_units=4096):
        """read_preamble, then every NAL unit: (integer, [unit dicts])."""
        integer, units = np.zeros(1, np.int64), np.zeros(1, np.int64)
        records = np.zeros(7 * max_units, np.int64)
        payloads = np.zeros(max(len(data), 1), np.uint8)
        self._check(self.lib.ufref_bs_parse(bytes(data), len(data), integer, records, max_units, units, payloads,
                                            payloads.size))
        out, used = [], 0
        for r in records[: 7 * int(units[0])].reshape(-1, 7):
            t, sid, w, h, qp, flags, n = (int(v) for v in r)
            if t == 0:
                out.append({"type": 0, "sps_id": sid, "width": w, "height": h})
            else:
                out.append({"type": t, "sps_id": sid, "qp": qp, "entropy_parallel": flags >> 1,
                            "reset": bool(flags & 1), "payload": payloads[used: used + n].tobytes()})
                used += n
        return bool(integer[0]), out

    def rans(self, tables):
        return RefRans(self, tables)

    def codec(self, image_tensors, image_identity_hex, video_tensors=None, video_identity_hex="",
              variant="htl", skip_threshold=0.0, threads=0):
        return RefCodec(self, image_tensors, image_identity_hex, video_tensors, video_identity_hex, variant,
                        skip_threshold, threads)

    def raw_frame(self, frame, height, width):
        """uf::IntegerCodec::raw_frame (src/integer_codec.cpp:294-323): int16
        [1, 3, fh, fw] (or [3, fh, fw]) -> YUV420 bytes of width x height."""
        frame = _c(frame, np.int16)
        if frame.ndim == 3:
            frame = frame[None]
        cap = width * height + 2 * ((height + 1) // 2) * ((width + 1) // 2)
        out = np.empty(max(cap, 1), np.uint8)
        n = self._check(self.lib.ufref_raw_frame(frame, _c(frame.shape, np.int64), width, height, out, out.size))
        return out[:n].copy()


class RefModel:
    """uf::IntegerModel + uf::Layers on torch::kCPU."""

    def __init__(self, ref: RefOracle, variant: str, tensors: dict):
        self.ref, L = ref, ref.lib
        names = sorted(tensors)
        arrays = [np.ascontiguousarray(tensors[n]) for n in names]
        self._keep = arrays
        c_names = (C.c_char_p * len(names))(*[n.encode() for n in names])
        dtypes = (C.c_int * len(names))(*[DTYPE_CODES[a.dtype] for a in arrays])
        ndims = (C.c_int * len(names))(*[a.ndim for a in arrays])
        flat = [int(s) for a in arrays for s in a.shape]
        shapes = (C.c_int64 * max(len(flat), 1))(*flat)
        data = (C.c_void_p * len(names))(*[a.ctypes.data for a in arrays])
        self.h = L.ufref_model_new(variant.encode(), len(names), c_names, dtypes, ndims, shapes, data)
        if not self.h:
            raise RefError(L.ufref_last_error().decode())
        self._keep = None

    def __del__(self):
        if getattr(self, "h", None):
            self.ref.lib.ufref_model_free(self.h)
            self.h = None

    def _check(self, rc):
        return self.ref._check(rc)

    def set_skip_threshold(self, t):
        self._check(self.ref.lib.ufref_model_set_skip(self.h, float(t)))

    def clear_dpb(self):
        self._check(self.ref.lib.ufref_model_clear_dpb(self.h))

    def add_ref_feature_from_frame(self, frame):
        frame = _c(frame, np.int16)
        self._check(self.ref.lib.ufref_model_add_ref(self.h, frame, _c(frame.shape, np.int64)))

    def _frames(self):
        L = self.ref.lib
        out = []
        for i in range(L.ufref_model_frame_count(self.h)):
            buf = np.empty(1 << 26, np.int16)
            shape = np.zeros(4, np.int64)
            self._check(L.ufref_model_frame(self.h, i, buf, buf.size, shape))
            out.append(buf[: int(np.prod(shape))].reshape(tuple(int(s) for s in shape)).copy())
        return out

    def compress(self, frames, qp, reset=False):
        frames = _c(frames, np.int16)
        L = self.ref.lib
        self._check(L.ufref_model_compress(self.h, frames, _c(frames.shape, np.int64), int(qp), int(reset)))
        n = L.ufref_model_payload(self.h, None, 0)
        payload = np.empty(n, np.uint8)
        L.ufref_model_payload(self.h, payload.ctypes.data, n)
        return payload.tobytes(), self._frames()

    def decompress(self, payload: bytes, width, height, qp, reset=False):
        buf = np.frombuffer(payload, np.uint8).copy()
        self._check(self.ref.lib.ufref_model_decompress(self.h, buf, buf.size, width, height, int(qp), int(reset)))
        return self._frames()

    def state(self, which):
        idx = {"reference": 0, "memory": 1, "context": 2}[which]
        buf = np.empty(1 << 26, np.int16)
        shape = np.zeros(4, np.int64)
        rc = self._check(self.ref.lib.ufref_model_state(self.h, idx, buf, buf.size, shape))
        if rc == 1:
            return None
        return buf[: int(np.prod(shape))].reshape(tuple(int(s) for s in shape)).copy()

    def run(self, module, *args):
        vs = [_c(a, np.int16) for a in args]
        arr = (C.c_void_p * len(vs))(*[v.ctypes.data for v in vs])
        shapes = _c([s for v in vs for s in v.shape], np.int64)
        buf = np.empty(1 << 26, np.int16)
        shape = np.zeros(4, np.int64)
        self._check(self.ref.lib.ufref_layers_run(self.h, module.encode(), len(vs), arr, shapes, buf,
                                                  buf.size, shape))
        return buf[: int(np.prod(shape))].reshape(tuple(int(s) for s in shape)).copy()

    def parameter(self, name, qp):
        buf = np.empty(1 << 20, np.int16)
        shape = np.zeros(4, np.int64)
        self._check(self.ref.lib.ufref_layers_parameter(self.h, name.encode(), qp, buf, buf.size, shape))
        return buf[: int(np.prod(shape))].reshape(tuple(int(s) for s in shape)).copy()


def _tensor_table(tensors: dict):
    names = sorted(tensors)
    arrays = [np.ascontiguousarray(tensors[n]) for n in names]
    flat = [int(s) for a in arrays for s in a.shape]
    return (arrays,
            (C.c_char_p * len(names))(*[n.encode() for n in names]),
            (C.c_int * len(names))(*[DTYPE_CODES[a.dtype] for a in arrays]),
            (C.c_int * len(names))(*[a.ndim for a in arrays]),
            (C.c_int64 * max(len(flat), 1))(*flat),
            (C.c_void_p * len(names))(*[a.ctypes.data for a in arrays]))


class RefCodec:
    """uf::IntegerCodec on torch::kCPU (src/integer_codec.cpp): the reference's
    own stream encode loop and decode loop (decoded-YUV SHA-256, raw frames)."""

    def __init__(self, ref: RefOracle, image_tensors, image_identity_hex, video_tensors, video_identity_hex,
                 variant, skip_threshold, threads):
        self.ref, L = ref, ref.lib
        img = _tensor_table(image_tensors)
        if video_tensors is not None:
            vid = _tensor_table(video_tensors)
            vargs = [video_identity_hex.encode(), len(vid[0])] + list(vid[1:])
        else:
            vargs = [b"", -1, None, None, None, None, None]
        self.h = L.ufref_codec_new(variant.encode(), float(skip_threshold), int(threads),
                                   image_identity_hex.encode(), len(img[0]), *img[1:], *vargs)
        if not self.h:
            raise RefError(L.ufref_last_error().decode())

    def __del__(self):
        if getattr(self, "h", None):
            self.ref.lib.ufref_codec_free(self.h)
            self.h = None

    def encode(self, frames_u8, width, height, qp_i, qp_p, reset_interval=32, intra_period=-1):
        """frames_u8: [T, 3, height, width] uint8 YUV444 -> (archive bytes, frames, packets)."""
        import tempfile
        frames_u8 = _c(frames_u8, np.uint8)
        stats = np.zeros(2, np.int64)
        with tempfile.TemporaryDirectory() as d:
            path = os.path.join(d, "video.bin")
            self.ref._check(self.ref.lib.ufref_codec_encode(self.h, frames_u8, frames_u8.shape[0], width, height,
                                                            qp_i, qp_p, reset_interval, intra_period,
                                                            path.encode(), stats))
            with open(path, "rb") as f:
                data = f.read()
        return data, int(stats[0]), int(stats[1])

    def decode(self, data: bytes, total_frames, total_packets, width=None, height=None):
        """-> (decoded-YUV SHA-256 hex, [raw YUV420 frames] or None, packets)."""
        digest = C.create_string_buffer(65)
        stats = np.zeros(3, np.int64)
        keep = width is not None and height is not None
        frame_bytes = width * height + 2 * (height // 2) * (width // 2) if keep else 0
        yuv = np.empty(max(frame_bytes * total_frames, 1), np.uint8) if keep else None
        self.ref._check(self.ref.lib.ufref_codec_decode(self.h, bytes(data), len(data), total_frames, total_packets,
                                                        digest, yuv.ctypes.data if keep else None,
                                                        yuv.size if keep else 0, stats))
        frames = [yuv[i * frame_bytes:(i + 1) * frame_bytes].copy() for i in range(int(stats[0]))] if keep else None
        return digest.value.decode(), frames, int(stats[1])


class RefRans:
    """uf::EntropyEncoder / uf::EntropyDecoder (src/entropy.cpp)."""

    def __init__(self, ref: RefOracle, tables: dict):
        self.ref, L = ref, ref.lib
        zc = _c(tables["tables.z_cdf"], np.int32)
        zl = _c(tables["tables.z_lengths"], np.int32)
        yc = _c(tables["tables.y_cdf"], np.int32)
        yl = _c(tables["tables.y_lengths"], np.int32)
        self.h = L.ufref_rans_new(zc.ctypes.data, zc.shape[0], zc.shape[1], zl.ctypes.data,
                                  yc.ctypes.data, yc.shape[0], yc.shape[1], yl.ctypes.data)
        if not self.h:
            raise RefError(L.ufref_last_error().decode())

    def __del__(self):
        if getattr(self, "h", None):
            self.ref.lib.ufref_rans_free(self.h)
            self.h = None

    def encode(self, y_parts, z, z_offset, z_channels):
        """Reference encode order (src/integer_model.cpp:325-331): Y parts in
        reverse, then Z, then flush."""
        L, ck = self.ref.lib, self.ref._check
        ck(L.ufref_rans_reset(self.h))
        for part in reversed(y_parts):
            part = _c(part, np.int16)
            if part.size:
                ck(L.ufref_rans_encode_y(self.h, part.ctypes.data, part.size))
        z = _c(z, np.int8)
        ck(L.ufref_rans_encode_z(self.h, z.ctypes.data, z.size, z_offset, z_channels))
        n = L.ufref_rans_flush(self.h, None, 0)
        if n < 0:
            raise RefError(L.ufref_last_error().decode())
        out = np.empty(n, np.uint8)
        L.ufref_rans_flush(self.h, out.ctypes.data, n)
        return out.tobytes()

    def decode(self, payload: bytes, z_count, z_offset, z_channels, y_index_parts):
        L, ck = self.ref.lib, self.ref._check
        buf = np.frombuffer(payload, np.uint8).copy()
        ck(L.ufref_rans_set_stream(self.h, buf.ctypes.data, buf.size))
        z = np.empty(z_count, np.int8)
        ck(L.ufref_rans_decode_z(self.h, z_count, z_offset, z_channels, z.ctypes.data))
        ys = []
        for idx in y_index_parts:
            idx = _c(idx, np.uint8)
            y = np.empty(idx.size, np.int8)
            if idx.size:
                ck(L.ufref_rans_decode_y(self.h, idx.ctypes.data, idx.size, y.ctypes.data))
            ys.append(y)
        return z, ys


_C = None
_REF = None


def c_oracle() -> COracle:
    global _C
    if _C is None:
        _C = COracle()
    return _C


def ref_oracle() -> RefOracle:
    global _REF
    if _REF is None:
        _REF = RefOracle()
    return _REF


def ref_available() -> bool:
    return os.path.exists(REF_LIB_PATH)
