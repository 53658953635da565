"""GPU: ufb_conv2d_noalloc -- the convolution entry point for callers that
cannot allocate GPU memory while they run (a host application that owns all
device memory, a real-time loop where an allocation could stall or fail) --
gives exactly what ufb_conv2d gives, through the C ABI, on two calls in a row
that share its fixed scratch array.  This file is collected last so a failure
here never hides another test's result."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _noalloc(lib):
    f = lib.ufb_conv2d_noalloc
    f.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int,
                  C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    f.restype = C.c_int
    return f


def _call(fn, x, w, b, bits, pad, out, stream):
    n, ci, h, wd = x.shape
    co, _, kh, kw = w.shape
    return fn(x.data_ptr(), n, ci, h, wd, w.data_ptr(), co, kh, kw, b.data_ptr() if b is not None else None, bits,
              1, 1, pad, pad, 1, out.data_ptr(), stream)


def test_noalloc_matches_conv2d_twice(ufb, dev):
    lib = ufb.library()
    noalloc = _noalloc(lib)
    stream = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    rng = np.random.default_rng(2024)
    cases = [  # two calls in a row with different shapes: the second reuses the first's scratch
        ((1, 64, 88, 160), (64, 64, 3, 3), np.int32, 1),   # BASELINE config-1 shape, int32 bias
        ((2, 192, 20, 36), (80, 192, 1, 1), np.int16, 0),  # 1x1, channel tails
    ]
    for xs, ws, bdt, pad in cases:
        x = torch.from_numpy(rng.integers(-32768, 32768, xs).astype(np.int16)).to(dev)
        w = torch.from_numpy(rng.integers(-32768, 32768, ws).astype(np.int16)).to(dev)
        b = torch.from_numpy(rng.integers(-(1 << 16), 1 << 16, ws[0]).astype(bdt)).to(dev)
        bits = 32 if bdt == np.int32 else 16
        oh, ow = xs[2] + 2 * pad - ws[2] + 1, xs[3] + 2 * pad - ws[3] + 1
        want = torch.empty((xs[0], ws[0], oh, ow), dtype=torch.int16, device=dev)
        got = torch.full_like(want, 12345)
        assert _call(lib.ufb_conv2d, x, w, b, bits, pad, want, stream) == 0, lib.ufb_last_error()
        assert _call(noalloc, x, w, b, bits, pad, got, stream) == 0, lib.ufb_last_error()
        torch.cuda.synchronize(dev)
        # integer arithmetic: the tolerance is exact equality
        assert torch.equal(got, want)
    assert ufb.device_status(dev.index or 0) == 0


def test_noalloc_rejects_oversized_staging(ufb, dev):
    lib = ufb.library()
    noalloc = _noalloc(lib)
    stream = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    x = torch.zeros((4, 512, 64, 64), dtype=torch.int16, device=dev)  # 16 MiB of split input alone
    w = torch.zeros((512, 512, 1, 1), dtype=torch.int16, device=dev)
    out = torch.empty((4, 512, 64, 64), dtype=torch.int16, device=dev)
    rc = _call(noalloc, x, w, None, 0, 0, out, stream)
    assert rc == -2
    assert b"UFB_NOALLOC_SCRATCH_BYTES" in lib.ufb_last_error()
