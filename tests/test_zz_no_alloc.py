"""GPU: ufb_conv2d_noalloc -- the convolution entry point for callers that
cannot allocate GPU memory while they run (a host application that owns all
device memory, a real-time loop where an allocation could stall or fail) --
gives exactly what ufb_conv2d gives, through the C ABI, on two calls in a row
that share its fixed scratch array.  This file is collected last so a failure
here never hides another test's result."""
import ctypes as C
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _noalloc(lib):
    f = lib.ufb_conv2d_noalloc
    f.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int,
                  C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    f.restype = C.c_int
    return f


def _call(fn, x, w, b, bits, pad, out, stream, stride=1, groups=1):
    n, ci, h, wd = x.shape
    co, _, kh, kw = w.shape
    return fn(x.data_ptr(), n, ci, h, wd, w.data_ptr(), co, kh, kw, b.data_ptr() if b is not None else None, bits,
              stride, stride, pad, pad, groups, out.data_ptr(), stream)


# (x shape, w shape, bias dtype or None, pad, stride, groups)
CASES = [
    ((1, 64, 88, 160), (64, 64, 3, 3), np.int32, 1, 1, 1),   # config-1 shape, int32 bias (tensor cores)
    ((2, 192, 20, 36), (80, 192, 1, 1), np.int16, 0, 1, 1),  # 1x1 with channel tails (tensor cores)
    ((1, 48, 30, 34), (40, 48, 3, 3), None, 1, 1, 1),        # no bias (tensor cores)
    ((1, 32, 31, 45), (24, 32, 3, 3), np.int16, 1, 2, 1),    # stride 2 (direct kernel)
    ((2, 64, 20, 28), (64, 1, 3, 3), np.int16, 1, 1, 64),    # depthwise 3x3, int16 bias (direct kernel)
]


def _run_pair(lib, noalloc, dev, rng, case, stream):
    xs, ws, bdt, pad, stride, groups = case
    x = torch.from_numpy(rng.integers(-32768, 32768, xs).astype(np.int16)).to(dev)
    w = torch.from_numpy(rng.integers(-32768, 32768, ws).astype(np.int16)).to(dev)
    b = None if bdt is None else torch.from_numpy(rng.integers(-(1 << 16), 1 << 16, ws[0]).astype(bdt)).to(dev)
    bits = 0 if bdt is None else (32 if bdt == np.int32 else 16)
    oh = (xs[2] + 2 * pad - ws[2]) // stride + 1
    ow = (xs[3] + 2 * pad - ws[3]) // stride + 1
    want = torch.empty((xs[0], ws[0], oh, ow), dtype=torch.int16, device=dev)
    got = torch.full_like(want, 12345)
    assert _call(noalloc, x, w, b, bits, pad, got, stream, stride, groups) == 0, lib.ufb_last_error()
    assert _call(lib.ufb_conv2d, x, w, b, bits, pad, want, stream, stride, groups) == 0, lib.ufb_last_error()
    torch.cuda.synchronize(dev)
    return got, want


def test_noalloc_matches_conv2d_twice(ufb, dev):
    lib = ufb.library()
    noalloc = _noalloc(lib)
    stream = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    rng = np.random.default_rng(2024)
    # each shape runs twice in a row: the second call reuses the scratch the
    # first one left behind, and consecutive shapes overwrite each other's
    for case in CASES:
        for _ in range(2):
            got, want = _run_pair(lib, noalloc, dev, rng, case, stream)
            # integer arithmetic: the tolerance is exact equality
            assert torch.equal(got, want), case
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


_FIRST_CALL = r"""
import ctypes as C, os, sys
import numpy as np, torch
sys.path.insert(0, os.environ["UFB_ROOT"])
import __graft_entry__ as entry
sys.path.insert(0, os.path.join(os.environ["UFB_ROOT"], "tests"))
from test_zz_no_alloc import CASES, _noalloc, _run_pair
ufb = entry.load_package()
dev = torch.device("cuda:0")
lib = ufb.library()
stream = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
rng = np.random.default_rng(7)
# the first library call in this process is ufb_conv2d_noalloc (inside _run_pair)
for case in (CASES[0], CASES[0]):
    got, want = _run_pair(lib, _noalloc(lib), dev, rng, case, stream)
    assert torch.equal(got, want)
assert ufb.device_status(0) == 0
print("first-call ok")
"""


def test_noalloc_as_first_call_in_fresh_process(dev):
    """In a new process the no-allocation entry point is the library's first
    call on the device: it sets up its scratch address and the status word the
    pipeline reports timeouts through without allocating, then matches
    ufb_conv2d on two calls in a row."""
    env = dict(os.environ, UFB_ROOT=ROOT)
    r = subprocess.run([sys.executable, "-c", _FIRST_CALL], capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "first-call ok" in r.stdout
