"""Regenerate tests/golden/model_free.npz from the reference's own CPU path.

The inputs are the reference's in-tree known-answer cases
(tests/model_free.cpp:570-621 of the reference): byte conversion over all 256
values, the rna tie cases, the elementwise parity tensor (1x8x7x8,
values (i*331) % 65536 - 32768), the four convolution geometries
{ci, co, k, stride, pad, groups} and the int64-accumulator extremes.  The
expected outputs are produced by running the reference's uf::int16 functions
(compiled from its sources into oracle/_ref/libufref.so by
`make -C oracle ref REF_ROOT=<reference checkout>`).

Run: python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402


def conv_cases():
    cases = []
    for ci, co, k, stride, pad, groups in [(8, 6, 3, 1, 1, 1), (16, 16, 1, 1, 0, 1), (8, 8, 3, 2, 1, 8),
                                           (8, 12, 3, 1, 1, 2)]:
        x = ((np.arange(ci * 56, dtype=np.int64) * 29) % 2048 - 1024).astype(np.int16).reshape(1, ci, 7, 8)
        w = ((np.arange(co * (ci // groups) * k * k, dtype=np.int64) * 37) % 4096 - 2048).astype(np.int16)
        w = w.reshape(co, ci // groups, k, k)
        b = (np.arange(co, dtype=np.int64) * 71 - 200).astype(np.int16)
        cases.append(("conv", (ci, co, k, stride, pad, groups), x, w, b))
    for kernel in (1, 3):
        for sign in (-1, 1):
            x = np.full((1, 32, 5, 5), 32767, np.int16)
            w = np.full((32, 32, kernel, kernel), 32767 if sign == 1 else -32768, np.int16)
            b = np.zeros(32, np.int16)
            cases.append(("extreme", (32, 32, kernel, 1, kernel // 2, 1), x, w, b))
    return cases


def main():
    ref = oracle.ref_oracle()
    out = {}
    bytes_in = np.arange(256, dtype=np.uint8)
    out["bytes_in"] = bytes_in
    out["bytes_out"] = ref.from_bytes(bytes_in)
    ties = np.array([-769, -768, -767, -257, -256, -255, 255, 256, 257, 767, 768, 769], np.int64)
    out["ties_in"] = ties
    out["ties_out"] = ref.divide_round(ties, 512)
    values = ((np.arange(448, dtype=np.int64) * 331) % 65536 - 32768).astype(np.int16).reshape(1, 8, 7, 8)
    other = np.ascontiguousarray(values[..., ::-1])
    scale = np.array([256, 512, 1024, 2048, 128, 257, 700, 32767], np.int16).reshape(1, 8, 1, 1)
    lut = np.arange(-32768, 32768, dtype=np.int64).astype(np.int16)
    out["ew_values"], out["ew_other"], out["ew_scale"], out["ew_lut"] = values, other, scale, lut
    out["ew_add"] = ref.add(values, other)
    out["ew_mul"] = ref.multiply(values, scale)
    out["ew_lookup"] = ref.lookup(values, lut)
    out["ew_wsilu4"] = ref.wsilu4(values, lut)
    for i, (kind, geom, x, w, b) in enumerate(conv_cases()):
        ci, co, k, stride, pad, groups = geom
        out[f"conv{i}_geom"] = np.array(geom, np.int64)
        out[f"conv{i}_x"], out[f"conv{i}_w"], out[f"conv{i}_b"] = x, w, b
        out[f"conv{i}_out"] = ref.conv2d(x, w, b, stride, pad, groups)
    np.savez_compressed(os.path.join(HERE, "model_free.npz"), **out)
    print("wrote", os.path.join(HERE, "model_free.npz"), len(out), "arrays")


if __name__ == "__main__":
    main()
