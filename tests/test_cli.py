"""CPU: the stream command line's file handling -- raw YUV420 reading with the
reference's 2 x 2 chroma repetition (src/integer_codec.cpp:125-148), prepared
model tables in .npz form, argument parsing."""
import importlib.util
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def cli(ufb):
    spec = importlib.util.spec_from_file_location("ufb200_cli", os.path.join(ROOT, "dcvc-uf-int16-cpp_b200", "cli.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_yuv420_to_444_repeats_chroma(cli):
    w, h = 6, 4
    rng = np.random.default_rng(0)
    planar = rng.integers(0, 256, w * h * 3 // 2, dtype=np.uint8)
    full = cli.yuv420_to_444(planar, w, h)
    assert full.shape == (3, h, w)
    assert np.array_equal(full[0].ravel(), planar[:w * h])
    u = planar[w * h: w * h + w * h // 4].reshape(h // 2, w // 2)
    v = planar[w * h + w * h // 4:].reshape(h // 2, w // 2)
    for y in range(h):
        for x in range(w):
            assert full[1, y, x] == u[y // 2, x // 2] and full[2, y, x] == v[y // 2, x // 2]


def test_read_yuv420_file(cli, tmp_path):
    w, h = 8, 6
    frames = np.random.default_rng(1).integers(0, 256, (3, w * h * 3 // 2), dtype=np.uint8)
    path = tmp_path / "in.yuv"
    frames.tofile(path)
    got = cli.read_yuv420(str(path), w, h)
    assert got.shape == (3, 3, h, w)
    assert np.array_equal(got[2], cli.yuv420_to_444(frames[2], w, h))
    assert cli.read_yuv420(str(path), w, h, max_frames=2).shape[0] == 2
    with open(path, "ab") as f:
        f.write(b"\x00" * 5)
    with pytest.raises(ValueError, match="Truncated raw YUV420 frame"):
        cli.read_yuv420(str(path), w, h)
    with pytest.raises(ValueError, match="Invalid UF encode settings"):
        cli.read_yuv420(str(path), 7, h)


def test_model_npz_round_trip(cli, ufb, tmp_path):
    t = {"a.weight": np.arange(12, dtype=np.int16).reshape(3, 4), "tables.x": np.arange(5, dtype=np.uint8)}
    path = str(tmp_path / "m.npz")
    cli.save_model_npz(path, t, "image", "abc")
    variant, source, tensors = cli.load_model_npz(path)
    assert (variant, source) == ("image", "abc")
    assert sorted(tensors) == sorted(t) and all(np.array_equal(tensors[k], t[k]) for k in t)
    assert ufb.prepared_identity(tensors, variant, source) == ufb.prepared_identity(t, "image", "abc")
    np.savez(str(tmp_path / "bad.npz"), x=np.zeros(2))
    with pytest.raises(ValueError, match="not a prepared model table"):
        cli.load_model_npz(str(tmp_path / "bad.npz"))


def test_parser(cli):
    a = cli.parser().parse_args(["verify", "--image", "i.npz", "--input", "v.bin", "--frames", "9", "--packets", "2"])
    assert (a.command, a.frames, a.packets, a.video, a.skip_threshold) == ("verify", 9, 2, None, 0.2)
    with pytest.raises(SystemExit):
        cli.parser().parse_args(["encode", "--image", "i.npz", "--input", "x.yuv"])
