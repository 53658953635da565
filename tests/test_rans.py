"""CPU: the engine's host rANS coder produces the reference's exact bytes
(src/entropy.cpp compiled from the reference) and decodes them back,
including bypass escapes and stream-corruption errors."""
import numpy as np
import pytest


@pytest.fixture(scope="module")
def tables(syn):
    t = syn.prepared("htl", 2)
    return {k: t[k] for k in ("tables.z_cdf", "tables.z_lengths", "tables.y_cdf", "tables.y_lengths")}


def _parts(rng, sizes, lo=-6, hi=7, escapes=0.02):
    parts = []
    for n in sizes:
        sym = rng.integers(lo, hi, n)
        esc = rng.random(n) < escapes
        sym[esc] = rng.integers(-128, 128, esc.sum())
        idx = rng.integers(0, 128, n)
        parts.append(((sym.astype(np.int64) * 256 + idx).astype(np.int16), idx.astype(np.uint8),
                      sym.astype(np.int8)))
    return parts


@pytest.mark.parametrize("seed", range(4))
def test_encode_matches_reference_bytes(ufb, ref, tables, seed):
    rng = np.random.default_rng(seed)
    parts = _parts(rng, [int(rng.integers(0, 500)) for _ in range(4)])
    z = rng.integers(-20, 21, 6 * 128).astype(np.int8)
    qp = int(rng.integers(0, 64))
    mine = ufb.Rans(tables).encode([p[0] for p in parts], z, qp * 128, 128)
    theirs = ref.rans(tables).encode([p[0] for p in parts], z, qp * 128, 128)
    assert mine == theirs


@pytest.mark.parametrize("seed", range(3))
def test_decode_round_trip_and_reference(ufb, ref, tables, seed):
    rng = np.random.default_rng(10 + seed)
    parts = _parts(rng, [300, 0, 200, 123], escapes=0.05)
    z = rng.integers(-128, 128, 2 * 128).astype(np.int8)
    payload = ref.rans(tables).encode([p[0] for p in parts], z, 5 * 128, 128)
    zd, ys = ufb.Rans(tables).decode(payload, z.size, 5 * 128, 128, [p[1] for p in parts])
    assert np.array_equal(zd, z)
    for (_, _, sym), y in zip(parts, ys):
        assert np.array_equal(y, sym)
    zr, yr = ref.rans(tables).decode(payload, z.size, 5 * 128, 128, [p[1] for p in parts])
    assert np.array_equal(zr, zd) and all(np.array_equal(a, b) for a, b in zip(yr, ys))


def test_truncated_stream_is_an_error(ufb, tables):
    rng = np.random.default_rng(3)
    parts = _parts(rng, [400])
    z = rng.integers(-5, 6, 128).astype(np.int8)
    r = ufb.Rans(tables)
    payload = r.encode([parts[0][0]], z, 0, 128)
    with pytest.raises(ufb.UfbError) as e:
        r.decode(payload[: len(payload) // 3], z.size, 0, 128, [parts[0][1]])
    assert e.value.code == -4
    with pytest.raises(ufb.UfbError):
        r.decode(payload[:3], z.size, 0, 128, [parts[0][1]])


def test_invalid_index_and_z_range(ufb, tables):
    r = ufb.Rans(tables)
    with pytest.raises(ufb.UfbError):
        r.encode([np.array([200], np.int16)], np.zeros(4, np.int8), 0, 4)  # index 200 >= 128 rows
    with pytest.raises(ufb.UfbError):
        r.encode([], np.zeros(4, np.int8), 64 * 128, 128)  # Z rows out of range
