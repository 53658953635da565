"""CPU: the UF16 bitstream container, the digests and the prepared-model
identity.  The writers must produce the reference's exact bytes and the
readers / scan_bitstream its exact results and error messages
(src/bitstream.cpp compiled from the reference), over systematic sweeps,
random streams and every truncation of a small stream."""
import hashlib

import numpy as np
import pytest

ID_I = hashlib.sha256(b"image").digest()
ID_V = hashlib.sha256(b"video").digest()


def outcome(fn, *args, **kw):
    """("ok", value) or ("err", message) of a call."""
    try:
        return "ok", fn(*args, **kw)
    except Exception as e:  # noqa: BLE001 -- compared as text
        return "err", str(e)


ADAPTIVE = [0, 1, 5, 126, 127, 128, 200, 255, 256, 16383, 16384, 65535, 65536, (1 << 24) - 1, 1 << 24,
            (1 << 30) - 1]


@pytest.mark.parametrize("v", ADAPTIVE)
def test_adaptive_integer_bytes(ufb, ref, v):
    mine = ufb.write_uint(v)
    assert mine == ref.bs_write_uint(v)
    assert len(mine) == (1 if v < 128 else 2 if v < 16384 else 4)
    assert ufb.read_uint(mine + b"\xff") == (v, len(mine))


def test_adaptive_integer_limit(ufb, ref):
    with pytest.raises(ufb.UfbError) as e:
        ufb.write_uint(1 << 30)
    assert e.value.code == -2
    assert outcome(ref.bs_write_uint, 1 << 30)[0] == "err"
    assert "30 bits" in str(e.value)


def test_adaptive_integer_non_canonical_and_truncated(ufb, ref):
    # a reader accepts longer forms than the writer emits (read_uint_adaptive)
    assert ufb.read_uint(b"\x80\x05") == (5, 2)
    assert ufb.read_uint(b"\xc0\x00\x00\x05") == (5, 4)
    # the SPS reader of the reference agrees on the same bytes
    stream = ufb.write_preamble(ID_I, ID_V) + b"\x00" + b"\x80\x40" + b"\xc0\x00\x00\x40"
    _, units = ref.bs_parse(stream)
    assert units == [{"type": 0, "sps_id": 0, "width": 64, "height": 64}]
    assert list(ufb.iter_nals(stream, 72)) == units
    for cut in (b"\x80", b"\xc0\x00", b"\xc0\x00\x00"):
        with pytest.raises(ufb.UfbError) as e:
            ufb.read_uint(cut)
        assert str(e.value) == "Truncated UF bitstream" and e.value.code == -4


def test_preamble_and_sps_bytes(ufb, ref):
    assert ufb.write_preamble(ID_I, ID_V) == ref.bs_write_preamble(ID_I, ID_V)
    assert ufb.write_preamble(ID_I, ID_V)[:8] == b"UF16\x01\x00\x00\x00"
    for sid in (0, 7, 15):
        for w, h in ((626, 352), (1, 1), (1920, 1088), (127, 128), (16384, 2), ((1 << 30) - 1, 3)):
            assert ufb.write_sps(sid, w, h) == ref.bs_write_sps(sid, w, h), (sid, w, h)
    for bad in ((16, 64, 64), (0, 0, 64), (0, 64, 0)):
        with pytest.raises(ufb.UfbError) as e:
            ufb.write_sps(*bad)
        assert e.value.code == -1
        assert outcome(ref.bs_write_sps, *bad) == ("err", "Invalid UF SPS")


@pytest.mark.parametrize("n", [0, 1, 127, 128, 16383, 16384, 70000])
def test_packet_bytes(ufb, ref, n):
    rng = np.random.default_rng(n)
    payload = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
    for nal_type, sid, qp, ep, reset in ((1, 0, 0, 1, False), (2, 15, 255, 127, True), (2, 3, 20, 1, True),
                                         (1, 9, 63, 0, True)):
        mine = ufb.write_packet(nal_type, sid, qp, ep, reset, payload)
        assert mine == ref.bs_write_packet(nal_type, sid, qp, ep, reset, payload)


def test_packet_writer_rejects(ufb, ref):
    for bad in ((0, 0, 0, 1, False), (3, 0, 0, 1, False), (1, 16, 0, 1, False), (1, 0, 0, 128, False)):
        with pytest.raises(ufb.UfbError) as e:
            ufb.write_packet(*bad, b"x")
        assert e.value.code == -1 and str(e.value) == "Invalid UF packet"
        assert outcome(ref.bs_write_packet, *bad, b"x") == ("err", "Invalid UF packet")


def _random_stream(rng, ufb, packets=None, corrupt=False):
    """A UF16 stream of random SPS and packet units (valid unless corrupt)."""
    parts = [ufb.write_preamble(ID_I, ID_V)]
    dims = (int(rng.integers(1, 3000)), int(rng.integers(1, 3000)))
    parts.append(ufb.write_sps(0, *dims))
    n = int(rng.integers(1, 12)) if packets is None else packets
    for i in range(n):
        if rng.random() < 0.15:  # a repeated or extra SPS
            sid = int(rng.integers(0, 16))
            parts.append(ufb.write_sps(sid, *dims))
        t = 1 if i == 0 or rng.random() < 0.2 else 2
        payload = rng.integers(0, 256, int(rng.choice([0, 3, 130, 17000])), dtype=np.uint8).tobytes()
        parts.append(ufb.write_packet(t, 0, int(rng.integers(0, 64)), int(rng.integers(1, 4)),
                                      bool(rng.integers(0, 2)), payload))
    data = b"".join(parts)
    if corrupt:
        b = bytearray(data)
        for _ in range(int(rng.integers(1, 4))):
            b[int(rng.integers(0, len(b)))] = int(rng.integers(0, 256))
        data = bytes(b)
    return data


@pytest.mark.parametrize("seed", range(24))
def test_random_streams_scan_and_parse(ufb, ref, seed):
    rng = np.random.default_rng(1000 + seed)
    data = _random_stream(rng, ufb, corrupt=seed % 3 == 2)
    for variant in ("htl", "ld"):
        for expected in (None, 1, 9, 17, 40):
            mine = outcome(ufb.scan_bitstream, data, variant, expected)
            theirs = outcome(ref.bs_scan, data, variant, expected)
            assert mine == theirs, (variant, expected)
    mine = outcome(lambda: list(ufb.iter_nals(data, ufb.read_preamble(data)[1])))
    theirs = outcome(lambda: ref.bs_parse(data)[1])
    assert mine == theirs


def test_every_truncation_matches_reference(ufb, ref):
    rng = np.random.default_rng(7)
    data = _random_stream(rng, ufb, packets=3)
    assert len(data) < 40000
    for cut in list(range(0, 120)) + list(range(120, len(data), 97)) + [len(data) - 1]:
        part = data[:cut]
        assert outcome(ufb.scan_bitstream, part, "htl") == outcome(ref.bs_scan, part, "htl"), cut


def test_scan_structure_errors(ufb, ref):
    pre = ufb.write_preamble(ID_I, ID_V)
    sps0, sps1 = ufb.write_sps(0, 64, 64), ufb.write_sps(1, 32, 64)
    i_pkt = ufb.write_packet(1, 0, 0, 1, False, b"ab")
    p_pkt = ufb.write_packet(2, 0, 20, 1, True, b"cd")
    cases = {
        "empty": (b"", "htl", None),
        "fp16 stream without packets": (sps0, "htl", None),
        "fp16 stream": (sps0 + i_pkt + p_pkt, "hts", 9),
        "bad signature": (b"UX16" + pre[4:] + sps0 + i_pkt, "htl", None),
        "bad version": (pre[:4] + b"\x02\x00\x00\x00" + pre[8:] + sps0 + i_pkt, "htl", None),
        "unknown sps": (pre + i_pkt, "htl", None),
        "starts with P": (pre + sps0 + p_pkt, "htl", None),
        "dimension change": (pre + sps0 + sps1 + i_pkt + ufb.write_packet(2, 1, 20, 1, False, b""), "htl", None),
        "extra packet": (pre + sps0 + i_pkt + p_pkt + p_pkt, "htl", 9),
        "too few": (pre + sps0 + i_pkt + p_pkt, "htl", 10),
        "no parallelism": (pre + sps0 + ufb.write_packet(1, 0, 0, 0, False, b""), "htl", None),
        "bad nal type": (pre + sps0 + i_pkt + b"\x30", "htl", None),
        "bad variant": (pre + sps0 + i_pkt, "lx", None),
        "zero dimension": (pre + b"\x00\x00\x05" + i_pkt, "htl", None),
        "ld chunks": (pre + sps0 + i_pkt + p_pkt + p_pkt, "ld", 3),
    }
    for name, (data, variant, expected) in cases.items():
        mine = outcome(ufb.scan_bitstream, data, variant, expected)
        assert mine == outcome(ref.bs_scan, data, variant, expected), name
    assert outcome(ufb.scan_bitstream, pre + sps0 + i_pkt + p_pkt, "htl", 10) == (
        "err", "UF bitstream has too few coded frames")


def test_fp16_preamble_consumes_nothing(ufb):
    sps0 = ufb.write_sps(0, 64, 64)
    info, pos = ufb.read_preamble(sps0)
    assert info["integer"] is False and pos == 0
    info, pos = ufb.read_preamble(b"")
    assert info["integer"] is False and pos == 0


@pytest.mark.parametrize("n", [0, 1, 55, 56, 63, 64, 65, 1000, 1 << 20])
def test_sha256_matches_hashlib(ufb, n):
    data = np.random.default_rng(n).integers(0, 256, n, dtype=np.uint8).tobytes()
    assert ufb.sha256(data) == hashlib.sha256(data).digest()


@pytest.mark.parametrize("variant,seed", [("image", 1), ("htl", 2)])
def test_prepared_identity_of_synthetic_models(ufb, syn, variant, seed):
    import oracle.stream as st
    t = syn.prepared(variant, seed)
    source = hashlib.sha256(variant.encode()).hexdigest()
    want = st.prepared_identity(t, variant, source)
    assert ufb.prepared_identity(t, variant, source) == want
    # any change to a tensor, the variant or the source changes it
    t2 = dict(t)
    name = sorted(t2)[0]
    a = t2[name].copy()
    a.reshape(-1)[0] ^= 1
    t2[name] = a
    assert ufb.prepared_identity(t2, variant, source) != want
    assert ufb.prepared_identity(t, variant, source[::-1]) != want


def test_prepared_identity_names_and_dtypes(ufb):
    import oracle.stream as st
    rng = np.random.default_rng(5)
    t = {
        "plain": rng.integers(-9, 9, (3, 4)).astype(np.int16),
        'quote"back\\slash': rng.integers(0, 255, 7).astype(np.uint8),
        "tab\tnew\nline\x01": np.arange(6, dtype=np.int32).reshape(2, 3),
        "café ☃ \U0001f600 \x7f": np.array([-1, 2], np.int8),
        "Zed": np.array(5, np.int64),
        "empty": np.zeros((0, 3), np.int16),
    }
    assert ufb.prepared_identity(t, "htl", "x") == st.prepared_identity(t, "htl", "x")
    assert ufb.prepared_identity({}, "image") == st.prepared_identity({}, "image")


def test_interrupt_flag(ufb):
    assert not ufb.interrupt_requested()
    ufb.set_interrupt(True)
    try:
        assert ufb.interrupt_requested()
    finally:
        ufb.set_interrupt(False)
    assert not ufb.interrupt_requested()
