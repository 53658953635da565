"""TEST INFRASTRUCTURE ONLY: stream-level checkers.

* ``prepared_identity`` restates ``content_hash`` (src/prepared.cpp:64-105):
  the reference builds its header with Python's compact, sorted, ASCII-only
  ``json.dumps`` conventions, which this function uses directly, and hashes
  each tensor's descriptor and little-endian bytes in name order.
* ``RefStreamCodec`` restates ``uf::IntegerCodec::encode`` and
  ``decode_stream_impl`` (src/integer_codec.cpp:215-292, 405-493) over the
  reference's own compiled ``IntegerModel`` (``RefModel``) and container writers
  and reader (``RefOracle.bs_*``, src/bitstream.cpp); frames are converted to
  YUV420 with the C oracle's ``raw_frame`` (src/integer_codec.cpp:294-323).
"""
from __future__ import annotations

import hashlib
import json

import numpy as np

PREPARED_FORMAT = "dcvc-uf-prepared-v1"
ARITHMETIC = "uf-int16-q9-w13-acc64-rna-sat-v1"
_TORCH_DTYPES = {np.dtype(np.int16): "torch.int16", np.dtype(np.uint8): "torch.uint8",
                 np.dtype(np.int32): "torch.int32", np.dtype(np.int8): "torch.int8",
                 np.dtype(np.int64): "torch.int64"}
CHUNK = 8


def _compact(value) -> bytes:
    return json.dumps(value, sort_keys=True, separators=(",", ":"), ensure_ascii=True).encode()


def prepared_identity(tensors: dict, variant: str, source_sha256: str = "", format: str = PREPARED_FORMAT,
                      arithmetic: str = ARITHMETIC) -> str:
    h = hashlib.sha256(_compact({"format": format, "arithmetic": arithmetic, "variant": variant,
                                 "source_sha256": source_sha256}))
    for name in sorted(tensors, key=lambda n: n.encode()):
        a = np.ascontiguousarray(tensors[name])
        h.update(_compact([name, _TORCH_DTYPES[a.dtype], [int(s) for s in a.shape]]))
        h.update(a.astype(a.dtype.newbyteorder("<"), copy=False).tobytes())
    return h.hexdigest()


class RefStreamCodec:
    """uf::IntegerCodec for one stream over the reference's CPU models."""

    def __init__(self, ref, ora, image_tensors: dict, video_tensors: dict | None, image_identity: bytes,
                 video_identity: bytes = bytes(32), skip_threshold: float = 0.0):
        self.ref, self.ora = ref, ora
        self.image = ref.model("image", image_tensors)
        self.video = ref.model("htl", video_tensors) if video_tensors is not None else None
        for m in (self.image, self.video):
            if m is not None:
                m.set_skip_threshold(skip_threshold)
        self.ids = (bytes(image_identity), bytes(video_identity) if video_tensors is not None else bytes(32))

    def encode(self, frames_u8, width, height, qp_i, qp_p, reset_interval=0, intra_period=-1):
        """frames_u8: [T, 3, height, width] uint8 YUV444 -> (bitstream, packets)."""
        if width % 2 or height % 2 or not 0 <= qp_i < 64 or not 0 <= qp_p < 64 or (
                intra_period > 1 and intra_period % CHUNK):
            raise ValueError("Invalid UF encode settings")
        r = self.ref
        out = r.bs_write_preamble(*self.ids) + r.bs_write_sps(0, width, height)
        count, packets, total = 0, 0, len(frames_u8)
        while count < total:
            intra = count == 0 or intra_period == 1 or (intra_period > 1 and count != 1 and
                                                        count % intra_period == 1)
            valid = min(1 if intra else CHUNK, total - count)
            chunk = [frames_u8[count + i] for i in range(valid)]
            if not intra:
                chunk += [chunk[-1]] * (CHUNK - valid)
            x = self.ora.from_bytes(np.concatenate(chunk, 0)[None])
            reset = not intra and reset_interval > 0 and (count + CHUNK) % reset_interval == 1
            if intra:
                payload, rec = self.image.compress(x, qp_i)
                if self.video is not None:
                    self.video.add_ref_feature_from_frame(rec[0])
            else:
                payload, _ = self.video.compress(x, qp_p, reset)
            out += r.bs_write_packet(1 if intra else 2, 0, qp_i if intra else qp_p, 1, reset, payload)
            count += valid
            packets += 1
        return out, packets

    def decode(self, data: bytes, total_frames: int, total_packets: int):
        """-> (sha256 hex of the raw YUV420 frames, [frames], packets)."""
        integer, units = self.ref.bs_parse(data)
        ids = data[8:40], data[40:72]
        if not integer or (bytes(ids[0]), bytes(ids[1])) != self.ids:
            raise ValueError("UF integer runtime/prepared-model identity mismatch")
        sps, digest, yuv, packets, first = {}, hashlib.sha256(), [], 0, True
        for u in units:
            if u["type"] == 0:
                sps[u["sps_id"]] = (u["width"], u["height"])
                continue
            if u["sps_id"] not in sps or len(yuv) >= total_frames:
                raise ValueError("Unexpected UF packet or unknown SPS")
            w, h = sps[u["sps_id"]]
            intra = u["type"] == 1
            if first and not intra:
                raise ValueError("UF stream must start with an I packet")
            first = False
            if intra:
                frames = self.image.decompress(u["payload"], w, h, u["qp"])
                if self.video is not None:
                    self.video.add_ref_feature_from_frame(frames[0])
            else:
                frames = self.video.decompress(u["payload"], w, h, u["qp"], u["reset"])
            for f in frames:
                if len(yuv) == total_frames:
                    break
                raw = self.ora.raw_frame(f[0], h, w)
                digest.update(raw.tobytes())
                yuv.append(raw)
            packets += 1
        if len(yuv) != total_frames or packets != total_packets:
            raise ValueError("Incomplete UF integer bitstream")
        return digest.hexdigest(), yuv, packets
