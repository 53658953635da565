"""TEST INFRASTRUCTURE ONLY: stream-level checkers.

* ``prepared_identity`` restates ``content_hash`` (src/prepared.cpp:64-105):
  the reference builds its header with Python's compact, sorted, ASCII-only
  ``json.dumps`` conventions, which this function uses directly, and hashes
  each tensor's descriptor and little-endian bytes in name order.
* ``RefStreamCodec`` runs the reference's own ``uf::IntegerCodec`` encode and
  decode loops (src/integer_codec.cpp:215-493, compiled from its sources into
  oracle/_ref) over in-memory frames and archives.
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
    """uf::IntegerCodec for one stream: the reference's own encode loop and
    decode loop (src/integer_codec.cpp:215-292, 405-493) compiled from its
    sources (``RefOracle.codec``), including its decoded-YUV SHA-256 over
    ``IntegerCodec::raw_frame`` (src/integer_codec.cpp:294-323)."""

    def __init__(self, ref, ora, image_tensors: dict, video_tensors: dict | None, image_identity: bytes,
                 video_identity: bytes = bytes(32), skip_threshold: float = 0.0, threads: int = 0):
        self.args = (image_tensors, bytes(image_identity).hex(), video_tensors,
                     bytes(video_identity).hex() if video_tensors is not None else "", "htl", skip_threshold,
                     threads)
        self.ref = ref
        self.size = None

    def encode(self, frames_u8, width, height, qp_i, qp_p, reset_interval=0, intra_period=-1):
        """frames_u8: [T, 3, height, width] uint8 YUV444 -> (bitstream, packets)."""
        data, _, packets = self.ref.codec(*self.args).encode(frames_u8, width, height, qp_i, qp_p, reset_interval,
                                                             intra_period)
        self.size = (width, height)
        return data, packets

    def decode(self, data: bytes, total_frames: int, total_packets: int):
        """-> (sha256 hex of the raw YUV420 frames, [frames], packets)."""
        integer, units = self.ref.bs_parse(data)
        sps = [u for u in units if u["type"] == 0]
        width, height = (sps[0]["width"], sps[0]["height"]) if sps else self.size
        digest, yuv, packets = self.ref.codec(*self.args).decode(data, total_frames, total_packets, width, height)
        return digest, yuv, packets
