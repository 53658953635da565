"""CPU: the model-level golden digests (tests/golden/config*.json, written by
tests/golden/make_model_golden.py from the reference's CPU path) are
self-consistent, and the seeded synthetic inputs they were made from are
reproduced bit for bit here, so a GPU mismatch against them points at the
engine rather than at the input generator."""
import hashlib
import json
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def load(case):
    path = os.path.join(GOLDEN, f"{case}.json")
    if not os.path.exists(path):
        pytest.skip(f"{path} not generated")
    with open(path) as f:
        return json.load(f)


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("case", ["config3", "config4", "config5"])
def test_synthetic_input_reproduced(syn, case):
    g = load(case)
    video = syn.synthetic_video(g["width"], g["height"], g["frames"], g["video_seed"])
    assert sha(video) == g["input_sha256"]


def test_config3_reference_decoder_reproduces_its_encoder():
    """The reference's decoder reproduces its encoder's reconstructions and
    DPB states (the property the 1080p digests of config 5 rely on)."""
    g = load("config3")
    assert [p["type"] for p in g["packets"]] == ["I", "P", "P"]
    assert [p.get("reset") for p in g["packets"][1:]] == [True, False]
    for p in g["packets"]:
        assert p["decoded"] == p["frames"]
        assert len(p["frames"]["int16"]) == (1 if p["type"] == "I" else 8)
        if p["type"] == "P":
            assert p["decoded_states"] == p["states"]


def test_config4_structure():
    g = load("config4")
    # 1 I packet + ceil(119 / 8) P packets, every P packet resetting at reset_interval 8
    assert g["packets"] == 1 + (g["frames"] - 1 + 7) // 8 == 16
    assert len(g["frame_yuv_sha256"]) == g["frames"] == 120
    assert len(set(g["frame_yuv_sha256"])) == g["frames"]  # the scene moves: no two frames alike
