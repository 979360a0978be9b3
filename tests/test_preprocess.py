"""Pins of the image-preprocessing oracle (CPU only).

The oracle's or_bilinear_resize_rgb restates the reference tool's
bilinear_resize_rgb (tools/sam3_vision_trunk.cpp:33-66; the arithmetic of
src/pipeline.cpp:45-83 load_image_rgb).  It must match, bit for bit:
  * the golden hashes in tests/golden/preprocess.json, made by running the
    reference's own function (tests/golden/make_golden.py), and
  * the reference itself, live, when oracle/_ref is built.
"""

import hashlib
import json

import numpy as np
import pytest

from conftest import GOLDEN

CASES = json.loads((GOLDEN / "preprocess.json").read_text())


def _image(i):
    c = CASES["cases"][i]
    return np.random.default_rng(c["seed"]).integers(0, 256, (c["height"], c["width"], 3), dtype=np.uint8)


def _sha(out):
    return hashlib.sha256(np.ascontiguousarray(out, "<f4").tobytes()).hexdigest()


@pytest.mark.parametrize("i", range(len(CASES["cases"])))
def test_oracle_matches_reference_golden(oracle, i):
    c = CASES["cases"][i]
    out = oracle.bilinear_resize_rgb(_image(i))
    assert out.shape == (3, 1008, 1008)
    flat = out.reshape(-1)
    assert np.array_equal(flat[np.array(CASES["picks"])].astype(np.float32), np.array(c["picks"], np.float32))
    assert _sha(out) == c["sha256"], (c["height"], c["width"])


def test_oracle_matches_live_reference(oracle, reference):
    rng = np.random.default_rng(11)
    for h, w in ((17, 23), (1008, 5), (700, 1300)):
        img = rng.integers(0, 256, (h, w, 3), dtype=np.uint8)
        a, b = oracle.bilinear_resize_rgb(img), reference.bilinear_resize_rgb(img)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), (h, w)


def test_value_range_and_edges(oracle):
    """Constant images map to (u/255 - 0.5)/0.5 everywhere, including the
    extrapolated top/left edge of an upsampled image."""
    for u in (0, 128, 255):
        img = np.full((5, 9, 3), u, np.uint8)
        out = oracle.bilinear_resize_rgb(img)
        expect = (np.float32(u) / np.float32(255.0) - np.float32(0.5)) / np.float32(0.5)
        assert np.all(out == expect)
