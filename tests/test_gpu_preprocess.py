"""Device image preprocessing and the uint8 trunk entry point.

s3t_preprocess_rgb8 must reproduce the reference's bilinear_resize_rgb
(tools/sam3_vision_trunk.cpp:33-66) bit for bit: it is compared with the
golden hashes made from the reference itself and with the oracle.
s3t_trunk_run_rgb8 must equal s3t_trunk_run on the oracle-preprocessed image
exactly (same fp32 image, same kernels).
"""

import hashlib
import json

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

CASES = json.loads((GOLDEN / "preprocess.json").read_text())


@pytest.fixture(scope="module")
def gpu(torch_cuda):
    import sam3cpp_b200
    sam3cpp_b200.lib()
    return sam3cpp_b200


def _image(i):
    c = CASES["cases"][i]
    return np.random.default_rng(c["seed"]).integers(0, 256, (c["height"], c["width"], 3), dtype=np.uint8)


def _device_preprocess(gpu, torch, imgs):
    src = torch.from_numpy(np.ascontiguousarray(imgs)).cuda()
    b, h, w = imgs.shape[:3]
    out = torch.empty((b, 3, 1008, 1008), dtype=torch.float32, device="cuda")
    gpu.preprocess_rgb8(0, src.data_ptr(), w, h, b, out.data_ptr())
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("i", range(len(CASES["cases"])))
def test_preprocess_bit_exact(gpu, torch_cuda, oracle, i):
    img = _image(i)
    got = _device_preprocess(gpu, torch_cuda, img[None])[0]
    sha = hashlib.sha256(np.ascontiguousarray(got, "<f4").tobytes()).hexdigest()
    assert sha == CASES["cases"][i]["sha256"]
    assert np.array_equal(got.view(np.uint32), oracle.bilinear_resize_rgb(img).view(np.uint32))


def test_preprocess_batch(gpu, torch_cuda, oracle):
    rng = np.random.default_rng(5)
    imgs = rng.integers(0, 256, (3, 61, 45, 3), dtype=np.uint8)
    got = _device_preprocess(gpu, torch_cuda, imgs)
    for b in range(3):
        assert np.array_equal(got[b].view(np.uint32), oracle.bilinear_resize_rgb(imgs[b]).view(np.uint32))


def test_preprocess_errors(gpu, torch_cuda):
    buf = torch_cuda.zeros(16, dtype=torch_cuda.uint8, device="cuda")
    out = torch_cuda.empty(3 * 1008 * 1008, dtype=torch_cuda.float32, device="cuda")
    for w, h, b in ((0, 4, 1), (4, -1, 1), (40000, 4, 1), (4, 4, 0)):
        with pytest.raises(gpu.S3TError, match="width and height|batch"):
            gpu.preprocess_rgb8(0, buf.data_ptr(), w, h, b, out.data_ptr())
    with pytest.raises(gpu.S3TError, match="null"):
        gpu.preprocess_rgb8(0, 0, 4, 4, 1, out.data_ptr())


def test_trunk_rgb8_matches_trunk(gpu, oracle):
    """Host uint8 images through s3t_trunk_run_rgb8 == s3t_trunk_run on the
    oracle's preprocessing of the same images (2-layer perturbed model)."""
    from sam3cpp_b200 import synthetic as s
    trunk = gpu.VisionTrunk(gpu.GgufModel(s.synthetic_gguf("f16", seed=0, layers=2, perturb=True)))
    rng = np.random.default_rng(9)
    imgs = rng.integers(0, 256, (2, 480, 640, 3), dtype=np.uint8)
    got = trunk.run_rgb8(imgs)
    pre = np.stack([oracle.bilinear_resize_rgb(im) for im in imgs])
    want = trunk.run_batch(pre)
    assert got.shape == (2, 1024, 72, 72)
    assert np.array_equal(got, want)
    # a different source size on the same context (the staging buffer grows)
    big = rng.integers(0, 256, (1500, 2000, 3), dtype=np.uint8)
    assert np.array_equal(trunk.run_rgb8(big)[0], trunk.run_batch(oracle.bilinear_resize_rgb(big)[None])[0])
