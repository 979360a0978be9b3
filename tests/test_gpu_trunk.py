"""Trunk-level parity of the CUDA path with the oracle, per weight format.

The bar: per-element relative L2 error <= 1e-2 and cosine similarity >=
0.999 against the CPU result of the same GGUF file.  Reduced-depth runs use
s3t_trunk_run_layers (the reference's export tool dumps the same per-layer
tensors); the 32-layer runs compare with golden outputs of the reference's
own VisionTrunk::run.

Q8_0 weights: ggml re-quantizes every GEMM input to Q8_0, so a 1e-7 change
of summation order flips int8 roundings that compound over the layers.  The
reference itself, built for AVX2 and for AVX-512 from the same sources, lands
1.56e-2 apart on the seeded Q8_0 file (F16: 5.1e-4).  For Q8_0 the relative
L2 bound is therefore max(1e-2, 1.25 x the measured spread of the reference /
oracle under a pure summation-order change), with cosine >= 0.999 kept.
"""

import numpy as np
import pytest

from conftest import GOLDEN, cosine, rel_l2

pytestmark = pytest.mark.gpu

REL_TOL, COS_TOL = 1e-2, 0.999


@pytest.fixture(scope="module")
def gpu(torch_cuda):
    import sam3cpp_b200
    sam3cpp_b200.lib()
    return sam3cpp_b200


def _models(fmt, layers, perturb):
    from oracle.pyoracle import TrunkTensors
    from sam3cpp_b200 import synthetic as s
    path = s.synthetic_gguf(fmt, seed=0, layers=layers, perturb=perturb)
    return path, TrunkTensors(path)


@pytest.mark.parametrize("fmt", ["f16", "q8_0", "f32"])
def test_stem_and_two_layers(gpu, oracle, fmt):
    """Patch embed + pos + ln_pre, then blocks 0-1 (windowed), with nonzero
    biases and LayerNorm affine terms."""
    from sam3cpp_b200 import synthetic as s
    path, tt = _models(fmt, 2, True)
    model = gpu.GgufModel(path)
    assert model.n_layers == 2
    trunk = gpu.VisionTrunk(model)
    img = s.synthetic_image(3)
    for n in (0, 2):
        got = trunk.run_batch(img, n_layers=n)
        ref = oracle.trunk(tt, img, n)
        assert got.shape == (1, 1024, 72, 72)
        r, c = rel_l2(got, ref), cosine(got, ref)
        assert r <= (2e-3 if n == 0 else REL_TOL) and c >= COS_TOL, (fmt, n, r, c)


@pytest.mark.parametrize("fmt", ["f16", "q8_0"])
def test_eight_layers_with_global(gpu, oracle, fmt):
    """Blocks 0-7: seven windowed layers and the first global layer (7)."""
    from sam3cpp_b200 import synthetic as s
    path, tt = _models(fmt, 8, True)
    trunk = gpu.VisionTrunk(gpu.GgufModel(path))
    img = s.synthetic_image(4)
    got = trunk.run_batch(img)
    ref = oracle.trunk(tt, img, 8)
    tol = REL_TOL
    if fmt == "q8_0":
        oracle.set_sum_variant(1)
        try:
            alt = oracle.trunk(tt, img, 8)
        finally:
            oracle.set_sum_variant(0)
        spread = rel_l2(alt, ref)
        tol = max(REL_TOL, 1.25 * spread)
    r, c = rel_l2(got, ref), cosine(got, ref)
    assert r <= tol and c >= COS_TOL, (fmt, r, c, tol)


def test_batch_matches_single(gpu):
    """Images of a batch are independent: batch-3 and batch-2 outputs equal
    batch-1 runs bit for bit.  One and two images run fc2 stream-K (84 and 164
    tiles on the CTA pairs, split at different K blocks), three images whole
    tiles: the accumulator hand-over keeps the K sum sequential."""
    from sam3cpp_b200 import synthetic as s
    path, _ = _models("f16", 2, True)
    trunk = gpu.VisionTrunk(gpu.GgufModel(path))
    imgs = s.synthetic_images(3)
    batched = trunk.run_batch(imgs)
    pair = trunk.run_batch(imgs[1:3])
    for i in range(3):
        single = trunk.run_batch(imgs[i:i + 1])
        assert np.array_equal(batched[i], single[0])
        if i:
            assert np.array_equal(pair[i - 1], single[0])


def test_host_pipelined_batch_matches_single(gpu):
    """A host-buffer batch larger than one pipeline chunk (10 = 8 + 2 images)
    is uploaded, computed and downloaded in overlapping chunks; every image
    must equal its own batch-1 run."""
    from sam3cpp_b200 import synthetic as s
    path, _ = _models("f16", 2, True)
    trunk = gpu.VisionTrunk(gpu.GgufModel(path))
    imgs = s.synthetic_images(10)
    batched = trunk.run_batch(imgs)
    for i in (0, 7, 8, 9):
        single = trunk.run_batch(imgs[i:i + 1])
        assert np.array_equal(batched[i], single[0]), i


def test_reference_errors(gpu):
    """Shape and payload errors follow src/vision_trunk.cpp:301-306."""
    from sam3cpp_b200 import synthetic as s
    path, _ = _models("f16", 2, True)
    trunk = gpu.VisionTrunk(gpu.GgufModel(path))
    with pytest.raises(gpu.S3TError, match=r"expects NCHW image shape \[1, 3, 1008, 1008\]"):
        trunk.run(np.zeros(3 * 1008 * 1008, np.float32), [1, 3, 1008, 1007])
    with pytest.raises(gpu.S3TError, match="payload size mismatch"):
        trunk.run(np.zeros(10, np.float32), [1, 3, 1008, 1008])
    out = trunk.run(s.synthetic_image(0).reshape(-1), [1, 3, 1008, 1008])
    assert out.shape_nchw == [1, 1024, 72, 72] and np.isfinite(out.trunk_nchw).all()


def test_missing_tensor_error(gpu):
    from sam3cpp_b200 import synthetic as s
    w = s.make_f32_weights(0, layers=1)
    del w["backbone.vision_backbone.trunk.blocks.0.mlp.fc2.bias"]
    tensors = {}
    for name, arr in w.items():
        qt, raw = s.encode_tensor(name, arr, "f16")
        tensors[name] = (qt, raw, list(reversed(arr.shape)))
    with pytest.raises(gpu.S3TError, match="missing tensor: .*blocks.0.mlp.fc2.bias"):
        gpu.GgufModel.from_tensors(tensors)


@pytest.mark.slow
@pytest.mark.parametrize("fmt", ["f16", "q8_0", "f32"])
def test_full_trunk_vs_reference_golden(gpu, fmt):
    """32 layers on the seeded file vs the reference's VisionTrunk::run output
    (tests/golden/trunk_<fmt>_img0.npz: every 61st element of the output plus
    whole-tensor statistics)."""
    from sam3cpp_b200 import synthetic as s
    gold = np.load(GOLDEN / f"trunk_{fmt}_img0.npz")
    trunk = gpu.VisionTrunk(gpu.GgufModel(s.synthetic_gguf(fmt)))
    got = trunk.run(s.synthetic_image(0).reshape(-1), [1, 3, 1008, 1008]).trunk_nchw.reshape(-1)
    stride = int(gold["stride"])
    sample = got[::stride]
    ref = gold["sample"].astype(np.float32)
    tol = REL_TOL
    if fmt == "q8_0":
        tol = max(REL_TOL, 1.25 * float(gold["isa_spread_rel_l2"]))
    r, c = rel_l2(sample, ref), cosine(sample, ref)
    assert r <= tol and c >= COS_TOL, (fmt, r, c, tol)
    assert abs(float(got.astype(np.float64).mean()) - float(gold["mean"])) < 2e-2 * float(gold["std"])
    assert abs(float(got.std()) - float(gold["std"])) < 1e-2 * float(gold["std"])


def test_trunk_profile_pass(gpu, torch_cuda):
    """s3t_trunk_profile: an eager pass with per-launch events gives the same
    output as the graph-replayed trunk and counts every launch of the
    8-layer (one global block) model."""
    from sam3cpp_b200 import synthetic as s
    torch = torch_cuda
    path, _ = _models("f16", 8, True)
    trunk = gpu.VisionTrunk(gpu.GgufModel(path))
    imgs = torch.from_numpy(s.synthetic_images(2)).cuda()
    out_a = torch.empty((2, 1024, 72, 72), device="cuda")
    out_b = torch.empty_like(out_a)
    trunk.run_device(imgs.data_ptr(), 2, out_a.data_ptr())
    trunk.sync()
    prof = trunk.profile(imgs.data_ptr(), 2, out_b.data_ptr())
    assert torch.equal(out_a, out_b)
    counts = {k: v[1] for k, v in prof.items()}
    assert counts == {"stem": 1, "qkv": 8, "attn_windowed": 7, "attn_global": 1, "proj": 8,
                      "layernorm": 15, "fc1": 8, "fc2": 8}
    assert all(v[0] > 0 for v in prof.values())


def test_graph_cache_eviction(gpu, torch_cuda):
    """A caller that hands the trunk a fresh output buffer on every call makes
    the context capture a graph per (input, output) pair; beyond 16 the least
    recently used graph is dropped, and every run still computes the same."""
    from sam3cpp_b200 import synthetic as s
    torch = torch_cuda
    path, _ = _models("f16", 2, True)
    trunk = gpu.VisionTrunk(gpu.GgufModel(path))
    img = torch.from_numpy(s.synthetic_images(1)).cuda()
    outs = [torch.empty((1, 1024, 72, 72), device="cuda") for _ in range(19)]
    for o in outs + outs[:3]:
        trunk.run_device(img.data_ptr(), 1, o.data_ptr())
    trunk.sync()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
