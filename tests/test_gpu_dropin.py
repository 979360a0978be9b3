"""Drop-in integration: the reference's own GgufModel loader (src/gguf_model.cpp,
compiled from the reference sources into oracle/_ref/libsam3ref_s3t.so) with
its src/vision_trunk.cpp replaced by sam3cpp_b200/dropin/vision_trunk.cpp,
i.e. the path pipeline.cpp and the sam3-vision-trunk CLI would take."""

from pathlib import Path

import numpy as np
import pytest

from conftest import GOLDEN, cosine, rel_l2

pytestmark = pytest.mark.gpu

LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libsam3ref_s3t.so"


@pytest.mark.skipif(not LIB.exists(), reason="oracle/_ref/libsam3ref_s3t.so not built (make -C oracle dropin)")
def test_reference_loader_with_dropin_trunk(torch_cuda):
    from oracle.pyoracle import Reference
    from sam3cpp_b200 import synthetic as s
    ref = Reference(LIB)
    got, _ = ref.trunk(s.synthetic_gguf("f16"), s.synthetic_image(0))
    gold = np.load(GOLDEN / "trunk_f16_img0.npz")
    sample = got.reshape(-1)[::int(gold["stride"])]
    r, c = rel_l2(sample, gold["sample"]), cosine(sample, gold["sample"])
    assert r <= 1e-2 and c >= 0.999, (r, c)
    # a second run reuses the cached device context of the same GgufModel path
    got2, _ = ref.trunk(s.synthetic_gguf("f16"), s.synthetic_image(0))
    assert np.array_equal(got, got2)


@pytest.mark.skipif(not LIB.exists(), reason="oracle/_ref/libsam3ref_s3t.so not built (make -C oracle dropin)")
def test_dropin_models_loaded_in_sequence_use_their_own_weights(torch_cuda):
    """ref_trunk_run loads a fresh GgufModel on its stack for every call, so
    consecutive models of different files usually share one address: each
    must still run on its own weights (the context cache is keyed by the
    loaded weights, not by the address alone)."""
    import sam3cpp_b200 as s3t
    from oracle.pyoracle import Reference
    from sam3cpp_b200 import synthetic as s
    ref = Reference(LIB)
    img = s.synthetic_image(1)
    for fmt in ("f16", "q8_0", "f16"):
        path = s.synthetic_gguf(fmt)
        got, _ = ref.trunk(path, img)
        own = s3t.VisionTrunk(s3t.GgufModel(path)).run(img.reshape(-1), [1, 3, 1008, 1008]).trunk_nchw
        assert np.array_equal(got, own), fmt
