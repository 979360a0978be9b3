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
