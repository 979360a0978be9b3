"""Synthetic model files follow the reference converter's contract
(tools/convert_mlx_sam3_to_gguf.py): hashed names + sidecar, per-tensor types."""

import hashlib
import json

import numpy as np

from sam3cpp_b200 import synthetic as s


def test_short_name_rule():
    n = "backbone.vision_backbone.trunk.blocks.3.attn.qkv.weight"
    assert s.short_name(n) == "t_" + hashlib.sha1(n.encode()).hexdigest()[:12]


def test_q8_0_quantizer_matches_gguf_py():
    from gguf import GGMLQuantizationType
    from gguf.quants import quantize
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((16, 256)) * 0.02).astype(np.float32)
    w[2, :32] = 0
    assert np.array_equal(s.quantize_q8_0_rows(w), quantize(w, GGMLQuantizationType.Q8_0))


def test_types_and_sidecar(tmp_path):
    from gguf import GGUFReader
    w = s.make_f32_weights(0, layers=1)
    for fmt, qkv_type in (("f32", 0), ("f16", 1), ("q8_0", 8)):
        p = s.write_gguf(tmp_path / f"m_{fmt}.gguf", w, fmt)
        side = json.loads((tmp_path / f"m_{fmt}.gguf.tensor_map.json").read_text())
        assert len(side) == len(w) == 16
        r = GGUFReader(str(p))
        types = {side[t.name]: int(t.tensor_type) for t in r.tensors}
        P = s.PREFIX
        assert types[f"{P}.blocks.0.attn.qkv.weight"] == qkv_type
        assert types[f"{P}.patch_embed.proj.weight"] == (0 if fmt == "f32" else 1)   # 4-D: never Q8_0
        assert types[f"{P}.pos_embed"] == 0 and types[f"{P}.blocks.0.norm1.weight"] == 0
        assert types[f"{P}.blocks.0.mlp.fc1.bias"] == 0
        # ln_pre.weight is neither a bias nor a "norm" tensor: the converter keeps the float type
        assert types[f"{P}.ln_pre.weight"] == (0 if fmt == "f32" else 1)


def test_weights_are_seeded_and_prefix_stable():
    a = s.make_f32_weights(0, layers=2)
    b = s.make_f32_weights(0, layers=3)
    k = f"{s.PREFIX}.blocks.1.mlp.fc2.weight"
    assert np.array_equal(a[k], b[k])
    assert abs(float(a[k].std()) - 0.02) < 1e-3
    img = s.synthetic_image(5)
    assert img.shape == (1, 3, 1008, 1008) and img.min() >= -1 and img.max() <= 1
