"""The device-resident hand-off from the trunk to the vision neck: the first
operation of each neck level (s3t_neck_first) reads the trunk's NCHW output
where s3t_trunk_run left it on the device, with no device-to-host copy in
between, and must match the reference's own ggml graph of that operation
(oracle/_ref ref_neck_first, pinned to sam3::VisionNeck::run by
tests/test_neck_pins.py) run on the same trunk output.

Bar: relative L2 <= 5e-3 and cosine >= 0.9999 (fp16 operands and an fp16
result against ggml's F16 operands and f32 result); batch 2 equals two batch-1
runs bit for bit.  The test copies the trunk output to the host only to hand
it to the reference."""

import numpy as np
import pytest

from conftest import cosine, rel_l2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fmt", ["f16", "f32"])
def test_neck_first_operation_on_device_trunk_output(torch_cuda, reference, fmt):
    import sam3cpp_b200 as s3t
    from sam3cpp_b200 import synthetic as s
    torch = torch_cuda
    path = s.synthetic_gguf(fmt, seed=0, layers=2, perturb=True, neck=True)
    trunk = s3t.VisionTrunk(s3t.GgufModel(path))
    imgs = torch.from_numpy(s.synthetic_images(2)).cuda()
    feats = torch.empty((2, 1024, 72, 72), device="cuda")
    trunk.run_device(imgs.data_ptr(), 2, feats.data_ptr())           # output stays on the device
    ref = reference.load(path, 0)
    try:
        for level in range(4):
            shape = trunk.neck_first_shape(level)
            out = torch.empty((2,) + tuple(shape[1:]), device="cuda")
            trunk.neck_first_device(level, feats.data_ptr(), 2, out.data_ptr())
            one = torch.empty_like(out[:1])
            trunk.neck_first_device(level, feats[1:].data_ptr(), 1, one.data_ptr())
            trunk.sync()
            assert torch.equal(out[1:], one), level
            want = ref.neck_first(level, feats[0:1].cpu().numpy())
            got = out[0:1].cpu().numpy()
            assert got.shape == want.shape, (level, got.shape, want.shape)
            r, c = rel_l2(got, want), cosine(got, want)
            print(f"neck {fmt} level {level}: rel_l2 {r:.2e} cos {c:.7f}")
            assert r <= 5e-3 and c >= 0.9999, (fmt, level, r, c)
    finally:
        ref.close()


def test_neck_weights_absent(torch_cuda):
    import sam3cpp_b200 as s3t
    from sam3cpp_b200 import synthetic as s
    trunk = s3t.VisionTrunk(s3t.GgufModel(s.synthetic_gguf("f16", seed=0, layers=2, perturb=True)))
    with pytest.raises(s3t.S3TError, match="missing tensor: backbone.vision_backbone.convs.2.conv_1x1"):
        trunk.neck_first_shape(2)
