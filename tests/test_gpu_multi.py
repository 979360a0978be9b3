"""The multi-GPU runner (s3t_multi_*): images sharded across the GPUs of one
node, one weight replica per GPU, features gathered to the first GPU by peer
copies.  Every image must come out bit-identical to a single-GPU run of the
same image, whatever GPU computed it and however it travelled.  Needs two or
more GPUs (skipped otherwise)."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def two_gpus(torch_cuda):
    if torch_cuda.cuda.device_count() < 2:
        pytest.skip("needs 2 or more GPUs")
    return torch_cuda


def _single(path, imgs):
    import sam3cpp_b200 as s3t
    trunk = s3t.VisionTrunk(s3t.GgufModel(path, device=0))
    return np.concatenate([trunk.run_batch(imgs[i:i + 1]) for i in range(len(imgs))])


def test_host_buffers_match_single_gpu(two_gpus):
    import sam3cpp_b200 as s3t
    from sam3cpp_b200 import synthetic as s
    path = s.synthetic_gguf("f16", seed=0, layers=2, perturb=True)
    imgs = s.synthetic_images(5)                     # shards of 3 and 2 images
    multi = s3t.MultiTrunk(path, [0, 1])
    assert multi.n_devices == 2
    got = multi.run_batch(imgs)
    assert np.array_equal(got, _single(path, imgs))


def test_device_buffers_gathered_to_first_gpu(two_gpus):
    """10 images on GPU 0: GPU 1 takes 5 of them in staged chunks of 4 and 1,
    peer-copies images in and features out while computing."""
    import sam3cpp_b200 as s3t
    from sam3cpp_b200 import synthetic as s
    torch = two_gpus
    path = s.synthetic_gguf("f16", seed=0, layers=2, perturb=True)
    imgs = s.synthetic_images(10)
    multi = s3t.MultiTrunk(path, [0, 1])
    dimg = torch.from_numpy(imgs).to("cuda:0")
    out = torch.empty((10, 1024, 72, 72), device="cuda:0")
    stream = torch.cuda.Stream(device=0)
    ref = _single(path, imgs)
    for _ in range(2):                               # a second run reuses the staging buffers
        out.zero_()
        torch.cuda.synchronize(0)
        multi.run_device(dimg.data_ptr(), 10, out.data_ptr(), stream.cuda_stream)
        multi.sync(stream.cuda_stream)
        assert np.array_equal(out.cpu().numpy(), ref)


def test_errors(two_gpus):
    import sam3cpp_b200 as s3t
    from sam3cpp_b200 import synthetic as s
    path = s.synthetic_gguf("f16", seed=0, layers=2, perturb=True)
    with pytest.raises(s3t.S3TError, match="listed twice"):
        s3t.MultiTrunk(path, [0, 0])
    with pytest.raises(s3t.S3TError, match="cannot open"):
        s3t.MultiTrunk("/nonexistent.gguf", [0, 1])
