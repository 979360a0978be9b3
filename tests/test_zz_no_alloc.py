"""The allocation-free stem entry point, s3t_stem_noalloc, through the C ABI.

Some callers of this library cannot call cudaMalloc — for example a plugin
whose host application owns every device allocation.  s3t_stem_noalloc serves
them: its only scratch buffer is a static device array inside the library
(one image), so the call itself allocates nothing.  This test checks two
consecutive calls against the allocating path that computes the same stem,
s3t_trunk_run_layers(..., n_layers=0, ...), within the stem tolerance of
tests/test_gpu_trunk.py; that a further call leaves the GPU's free memory
unchanged (cudaMemGetInfo before and after); and that a batch beyond the
array, a misaligned pointer and a host pointer are rejected with an error.
It lives in a file of its own so that it is collected after the other tests.
"""

import ctypes as C

import numpy as np
import pytest

from conftest import cosine, rel_l2

pytestmark = pytest.mark.gpu

STEM_REL_TOL = 2e-3   # the stem bound used in tests/test_gpu_trunk.py


def test_stem_noalloc_matches_allocating_stem(torch_cuda):
    torch = torch_cuda
    import sam3cpp_b200 as s3t
    from sam3cpp_b200 import synthetic as syn

    L = s3t.lib()
    model = s3t.GgufModel(syn.synthetic_gguf("f16", seed=0, layers=2, perturb=True), device=0)
    trunk = s3t.VisionTrunk(model)
    out = torch.empty((5184, 1024), dtype=torch.float32, device="cuda")
    for i in (0, 1):   # two calls in a row, on different images
        img = syn.synthetic_image(20 + i)
        ref = trunk.run_batch(img, n_layers=0)                      # [1, 1024, 72, 72]
        dimg = torch.from_numpy(img).cuda()
        torch.cuda.synchronize()
        rc = L.s3t_stem_noalloc(model.ctx, C.c_void_p(dimg.data_ptr()), 1, C.c_void_p(out.data_ptr()), None)
        assert rc == 0, L.s3t_last_error().decode()
        assert L.s3t_device_status(0) == 0, L.s3t_last_error().decode()
        got = out.cpu().numpy().T.reshape(1, 1024, 72, 72)
        r, c = rel_l2(got, ref), cosine(got, ref)
        assert r <= STEM_REL_TOL and c >= 0.999, (i, r, c)

    # after the calls above (module loading and the array's address look-up
    # are done), one more call must not change the device's free memory
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    rc = L.s3t_stem_noalloc(model.ctx, C.c_void_p(dimg.data_ptr()), 1, C.c_void_p(out.data_ptr()), None)
    assert rc == 0, L.s3t_last_error().decode()
    assert L.s3t_device_status(0) == 0, L.s3t_last_error().decode()
    assert torch.cuda.mem_get_info()[0] == free_before

    rc = L.s3t_stem_noalloc(model.ctx, C.c_void_p(dimg.data_ptr()), 2, C.c_void_p(out.data_ptr()), None)
    assert rc == -1
    assert b"batch 2" in L.s3t_last_error()
    rc = L.s3t_stem_noalloc(model.ctx, C.c_void_p(dimg.data_ptr()), 1, C.c_void_p(out.data_ptr() + 4), None)
    assert rc == -1
    assert b"16-byte aligned" in L.s3t_last_error()
    host = np.empty((5184, 1024), np.float32)
    rc = L.s3t_stem_noalloc(model.ctx, C.c_void_p(dimg.data_ptr()), 1, C.c_void_p(host.ctypes.data), None)
    assert rc == -1
    assert b"not device memory" in L.s3t_last_error()
