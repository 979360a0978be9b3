"""Op-level parity of the CUDA kernels (through the C ABI) with the oracle.

Each op is checked on seeded inputs at sizes the oracle finishes in seconds,
including the tails the trunk has (M not a multiple of 128, N = 4736 with a
half tile, L = 576 and 5184 attention groups).
"""

import ctypes as C

import numpy as np
import pytest

from conftest import cosine, rel_l2

pytestmark = pytest.mark.gpu

F32, F16, Q8_0 = 0, 1, 8


@pytest.fixture(scope="module")
def s3t(torch_cuda):
    from sam3cpp_b200 import lib
    return lib()


def _p(t):
    return C.c_void_p(t.data_ptr())


def _ok(L, rc):
    assert rc == 0, L.s3t_last_error().decode()


@pytest.mark.parametrize("M,N,K", [(256, 3072, 1024), (200, 4736, 1024), (333, 1024, 4736), (5184, 1024, 640),
                                   (128, 256, 64)])
def test_gemm_f16_bias(s3t, torch_cuda, oracle, M, N, K):
    torch = torch_cuda
    rng = np.random.default_rng(M * 7 + N)
    x = rng.standard_normal((M, K)).astype(np.float16)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
    b = rng.standard_normal(N).astype(np.float32) * 0.1
    xd, wd, bd = (torch.from_numpy(a).cuda() for a in (x, w, b))
    yd = torch.empty((M, N), dtype=torch.float16, device="cuda")
    _ok(s3t, s3t.s3t_gemm_f16(0, _p(xd), _p(wd), _p(bd), M, N, K, 0, 0, _p(yd), None))
    _ok(s3t, s3t.s3t_device_status(0))
    ref = oracle.linear(F16, w.view(np.uint16), N, K, x.astype(np.float32), b)
    got = yd.float().cpu().numpy()
    assert rel_l2(got, ref) < 1e-3
    assert np.abs(got - ref).max() < 1e-2 * max(1.0, np.abs(ref).max())


@pytest.mark.parametrize("q8", [0, 1])
def test_gemm_gelu_q8(s3t, torch_cuda, oracle, q8):
    torch = torch_cuda
    M, N, K = 300, 4736, 1024
    rng = np.random.default_rng(11 + q8)
    x = rng.standard_normal((M, K)).astype(np.float16)
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float16)
    b = rng.standard_normal(N).astype(np.float32) * 0.5
    xd, wd, bd = (torch.from_numpy(a).cuda() for a in (x, w, b))
    yd = torch.empty((M, N), dtype=torch.float16, device="cuda")
    _ok(s3t, s3t.s3t_gemm_f16(0, _p(xd), _p(wd), _p(bd), M, N, K, 1, q8, _p(yd), None))
    _ok(s3t, s3t.s3t_device_status(0))
    ref = oracle.gelu_erf(oracle.linear(F16, w.view(np.uint16), N, K, x.astype(np.float32), b))
    if q8:
        ref = oracle.round_activations(Q8_0, ref)
    got = yd.float().cpu().numpy()
    assert rel_l2(got, ref) < (4e-3 if q8 else 1e-3)


@pytest.mark.parametrize("q8", [0, 1])
def test_layernorm(s3t, torch_cuda, oracle, q8):
    torch = torch_cuda
    rng = np.random.default_rng(3)
    rows = 1000
    x = (rng.standard_normal((rows, 1024)) * 3 + 0.7).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(1024)).astype(np.float32)
    bb = (0.1 * rng.standard_normal(1024)).astype(np.float32)
    xd, gd, bd = (torch.from_numpy(a).cuda() for a in (x, g, bb))
    yd = torch.empty((rows, 1024), dtype=torch.float16, device="cuda")
    _ok(s3t, s3t.s3t_layernorm(0, _p(xd), rows, _p(gd), _p(bd), _p(yd), q8, None))
    _ok(s3t, s3t.s3t_device_status(0))
    ref = oracle.layer_norm(x, g, bb)
    ref = oracle.round_activations(Q8_0 if q8 else F16, ref)
    got = yd.float().cpu().numpy()
    assert rel_l2(got, ref) < (3e-3 if q8 else 1e-3)


def test_dequant_bit_exact(s3t, torch_cuda, oracle):
    """The file-format dequantization on the device (s3t_dequantize, to fp32)
    is bit-identical to ggml's dequantize_row_q8_0 / fp16->fp32 (restated by
    the oracle).  This proves the decoding of the GGUF bytes; the operand the
    trunk's GEMMs consume is checked by test_gemm_weight_operand_bit_exact."""
    torch = torch_cuda
    from sam3cpp_b200.synthetic import quantize_q8_0_rows
    rng = np.random.default_rng(9)
    w = (rng.standard_normal((512, 1024)) * 0.02).astype(np.float32)
    w[3, :32] = 0.0                         # a zero block (d = 0)
    w[7, 5] = 10.0                          # an outlier
    q = quantize_q8_0_rows(w).reshape(-1)
    n = w.size
    qd = torch.from_numpy(q).cuda()
    yd = torch.empty(n, dtype=torch.float32, device="cuda")
    _ok(s3t, s3t.s3t_dequantize(Q8_0, _p(qd), n, _p(yd), None))
    torch.cuda.synchronize()
    assert np.array_equal(yd.cpu().numpy().view(np.uint32), oracle.dequantize(Q8_0, q, n).view(np.uint32))
    h = w.astype(np.float16)
    hd = torch.from_numpy(h.view(np.uint16).reshape(-1).view(np.int16)).cuda()
    _ok(s3t, s3t.s3t_dequantize(F16, _p(hd), n, _p(yd), None))
    torch.cuda.synchronize()
    assert np.array_equal(yd.cpu().numpy().view(np.uint32), oracle.dequantize(F16, h.view(np.uint16), n).view(np.uint32))


def test_gemm_weight_operand_bit_exact(s3t, torch_cuda):
    """The fp16 operand the trunk's GEMMs consume (s3t_weight_operand, the
    conversion s3t_finalize_weights applies): for Q8_0 it is fp16(q*d), the
    exact product of dequantize_row_q8_0 rounded to nearest even fp16 -- not
    q*d itself, which needs up to 19 significant bits; for F32 it is the
    round-to-nearest-even fp16 of the weight; F16 weights pass unchanged."""
    torch = torch_cuda
    from sam3cpp_b200.synthetic import quantize_q8_0_rows
    rng = np.random.default_rng(10)
    w = (rng.standard_normal((256, 1024)) * 0.02).astype(np.float32)
    w[3, :32] = 0.0
    w[7, 5] = 10.0
    w[9, 64:96] = np.linspace(-1e-3, 1e-3, 32)   # scale d in the fp16 subnormal range
    n = w.size
    raw = quantize_q8_0_rows(w)
    d = raw.reshape(-1, 34)[:, :2].copy().view(np.float16).astype(np.float64)
    q = raw.reshape(-1, 34)[:, 2:].view(np.int8).astype(np.float64)
    expect = (q * d).reshape(-1).astype(np.float16)          # float64 -> fp16 rounds to nearest even
    out = torch.empty(n, dtype=torch.float16, device="cuda")
    src = torch.from_numpy(raw.reshape(-1)).cuda()
    _ok(s3t, s3t.s3t_weight_operand(Q8_0, _p(src), n, _p(out), None))
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint16), expect.view(np.uint16))
    src = torch.from_numpy(w.reshape(-1)).cuda()
    _ok(s3t, s3t.s3t_weight_operand(F32, _p(src), n, _p(out), None))
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint16), w.reshape(-1).astype(np.float16).view(np.uint16))
    h = torch.from_numpy(w.reshape(-1).astype(np.float16)).cuda()
    _ok(s3t, s3t.s3t_weight_operand(F16, _p(h), n, _p(out), None))
    torch.cuda.synchronize()
    assert torch.equal(out, h)


def _grouped_to_oracle(a, groups, L):
    # [groups*16][L][64] -> per group [L][16][64]
    return a.reshape(groups, 16, L, 64).transpose(0, 2, 1, 3)


@pytest.mark.parametrize("windowed,bf16", [(1, 0), (0, 0), (1, 1)])
def test_attention(s3t, torch_cuda, oracle, windowed, bf16):
    torch = torch_cuda
    L = 576 if windowed else 5184
    groups = 9 if windowed else 1
    rng = np.random.default_rng(21 + windowed)
    dt = torch.bfloat16 if bf16 else torch.float16
    q, k, v = (torch.from_numpy(rng.standard_normal((groups * 16, L, 64)).astype(np.float32)).to(dt).cuda()
               for _ in range(3))
    out = torch.empty((5184, 1024), dtype=dt, device="cuda")
    _ok(s3t, s3t.s3t_attention(0, _p(q), _p(k), _p(v), groups, L, windowed, bf16, _p(out), None))
    _ok(s3t, s3t.s3t_device_status(0))
    qf, kf, vf = (_grouped_to_oracle(t.float().cpu().numpy(), groups, L) for t in (q, k, v))
    got = out.float().cpu().numpy()
    ref = np.empty((5184, 1024), np.float32)
    for g in range(groups):
        o = oracle.attention(qf[g], kf[g], vf[g], 0.125).reshape(L, 1024)
        if windowed:
            wy, wx = divmod(g, 3)
            idx = np.array([(wy * 24 + i // 24) * 72 + wx * 24 + i % 24 for i in range(L)])
            ref[idx] = o
        else:
            ref[:] = o
    assert rel_l2(got, ref) < (1e-2 if bf16 else 2e-3)
    assert cosine(got, ref) > 0.9999


@pytest.mark.parametrize("windowed", [1, 0])
def test_rope(s3t, torch_cuda, oracle, windowed):
    torch = torch_cuda
    L = 576 if windowed else 5184
    rng = np.random.default_rng(5)
    x = rng.standard_normal((16, L, 64)).astype(np.float32)
    xd = torch.from_numpy(x).half().cuda()
    _ok(s3t, s3t.s3t_rope(0, _p(xd), 1, L, windowed, 0, None))
    torch.cuda.synchronize()
    grid = 24 if windowed else 72
    pos = np.arange(L)
    xin = xd.new_tensor(x).half().float().cpu().numpy()  # fp16-rounded input
    ref = oracle.rope_axial(xin.transpose(1, 0, 2), pos % grid, pos // grid, 1.0 if windowed else 24 / 72)
    got = xd.float().cpu().numpy().transpose(1, 0, 2)
    assert rel_l2(got, ref) < 1e-3


def test_bounded_wait_reports_timeout_and_device_stays_usable(s3t, torch_cuda):
    """Failure detection without a GPU fault: a device wait on an mbarrier that
    nothing arrives at gives up after its limit (100 ms here), the status word
    reports the timeout once, and the next kernels run normally."""
    torch = torch_cuda
    _ok(s3t, s3t.s3t_device_status(0))
    _ok(s3t, s3t.s3t_selftest_wait_timeout(0, 100))
    assert s3t.s3t_device_status(0) != 0
    assert "self-test" in s3t.s3t_last_error().decode()
    _ok(s3t, s3t.s3t_device_status(0))          # reported once, then cleared
    x = torch.randn(256, 1024, device="cuda", dtype=torch.float16)
    w = torch.randn(1024, 1024, device="cuda", dtype=torch.float16) * 0.02
    y = torch.empty(256, 1024, device="cuda", dtype=torch.float16)
    _ok(s3t, s3t.s3t_gemm_f16(0, _p(x), _p(w), None, 256, 1024, 1024, 0, 0, _p(y), None))
    _ok(s3t, s3t.s3t_device_status(0))
    ref = x.float() @ w.float().t()
    assert float((y.float() - ref).norm() / ref.norm()) < 1e-3
