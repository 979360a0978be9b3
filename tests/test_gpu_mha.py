"""Parity of the encoder-fusion attention kernel (s3t_mha_d32) through the C ABI.

The reference is mha() of src/encoder_fusion.cpp:63-88: ggml_flash_attn_ext,
prec F32, 8 heads of 32, scale 1/sqrt(32), with the prompt mask of :120-133
on the image-to-prompt cross attention; and mha() of src/decoder.cpp:95-127
(ggml_mul_mat + ggml_soft_max_ext) for the decoder's self, text and image
cross attention, the last with a full box relative-position bias
(S3T_MHA_BIAS).  Checked against the reference's own outputs
(tests/golden/mha_d32.npz, mha_d32_decoder.npz, made by
tests/golden/make_golden.py) and, at full sizes (5184 image tokens), against
the oracle.

Tolerance: the kernel takes fp16 (or bf16) q/k/v, accumulates in fp32 and
rounds P to the operand type, so it is compared within rel-L2 2e-3 (fp16) /
1e-2 (bf16) and cosine > 0.9999; rows whose keys are all masked must be 0
exactly, as in ggml's CPU kernel.
"""

import numpy as np
import pytest

from conftest import GOLDEN, cosine, rel_l2

pytestmark = pytest.mark.gpu

SCALE = float(np.float32(1.0) / np.sqrt(np.float32(32.0)))
CASES = ["cross", "self", "single", "allmasked", "long"]


@pytest.fixture(scope="module")
def s3t(torch_cuda):
    import sam3cpp_b200 as s
    s.lib()
    return s


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN / "mha_d32.npz")


def _run(s3t, torch, q, k, v, mask, flags=0, out_dtype=None):
    """q/k/v: host arrays [len][8][32] -> device run -> host fp32 [q_len][8][32]."""
    dt = torch.bfloat16 if flags & s3t.MHA_BF16 else torch.float16
    dq, dk, dv = (torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dt).cuda().reshape(a.shape[0], 256)
                  for a in (q, k, v))
    dm = None if mask is None else torch.from_numpy(np.ascontiguousarray(mask, np.float32)).cuda()
    odt = dt if flags & s3t.MHA_OUT_F16 else torch.float32
    out = torch.full((q.shape[0], 256), float("nan"), dtype=odt, device="cuda")
    s3t.mha_d32(0, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), 1, q.shape[0], k.shape[0],
                None if dm is None else dm.data_ptr(), out.data_ptr(), flags)
    torch.cuda.synchronize()
    assert s3t.lib().s3t_device_status(0) == 0
    return out.float().cpu().numpy().reshape(q.shape[0], 8, 32)


@pytest.mark.parametrize("case", CASES)
def test_mha_golden(s3t, torch_cuda, golden, case):
    q, k, v = golden[f"{case}_q"], golden[f"{case}_k"], golden[f"{case}_v"]
    mask = golden[f"{case}_mask"] if f"{case}_mask" in golden.files else None
    ref = golden[f"{case}_out"]
    got = _run(s3t, torch_cuda, q, k, v, mask)
    assert np.isfinite(got).all()
    if case == "allmasked":
        assert np.all(got == 0.0)
        return
    assert rel_l2(got, ref) < 2e-3, rel_l2(got, ref)
    assert cosine(got, ref) > 0.9999


def _inputs(seed, nq, nk, scale=1.5):
    rng = np.random.default_rng(seed)
    q = (rng.standard_normal((nq, 8, 32)) * scale).astype(np.float16).astype(np.float32)
    k = (rng.standard_normal((nk, 8, 32)) * scale).astype(np.float16).astype(np.float32)
    v = rng.standard_normal((nk, 8, 32)).astype(np.float16).astype(np.float32)
    return q, k, v


def test_mha_encoder_self_attention_full(s3t, torch_cuda, oracle):
    # Self attention of one encoder layer: 72 x 72 image tokens, no mask.
    # The oracle checks a spread of 320 query rows against all 5184 keys.
    q, k, v = _inputs(71, 5184, 5184)
    got = _run(s3t, torch_cuda, q, k, v, None)
    rows = np.linspace(0, 5183, 320).astype(np.int64)
    ref = oracle.attention_masked(q[rows], k, v, SCALE, None)
    assert rel_l2(got[rows], ref) < 2e-3
    assert cosine(got[rows], ref) > 0.9999
    assert np.isfinite(got).all()


def test_mha_encoder_cross_attention_full(s3t, torch_cuda, oracle):
    # Image-to-prompt cross attention: 5184 queries, 33 prompt keys, 9 padded.
    q, k, v = _inputs(72, 5184, 33)
    mask = np.zeros(33, np.float32)
    mask[24:] = -np.inf
    got = _run(s3t, torch_cuda, q, k, v, mask)
    ref = oracle.attention_masked(q, k, v, SCALE, mask)
    assert rel_l2(got, ref) < 2e-3
    assert cosine(got, ref) > 0.9999
    # Masked keys take no part: changing their values changes nothing.
    k2, v2 = k.copy(), v.copy()
    k2[24:] = 7.0
    v2[24:] = -3.0
    got2 = _run(s3t, torch_cuda, q, k2, v2, mask)
    assert np.array_equal(got, got2)


def test_mha_bf16_and_f16_output(s3t, torch_cuda, oracle, golden):
    q, k, v = golden["long_q"].astype(np.float32), golden["long_k"].astype(np.float32), golden["long_v"].astype(np.float32)
    mask = golden["long_mask"]
    import torch
    qb, kb, vb = (torch.from_numpy(a).to(torch.bfloat16).float().numpy() for a in (q, k, v))
    got = _run(s3t, torch_cuda, qb, kb, vb, mask, flags=s3t.MHA_BF16)
    ref = oracle.attention_masked(qb, kb, vb, SCALE, mask)
    assert rel_l2(got, ref) < 1e-2
    assert cosine(got, ref) > 0.999
    f32 = _run(s3t, torch_cuda, q, k, v, mask)
    f16 = _run(s3t, torch_cuda, q, k, v, mask, flags=s3t.MHA_OUT_F16)
    assert np.array_equal(f16, f32.astype(np.float16).astype(np.float32))


def test_mha_batched_sequences(s3t, torch_cuda, oracle):
    # Three sequences in one launch, ragged lengths, a mask row per sequence;
    # the middle sequence has every key masked (its output must be 0).
    import torch
    B, nq, nk = 3, 300, 70
    rng = np.random.default_rng(73)
    qs, ks, vs = zip(*(_inputs(80 + b, nq, nk) for b in range(B)))
    mask = np.zeros((B, nk), np.float32)
    mask[0, rng.random(nk) < 0.3] = -np.inf
    mask[0, 0] = 0.0
    mask[1, :] = -np.inf
    mask[2, 5] = -1.25
    dq, dk, dv = (torch.from_numpy(np.stack(a)).half().cuda().reshape(B, -1, 256) for a in (qs, ks, vs))
    dm = torch.from_numpy(mask).cuda()
    out = torch.full((B, nq, 256), float("nan"), device="cuda")
    s3t.mha_d32(0, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, nq, nk, dm.data_ptr(), out.data_ptr())
    torch.cuda.synchronize()
    assert s3t.lib().s3t_device_status(0) == 0
    got = out.cpu().numpy().reshape(B, nq, 8, 32)
    for b in range(B):
        ref = oracle.attention_masked(qs[b], ks[b], vs[b], SCALE, mask[b])
        if b == 1:
            assert np.all(got[b] == 0.0)
        else:
            assert rel_l2(got[b], ref) < 2e-3
            assert cosine(got[b], ref) > 0.9999
    # Batched and one-at-a-time launches give the same bits.
    one = _run(s3t, torch_cuda, qs[2], ks[2], vs[2], mask[2])
    assert np.array_equal(got[2], one)


def _run_bias(s3t, torch, q, k, v, bias):
    dq, dk, dv = (torch.from_numpy(np.ascontiguousarray(a, np.float32)).half().cuda().reshape(a.shape[0], 256)
                  for a in (q, k, v))
    db = torch.from_numpy(np.ascontiguousarray(bias, np.float32)).cuda()
    out = torch.full((q.shape[0], 256), float("nan"), device="cuda")
    s3t.mha_d32(0, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), 1, q.shape[0], k.shape[0], db.data_ptr(),
                out.data_ptr(), s3t.MHA_BIAS)
    torch.cuda.synchronize()
    assert s3t.lib().s3t_device_status(0) == 0
    return out.cpu().numpy().reshape(q.shape[0], 8, 32)


@pytest.mark.parametrize("case", ["dec_self", "dec_text", "dec_image"])
def test_mha_decoder_golden(s3t, torch_cuda, case):
    g = np.load(GOLDEN / "mha_d32_decoder.npz")
    q, k, v, ref = g[f"{case}_q"], g[f"{case}_k"], g[f"{case}_v"], g[f"{case}_out"]
    if f"{case}_bias" in g.files:
        got = _run_bias(s3t, torch_cuda, q, k, v, g[f"{case}_bias"])
    else:
        got = _run(s3t, torch_cuda, q, k, v, g[f"{case}_mask"] if f"{case}_mask" in g.files else None)
    assert np.isfinite(got).all()
    assert rel_l2(got, ref) < 2e-3, rel_l2(got, ref)
    assert cosine(got, ref) > 0.9999


def test_mha_decoder_image_cross_attention_full(s3t, torch_cuda, oracle):
    # The decoder's 201 queries against the 5184 image tokens with a bias per
    # head, query and key; some bias entries are -inf (keys that take no part).
    q, k, v = _inputs(74, 201, 5184)
    rng = np.random.default_rng(75)
    bias = (rng.standard_normal((8, 201, 5184)) * 2.0).astype(np.float32)
    bias[rng.random(bias.shape) < 0.05] = -np.inf
    got = _run_bias(s3t, torch_cuda, q, k, v, bias)
    ref = oracle.attention_softmax(q, k, v, SCALE, bias=bias)
    assert rel_l2(got, ref) < 2e-3
    assert cosine(got, ref) > 0.9999


def test_mha_split_key_ranges(s3t, torch_cuda, oracle):
    # Few query tiles against many keys: the kernel splits each tile's keys
    # into ranges and merges the partials.  Sequence 0 has a long run of masked
    # keys (whole ranges see nothing but -inf) and scattered masked keys;
    # sequence 1 has every key masked and must come out 0.
    import torch
    B, nq, nk = 2, 100, 2000
    rng = np.random.default_rng(77)
    qs, ks, vs = zip(*(_inputs(90 + b, nq, nk) for b in range(B)))
    mask = np.zeros((B, nk), np.float32)
    mask[0, 256:1280] = -np.inf
    mask[0, rng.random(nk) < 0.1] = -np.inf
    mask[0, 7] = 0.5
    mask[1, :] = -np.inf
    dq, dk, dv = (torch.from_numpy(np.stack(a)).half().cuda().reshape(B, -1, 256) for a in (qs, ks, vs))
    dm = torch.from_numpy(mask).cuda()
    for flags, odt in ((0, torch.float32), (s3t.MHA_OUT_F16, torch.float16)):
        out = torch.full((B, nq, 256), float("nan"), dtype=odt, device="cuda")
        s3t.mha_d32(0, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, nq, nk, dm.data_ptr(), out.data_ptr(), flags)
        torch.cuda.synchronize()
        assert s3t.lib().s3t_device_status(0) == 0
        got = out.float().cpu().numpy().reshape(B, nq, 8, 32)
        ref = oracle.attention_masked(qs[0], ks[0], vs[0], SCALE, mask[0])
        assert rel_l2(got[0], ref) < 2e-3
        assert cosine(got[0], ref) > 0.9999
        assert np.all(got[1] == 0.0)
    # The same rows without a mask, against the oracle too.
    out = torch.full((B, nq, 256), float("nan"), device="cuda")
    s3t.mha_d32(0, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, nq, nk, None, out.data_ptr())
    torch.cuda.synchronize()
    got = out.cpu().numpy().reshape(B, nq, 8, 32)
    for b in range(B):
        assert rel_l2(got[b], oracle.attention_masked(qs[b], ks[b], vs[b], SCALE, None)) < 2e-3


def test_mha_rejects_bad_arguments(s3t, torch_cuda):
    import torch
    x = torch.zeros((64, 256), dtype=torch.float16, device="cuda")
    out = torch.zeros((64, 256), dtype=torch.float32, device="cuda")
    with pytest.raises(s3t.S3TError, match="q_len"):
        s3t.mha_d32(0, x.data_ptr(), x.data_ptr(), x.data_ptr(), 1, 0, 64, None, out.data_ptr())
    with pytest.raises(s3t.S3TError, match="batch"):
        s3t.mha_d32(0, x.data_ptr(), x.data_ptr(), x.data_ptr(), 0, 64, 64, None, out.data_ptr())
    with pytest.raises(s3t.S3TError, match="aligned"):
        s3t.mha_d32(0, x.data_ptr() + 2, x.data_ptr(), x.data_ptr(), 1, 64, 64, None, out.data_ptr())
    with pytest.raises(s3t.S3TError, match="flags"):
        s3t.mha_d32(0, x.data_ptr(), x.data_ptr(), x.data_ptr(), 1, 64, 64, None, out.data_ptr(), 8)
    with pytest.raises(s3t.S3TError, match="BIAS"):
        s3t.mha_d32(0, x.data_ptr(), x.data_ptr(), x.data_ptr(), 1, 64, 64, None, out.data_ptr(), s3t.MHA_BIAS)
    assert s3t.lib().s3t_device_status(0) == 0
