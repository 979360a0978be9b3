"""Pin the neck's first-operation graphs (oracle/ref_harness.cpp
ref_neck_first) to the reference's own sam3::VisionNeck::run.

Note on the reference's 2x2 deconv (deconv2d_bias with input_ch_first false,
src/vision_neck.cpp:94-105): it prepares its input with
ggml_permute(x, 2, 0, 1, 3) on x = [W, H, IC].  ggml_permute sends source axis
i to position axis_i, so the result is [H, IC, W], not the [IC, W, H] the
comment there says; the [IC, W*H] reshape that follows therefore reads 1024
consecutive values of that [H, IC, W] array per column.  The harness and the
CUDA path reproduce this arithmetic, since parity is with the reference.

The file has the seeded neck with every conv_3x3 replaced by the identity
(centre tap 1 on the diagonal, bias 0) and F32 weights, so a level's output
is exactly what comes before its conv_3x3 (a sum whose other terms are exact
zeros).  Levels 2 and 3 then end in their first operation plus nothing: the
harness graph must equal VisionNeck::run bit for bit.  Levels 0 and 1 continue
past the first operation (deconv, GELU, 1x1 conv); numpy carries the harness's
first-operation output through those remaining layers and must land on
VisionNeck::run's output, which pins the deconv's pixel-shuffle layout.
"""

import numpy as np
import pytest

from conftest import rel_l2


@pytest.fixture(scope="module")
def neck_model(reference):
    from sam3cpp_b200 import synthetic as s
    m = reference.load(s.synthetic_gguf("f32", seed=0, layers=1, neck=True, identity_3x3=True), 0)
    yield m
    m.close()


def trunk_like(seed=11):
    return (np.random.default_rng(seed).standard_normal((1, 1024, 72, 72)) * 2.0).astype(np.float32)


@pytest.mark.parametrize("level", [2, 3])
def test_conv_levels_equal_reference_neck(neck_model, level):
    x = trunk_like()
    first = neck_model.neck_first(level, x)
    full = neck_model.neck_run(level, x)
    assert first.shape == full.shape == ((1, 256, 72, 72) if level == 2 else (1, 256, 36, 36))
    assert np.array_equal(first.view(np.uint32), full.view(np.uint32))


def _deconv(x, w, b):
    # x [IC, H, W] already in the deconv's input order; w MLX [OC, KH, KW, IC] -> [OC, 2H, 2W]
    oc, _, _, ic = w.shape
    h, wd = x.shape[1:]
    y = np.einsum("okli,ihw->ohkwl", w.astype(np.float64), x.astype(np.float64)).reshape(oc, 2 * h, 2 * wd)
    return y + b[:, None, None]


def reference_deconv_input(x):
    """x [C, H, W] (the trunk's NCHW) -> the [C, H, W] array the reference's
    deconv actually multiplies: column t = w + W*h of its [IC, W*H] operand
    is values [1024 t, 1024 t + 1024) of x laid out as ggml [H, C, W]."""
    c, h, wd = x.shape
    flat = np.ascontiguousarray(np.transpose(x, (2, 0, 1))).reshape(-1)     # numpy [W][C][H] = ggml [H, C, W]
    return flat.reshape(h * wd, c).T.reshape(c, h, wd)


def _conv1x1(x, w, b):
    return np.einsum("oi,ihw->ohw", w[:, 0, 0, :].astype(np.float64), x.astype(np.float64)) + b[:, None, None]


def _gelu(x):
    from math import erf
    return 0.5 * x * (1.0 + np.vectorize(erf)(x / np.sqrt(2.0)))


@pytest.mark.parametrize("level", [0, 1])
def test_deconv_levels_continue_into_reference_neck(neck_model, level):
    from sam3cpp_b200 import synthetic as s
    w = s.make_neck_weights(0, identity_3x3=True)
    p = f"{s.NECK}.{level}."
    x = trunk_like()
    first = neck_model.neck_first(level, x)[0]
    assert first.shape == (512, 144, 144)
    xin = reference_deconv_input(x[0])
    if level == 0:
        ref_first = _gelu(_deconv(xin, w[p + "dconv_2x2_0.weight"], w[p + "dconv_2x2_0.bias"]))
        rest = _deconv(first, w[p + "dconv_2x2_1.weight"], w[p + "dconv_2x2_1.bias"])   # channel-first input
    else:
        ref_first = _deconv(xin, w[p + "dconv_2x2.weight"], w[p + "dconv_2x2.bias"])
        rest = first
    assert rel_l2(first, ref_first) < 1e-5
    rest = _conv1x1(rest, w[p + "conv_1x1.weight"], w[p + "conv_1x1.bias"])
    full = neck_model.neck_run(level, x)[0]
    assert full.shape == rest.shape
    assert rel_l2(rest, full) < 1e-5
