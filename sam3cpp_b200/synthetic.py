"""Seeded synthetic SAM 3 vision-trunk weights and images.

No checkpoint is available offline, so every test and benchmark runs on
random-init weights of the real architecture, written as GGUF files the way
the reference's converter writes them (tools/convert_mlx_sam3_to_gguf.py):

* tensor names hashed to ``t_<sha1[:12]>`` (convert:378-380, :489) with the
  ``<file>.tensor_map.json`` sidecar mapping short -> original name
  (convert:596-598), which the loader resolves like src/gguf_model.cpp:28-47;
* weight types per scheme (convert:223-269): ``f32`` everything F32;
  ``f16`` the 2-D linears and the 4-D patch-embed F16, biases / norms /
  pos_embed F32; ``q8_0`` the 2-D linears Q8_0, patch-embed F16 (not 2-D),
  biases / norms / pos_embed F32.

Values: numpy PCG64 ``default_rng(seed)`` drawn in tensor order
patch_embed, pos_embed, then blocks 0..31 (qkv.w, proj.w, fc1.w, fc2.w), each
N(0, 0.02) in float32; biases 0; LayerNorm gamma 1, beta 0 (``perturb=True``
draws biases and LN affine terms too, for tests that must see them).  F16
files hold the same values cast to fp16; Q8_0 files quantize the F32 values
with gguf-py's Q8_0 quantizer (bit-identical to ggml's quantize_row_q8_0_ref).
Images are NCHW fp32 uniform[-1, 1], image i from ``default_rng(1000 + i)``.
"""

from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path

import numpy as np

PREFIX = "backbone.vision_backbone.trunk"
DIM, MLP, LAYERS, PATCH, IMG, GRID = 1024, 4736, 32, 14, 1008, 72
GLOBAL_LAYERS = (7, 15, 23, 31)

GGML_F32, GGML_F16, GGML_Q8_0 = 0, 1, 8
FORMATS = {"f32": GGML_F32, "f16": GGML_F16, "q8_0": GGML_Q8_0}


def short_name(name: str) -> str:
    return "t_" + hashlib.sha1(name.encode()).hexdigest()[:12]


def trunk_tensor_names(layers: int = LAYERS) -> list[str]:
    names = [f"{PREFIX}.patch_embed.proj.weight", f"{PREFIX}.pos_embed",
             f"{PREFIX}.ln_pre.weight", f"{PREFIX}.ln_pre.bias"]
    for i in range(layers):
        b = f"{PREFIX}.blocks.{i}"
        names += [f"{b}.norm1.weight", f"{b}.norm1.bias", f"{b}.attn.qkv.weight", f"{b}.attn.qkv.bias",
                  f"{b}.attn.proj.weight", f"{b}.attn.proj.bias", f"{b}.norm2.weight", f"{b}.norm2.bias",
                  f"{b}.mlp.fc1.weight", f"{b}.mlp.fc1.bias", f"{b}.mlp.fc2.weight", f"{b}.mlp.fc2.bias"]
    return names


def make_f32_weights(seed: int = 0, layers: int = LAYERS, perturb: bool = False) -> dict[str, np.ndarray]:
    """Float32 master weights, numpy shapes as the MLX checkpoint stores them."""
    rng = np.random.default_rng(seed)
    std = np.float32(0.02)

    def normal(*shape):
        return rng.standard_normal(shape, dtype=np.float32) * std

    w: dict[str, np.ndarray] = {}
    w[f"{PREFIX}.patch_embed.proj.weight"] = normal(DIM, PATCH, PATCH, 3)   # [O, KH, KW, I]
    w[f"{PREFIX}.pos_embed"] = normal(1, 24 * 24 + 1, DIM)
    for i in range(layers):
        b = f"{PREFIX}.blocks.{i}"
        w[f"{b}.attn.qkv.weight"] = normal(3 * DIM, DIM)
        w[f"{b}.attn.proj.weight"] = normal(DIM, DIM)
        w[f"{b}.mlp.fc1.weight"] = normal(MLP, DIM)
        w[f"{b}.mlp.fc2.weight"] = normal(DIM, MLP)
    prng = np.random.default_rng(seed + 7919) if perturb else None

    def vec(n, base):
        if prng is None:
            return np.full(n, base, np.float32)
        return (np.float32(base) + prng.standard_normal(n, dtype=np.float32) * np.float32(0.1)).astype(np.float32)

    w[f"{PREFIX}.ln_pre.weight"] = vec(DIM, 1.0)
    w[f"{PREFIX}.ln_pre.bias"] = vec(DIM, 0.0)
    for i in range(layers):
        b = f"{PREFIX}.blocks.{i}"
        w[f"{b}.norm1.weight"] = vec(DIM, 1.0)
        w[f"{b}.norm1.bias"] = vec(DIM, 0.0)
        w[f"{b}.attn.qkv.bias"] = vec(3 * DIM, 0.0)
        w[f"{b}.attn.proj.bias"] = vec(DIM, 0.0)
        w[f"{b}.norm2.weight"] = vec(DIM, 1.0)
        w[f"{b}.norm2.bias"] = vec(DIM, 0.0)
        w[f"{b}.mlp.fc1.bias"] = vec(MLP, 0.0)
        w[f"{b}.mlp.fc2.bias"] = vec(DIM, 0.0)
    return w


NECK = "backbone.vision_backbone.convs"
# The SAM 3 neck (src/vision_neck.cpp:262-347): output channels of each conv
# and, per level, the layers in order.  MLX layouts: Conv2d and
# ConvTranspose2d weights [OC, KH, KW, IC].
NECK_LAYERS = {
    0: [("dconv_2x2_0", 512, 2, DIM), ("dconv_2x2_1", 256, 2, 512), ("conv_1x1", 256, 1, 256), ("conv_3x3", 256, 3, 256)],
    1: [("dconv_2x2", 512, 2, DIM), ("conv_1x1", 256, 1, 512), ("conv_3x3", 256, 3, 256)],
    2: [("conv_1x1", 256, 1, DIM), ("conv_3x3", 256, 3, 256)],
    3: [("conv_1x1", 256, 1, DIM), ("conv_3x3", 256, 3, 256)],
}


def make_neck_weights(seed: int = 0, identity_3x3: bool = False) -> dict[str, np.ndarray]:
    """Seeded neck weights (default_rng(seed + 104729), drawn level by level in
    NECK_LAYERS order): conv/deconv weights N(0, 0.02), biases N(0, 0.1).
    identity_3x3 replaces every conv_3x3 by the identity (centre tap 1 on the
    diagonal, bias 0), so a level's output equals its 1x1 conv's output."""
    rng = np.random.default_rng(seed + 104729)
    w: dict[str, np.ndarray] = {}
    for lvl, layers in NECK_LAYERS.items():
        for name, oc, k, ic in layers:
            key = f"{NECK}.{lvl}.{name}"
            wt = rng.standard_normal((oc, k, k, ic), dtype=np.float32) * np.float32(0.02)
            b = rng.standard_normal(oc, dtype=np.float32) * np.float32(0.1)
            if identity_3x3 and name == "conv_3x3":
                wt = np.zeros((oc, k, k, ic), np.float32)
                wt[np.arange(oc), 1, 1, np.arange(oc)] = 1.0
                b = np.zeros(oc, np.float32)
            w[key + ".weight"], w[key + ".bias"] = wt, b
    return w


def is_sensitive(name: str) -> bool:
    """convert_mlx_sam3_to_gguf.py:223-229 (bias, *norm*, pos_embed stay F32)."""
    low = name.lower()
    return name.endswith(".bias") or "norm" in low or "pos_embed" in low


def tensor_qtype(name: str, arr: np.ndarray, fmt: str) -> int:
    """Type the converter assigns (convert:243-269) for scheme f32_ref / f16_ref / q8_0."""
    if fmt == "f32" or is_sensitive(name):
        return GGML_F32
    if fmt == "q8_0" and arr.ndim == 2:
        return GGML_Q8_0
    return GGML_F16


def quantize_q8_0_rows(x: np.ndarray) -> np.ndarray:
    """Q8_0 bytes of a float32 [rows, K] array (34-byte blocks: fp16 d + 32 int8).

    Same arithmetic as ggml's quantize_row_q8_0_ref (ggml-quants.c:199-221):
    d = amax/127, id = 1/d, q = roundf(x*id) (half away from zero).
    """
    rows, k = x.shape
    blocks = x.reshape(-1, 32).astype(np.float32)
    d = np.abs(blocks).max(axis=1, keepdims=True) / np.float32(127)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    v = blocks * inv
    q = (np.sign(v) * np.floor(np.abs(v) + np.float32(0.5))).astype(np.int8)
    out = np.concatenate([d.astype(np.float16).view(np.uint8), q.view(np.uint8)], axis=1)
    return out.reshape(rows, (k // 32) * 34)


def encode_tensor(name: str, arr: np.ndarray, fmt: str) -> tuple[int, np.ndarray]:
    qt = tensor_qtype(name, arr, fmt)
    if qt == GGML_F32:
        return qt, np.ascontiguousarray(arr, np.float32)
    if qt == GGML_F16:
        return qt, np.ascontiguousarray(arr.astype(np.float16))
    return qt, quantize_q8_0_rows(arr)


def write_gguf(path: str | os.PathLike, weights: dict[str, np.ndarray], fmt: str,
               hashed_names: bool = True) -> Path:
    """Write a trunk GGUF (+ tensor_map.json sidecar when names are hashed)."""
    from gguf import GGUFWriter, GGMLQuantizationType

    path = Path(path)
    # A per-process partial name: processes that create the same file at once
    # each write their own copy and the last atomic rename wins.
    tmp = path.with_suffix(path.suffix + f".{os.getpid()}.partial")
    writer = GGUFWriter(str(tmp), arch="sam3")
    writer.add_int32("sam3.image_size", IMG)
    writer.add_int32("sam3.patch_size", PATCH)
    layers = sum(1 for n in weights if n.endswith(".attn.qkv.weight"))
    writer.add_int32("sam3.vision_layers", layers)
    name_map = {}
    for name in weights:
        qt, data = encode_tensor(name, weights[name], fmt)
        out_name = short_name(name) if hashed_names else name
        name_map[out_name] = name
        if qt == GGML_Q8_0:
            writer.add_tensor(out_name, data, raw_dtype=GGMLQuantizationType.Q8_0)
        else:
            writer.add_tensor(out_name, data)
    writer.write_header_to_file()
    writer.write_kv_data_to_file()
    writer.write_tensors_to_file()
    writer.close()
    if hashed_names:   # the sidecar first: a file that exists has its names
        side = Path(str(path) + ".tensor_map.json")
        side_tmp = side.with_suffix(f".{os.getpid()}.partial")
        with open(side_tmp, "w") as f:
            json.dump(name_map, f, indent=2, sort_keys=True)
        os.replace(side_tmp, side)
    os.replace(tmp, path)
    return path


def cache_dir() -> Path:
    """Where seeded files are cached: $S3T_CACHE, else s3t_synth in the
    system's temporary directory (outside the source tree: the full-size
    files are 0.5-1.8 GB)."""
    import tempfile
    d = Path(os.environ.get("S3T_CACHE") or Path(tempfile.gettempdir()) / "s3t_synth")
    d.mkdir(parents=True, exist_ok=True)
    return d


def synthetic_gguf(fmt: str, seed: int = 0, layers: int = LAYERS, perturb: bool = False, neck: bool = False,
                   identity_3x3: bool = False) -> Path:
    """Path of the cached seeded GGUF for ``fmt`` (created on first use);
    neck=True appends the seeded neck weights (make_neck_weights)."""
    tag = (f"sam3_trunk_{fmt}_s{seed}_L{layers}{'_p' if perturb else ''}"
           f"{('_neck' + ('_id3' if identity_3x3 else '')) if neck else ''}.gguf")
    p = cache_dir() / tag
    if not p.exists():
        w = make_f32_weights(seed, layers, perturb)
        if neck:
            w.update(make_neck_weights(seed, identity_3x3))
        write_gguf(p, w, fmt)
    return p


def synthetic_image(i: int, dtype=np.float32) -> np.ndarray:
    """Image i: [1, 3, 1008, 1008] uniform[-1, 1] from default_rng(1000 + i)."""
    rng = np.random.default_rng(1000 + i)
    return rng.uniform(-1.0, 1.0, size=(1, 3, IMG, IMG)).astype(dtype)


def synthetic_images(n: int, start: int = 0) -> np.ndarray:
    return np.concatenate([synthetic_image(start + i) for i in range(n)], axis=0)
