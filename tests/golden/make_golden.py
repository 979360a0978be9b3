"""Generate the golden fixtures in tests/golden/ from the reference itself.

Runs where the reference sources are available (oracle/_ref built by
`make -C oracle ref`): every expected value here is computed by the
reference's own code — ggml's CPU ops for the op-level vectors and
sam3::VisionTrunk::run for the full-trunk outputs — on seeded inputs.

    python tests/golden/make_golden.py            # op vectors + all three trunks
    python tests/golden/make_golden.py --ops-only
    python tests/golden/make_golden.py --preprocess-only
    python tests/golden/make_golden.py --mha-only
    python tests/golden/make_golden.py --blocks-only

Files:
  ops.npz                   inputs and ggml outputs of small op cases
  trunk_<fmt>_img0.npz      32-layer output on the seeded <fmt> file and image 0:
                            every STRIDE-th element, plus mean/std of all of it
  mha_d32.npz               ggml_flash_attn_ext with the encoder fusion's shapes
                            (8 heads of 32, scale 1/sqrt(32), F16 prompt mask;
                            src/encoder_fusion.cpp:63-88) on seeded fp16-exact
                            inputs: MHA_CASES
  mha_d32_decoder.npz       mha() of src/decoder.cpp:95-127 (mul_mat, soft_max_ext
                            with the prompt mask or the box bias, mul_mat) run by
                            ggml on seeded fp16-exact inputs: DECODER_CASES
  block_pin_<fmt>.npz       VisionTrunk::run on a file whose blocks other than k
                            (k in PIN_BLOCKS) are exact identities (all their
                            weights and biases zero): the reference's own
                            block_k(stem(image 0)), every PIN_STRIDE-th element
                            of the NCHW output; pins the harness's per-block
                            graphs (oracle/ref_harness.cpp ref_trunk_block)
  preprocess.json           the reference tool's bilinear_resize_rgb
                            (tools/sam3_vision_trunk.cpp:33-66) on seeded uint8
                            images of PREPROCESS_SIZES: sha256 of the fp32
                            output bytes and the values at PREPROCESS_PICKS
"""

from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from oracle.pyoracle import F16, F32, Q8_0, Reference  # noqa: E402
from sam3cpp_b200 import synthetic as s  # noqa: E402

STRIDE = 61
PIN_STRIDE = 211
PIN_BLOCKS = (0, 7)   # a windowed block and the first global one

# (height, width) of the seeded uint8 RGB test images: identity size,
# upsampling, downsampling, degenerate and odd sizes.  Image i is
# default_rng(100 + i).integers(0, 256, (h, w, 3), dtype=uint8).
PREPROCESS_SIZES = [(1008, 1008), (480, 640), (2000, 1500), (1, 1), (3, 7), (1009, 1007), (333, 2017)]


def preprocess_image(i: int) -> np.ndarray:
    h, w = PREPROCESS_SIZES[i]
    return np.random.default_rng(100 + i).integers(0, 256, (h, w, 3), dtype=np.uint8)


def preprocess_picks() -> np.ndarray:
    n = 3 * 1008 * 1008
    corners = [c * 1008 * 1008 + o for c in range(3) for o in (0, 1007, 1007 * 1008, n // 3 - 1)]
    return np.unique(np.concatenate([np.random.default_rng(7).integers(0, n, 64), corners])).astype(np.int64)


def preprocess_golden(ref: Reference) -> dict:
    import hashlib
    picks = preprocess_picks()
    cases = []
    for i, (h, w) in enumerate(PREPROCESS_SIZES):
        out = ref.bilinear_resize_rgb(preprocess_image(i)).reshape(-1)
        cases.append({"height": h, "width": w, "seed": 100 + i,
                      "sha256": hashlib.sha256(out.astype("<f4").tobytes()).hexdigest(),
                      "picks": [float(v) for v in out[picks]]})
    return {"reference": "tools/sam3_vision_trunk.cpp:33-66 bilinear_resize_rgb via oracle/_ref",
            "picks": [int(p) for p in picks], "cases": cases}


def op_vectors(ref: Reference) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(2024)
    out: dict[str, np.ndarray] = {}
    x = (rng.standard_normal(4096) * 3).astype(np.float32)
    x[::97] = 0
    x[:8] = [65519.9, 65520.0, 1e-6, 6e-8, -3e-5, 2.5e-8, -65504.0, 7e-5]
    out["fp16_in"] = x
    out["fp16_out"] = ref.fp16(x)
    out["q8act_in"] = x
    out["q8act_out"] = ref.quantize_q8_0_act(x)
    w = (rng.standard_normal((96, 256)) * 0.02).astype(np.float32)
    w[0, :32] = 0
    qw = s.quantize_q8_0_rows(w)
    out["q8w_bytes"] = qw
    out["q8w_f32"] = ref.to_float(Q8_0, qw, w.size)
    xa = rng.standard_normal((37, 256)).astype(np.float32)
    out["mm_x"] = xa
    out["mm_w_f32"] = w
    out["mm_w_f16"] = w.astype(np.float16).view(np.uint16)
    out["mm_w_q8"] = qw
    out["mm_y_f32"] = ref.mul_mat(F32, w, 96, 256, xa)
    out["mm_y_f16"] = ref.mul_mat(F16, out["mm_w_f16"], 96, 256, xa)
    out["mm_y_q8"] = ref.mul_mat(Q8_0, qw, 96, 256, xa)
    xn = (rng.standard_normal((16, 1024)) * 2 + 0.3).astype(np.float32)
    out["norm_x"] = xn
    out["norm_y"] = ref.norm(xn)
    # RoPE at window-local (24x24) positions and at a sample of the 72x72 grid
    xr = rng.standard_normal((576, 2, 64)).astype(np.float32)
    pos = np.arange(576)
    out["rope_x"] = xr
    out["rope_local"] = ref.rope_axial(xr, pos % 24, pos // 24, 1.0)
    pg = rng.choice(5184, 400, replace=False)
    out["rope_gpos"] = pg.astype(np.int32)
    xg = rng.standard_normal((400, 2, 64)).astype(np.float32)
    out["rope_gx"] = xg
    out["rope_global"] = ref.rope_axial(xg, pg % 72, pg // 72, np.float32(24) / np.float32(72))
    q, k, v = (rng.standard_normal((192, 2, 64)).astype(np.float32) for _ in range(3))
    out["fa_q"], out["fa_k"], out["fa_v"] = q, k, v
    out["fa_out"] = ref.flash_attn(q, k, v, 0.125)
    g = (rng.standard_normal(4000) * 3).astype(np.float32)
    out["gelu_x"] = g
    out["gelu_y"] = ref.gelu_erf(g)
    # patch embed of image 0 with seeded F16 weights (weights regenerated
    # from the seed by the test; every 997th output element stored)
    prng = np.random.default_rng(77)
    pw = (prng.standard_normal((1024, 14, 14, 3)) * 0.02).astype(np.float32).astype(np.float16)
    img = s.synthetic_image(0)
    pe16 = ref.patch_embed(F16, pw.view(np.uint16), img)
    out["patch_y_f16_sample"] = pe16.reshape(-1)[::997]
    return out


# (name, q_len, kv_len, mask kind): ragged lengths on both sides, a prompt-like
# cross attention with padded keys, a single key, a row set with every key
# masked, and several key blocks with a mask (rescaling across blocks).
MHA_CASES = [("cross", 150, 33, "prompt"), ("self", 150, 150, None), ("single", 20, 1, None),
             ("allmasked", 9, 5, "all"), ("long", 64, 200, "prompt")]


def mha_inputs(i: int):
    """Seeded inputs of MHA_CASES[i]: fp16 q [q_len][8][32], k/v [kv_len][8][32]
    and the fp32 key mask (or None)."""
    name, nq, nk, kind = MHA_CASES[i]
    rng = np.random.default_rng(4000 + i)
    q = (rng.standard_normal((nq, 8, 32)) * 1.5).astype(np.float16)
    k = (rng.standard_normal((nk, 8, 32)) * 1.5).astype(np.float16)
    v = rng.standard_normal((nk, 8, 32)).astype(np.float16)
    mask = None
    if kind == "prompt":
        mask = np.zeros(nk, np.float32)
        mask[rng.random(nk) < 0.3] = -np.inf
        mask[1] = -0.75          # one finite entry: added to the score
        mask[0] = 0.0            # at least one key takes part
    elif kind == "all":
        mask = np.full(nk, -np.inf, np.float32)
    return q, k, v, mask


# The decoder's three attentions at its 201 queries: self attention, the text
# cross attention with a padded prompt, and the image cross attention with a
# full [8][201][kv] relative-position bias (fewer keys than 5184 to keep the
# file small; the GPU tests run 5184 against the oracle).
DECODER_CASES = [("dec_self", 201, 201, None), ("dec_text", 201, 33, "prompt"), ("dec_image", 201, 70, "bias")]


def decoder_inputs(i: int):
    name, nq, nk, kind = DECODER_CASES[i]
    rng = np.random.default_rng(4100 + i)
    q = (rng.standard_normal((nq, 8, 32)) * 1.5).astype(np.float16)
    k = (rng.standard_normal((nk, 8, 32)) * 1.5).astype(np.float16)
    v = rng.standard_normal((nk, 8, 32)).astype(np.float16)
    mask = bias = None
    if kind == "prompt":
        mask = np.zeros(nk, np.float32)
        mask[24:] = -np.inf
    elif kind == "bias":
        bias = (rng.standard_normal((8, nq, nk)) * 2.0).astype(np.float32)
        bias[:, :, 3] = -np.inf      # a key no query of any head may use
    return q, k, v, mask, bias


def decoder_golden(ref: Reference) -> dict[str, np.ndarray]:
    scale = float(np.float32(1.0) / np.sqrt(np.float32(32.0)))
    out = {}
    for i, (name, nq, nk, kind) in enumerate(DECODER_CASES):
        q, k, v, mask, bias = decoder_inputs(i)
        o = ref.decoder_mha(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32), scale, bias=bias,
                            key_mask=mask)
        out[f"{name}_q"], out[f"{name}_k"], out[f"{name}_v"] = q, k, v
        if mask is not None:
            out[f"{name}_mask"] = mask
        if bias is not None:
            out[f"{name}_bias"] = bias
        out[f"{name}_out"] = o.astype(np.float32)
    return out


def mha_golden(ref: Reference) -> dict[str, np.ndarray]:
    scale = float(np.float32(1.0) / np.sqrt(np.float32(32.0)))
    out = {}
    for i, (name, nq, nk, kind) in enumerate(MHA_CASES):
        q, k, v, mask = mha_inputs(i)
        o = ref.flash_attn_masked(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32), scale, mask)
        out[f"{name}_q"], out[f"{name}_k"], out[f"{name}_v"] = q, k, v
        if mask is not None:
            out[f"{name}_mask"] = mask
        out[f"{name}_out"] = o.astype(np.float32)
    return out


def trunk_golden(ref: Reference, fmt: str, threads: int) -> dict:
    path = s.synthetic_gguf(fmt)
    img = s.synthetic_image(0)
    t0 = time.time()
    y, sec = ref.trunk(path, img, threads)
    flat = y.reshape(-1)
    return {
        "sample": flat[::STRIDE].astype(np.float32),
        "stride": np.int64(STRIDE),
        "mean": np.float64(flat.astype(np.float64).mean()),
        "std": np.float64(flat.astype(np.float64).std()),
        "absmax": np.float64(np.abs(flat).max()),
        "run_seconds": np.float64(sec),
        "threads": np.int64(threads),
        "wall": np.float64(time.time() - t0),
    }


def isolated_block_weights(k: int) -> dict[str, np.ndarray]:
    """The seeded 32-block weights with every block but k made an exact
    identity: a block whose weights and biases are all zero adds 0 to the
    residual twice (attention output 0 through proj, GELU(0) = 0 through fc2).
    Blocks 0..7 of the seeded files equal those of the seeded 8-layer file
    (same draws in the same order), which the pin test runs."""
    w = s.make_f32_weights(0, layers=8)
    full = s.make_f32_weights(0, layers=0)
    for i in range(s.LAYERS):
        b = f"{s.PREFIX}.blocks.{i}"
        for name, shape in (("attn.qkv", (3 * s.DIM, s.DIM)), ("attn.proj", (s.DIM, s.DIM)),
                            ("mlp.fc1", (s.MLP, s.DIM)), ("mlp.fc2", (s.DIM, s.MLP))):
            if i == k:
                full[f"{b}.{name}.weight"] = w[f"{b}.{name}.weight"]
                full[f"{b}.{name}.bias"] = w[f"{b}.{name}.bias"]
            else:
                full[f"{b}.{name}.weight"] = np.zeros(shape, np.float32)
                full[f"{b}.{name}.bias"] = np.zeros(shape[0], np.float32)
        for nm in ("norm1", "norm2"):
            full[f"{b}.{nm}.weight"] = np.ones(s.DIM, np.float32)
            full[f"{b}.{nm}.bias"] = np.zeros(s.DIM, np.float32)
    return full


def block_pin_golden(ref: Reference, fmt: str, threads: int) -> dict:
    import tempfile
    out = {"stride": np.int64(PIN_STRIDE), "blocks": np.array(PIN_BLOCKS, np.int64)}
    img = s.synthetic_image(0)
    with tempfile.TemporaryDirectory() as d:
        for k in PIN_BLOCKS:
            path = s.write_gguf(Path(d) / f"isolated_{k}.gguf", isolated_block_weights(k), fmt)
            y, _ = ref.trunk(path, img, threads)
            flat = y.reshape(-1)
            out[f"block{k}_sample"] = flat[::PIN_STRIDE].astype(np.float32)
            out[f"block{k}_mean"] = np.float64(flat.astype(np.float64).mean())
            out[f"block{k}_std"] = np.float64(flat.astype(np.float64).std())
            path.unlink()
    return out


def isa_spread(fmt: str, threads: int, gold: dict) -> dict:
    """Distance between two builds of the same reference code on the same file:
    the AVX2 build (libsam3ref_v3) against the golden AVX-512 build (v4).
    They differ only in SIMD summation order; for Q8_0 weights the activation
    re-quantization before every GEMM amplifies that into a large spread."""
    v3 = Reference(HERE.parents[1] / "oracle" / "_ref" / "libsam3ref_v3.so")
    y, _ = v3.trunk(s.synthetic_gguf(fmt), s.synthetic_image(0), threads)
    smp = y.reshape(-1)[::STRIDE].astype(np.float64)
    ref = gold["sample"].astype(np.float64)
    rel = float(np.linalg.norm(smp - ref) / np.linalg.norm(ref))
    cos = float(smp @ ref / (np.linalg.norm(smp) * np.linalg.norm(ref)))
    return {"isa_spread_rel_l2": np.float64(rel), "isa_spread_cos": np.float64(cos)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ops-only", action="store_true")
    ap.add_argument("--preprocess-only", action="store_true")
    ap.add_argument("--mha-only", action="store_true")
    ap.add_argument("--blocks-only", action="store_true")
    ap.add_argument("--formats", default="f16,q8_0,f32")
    ap.add_argument("--threads", type=int, default=8)
    a = ap.parse_args()
    ref = Reference()
    if a.blocks_only:
        for fmt in a.formats.split(","):
            np.savez_compressed(HERE / f"block_pin_{fmt}.npz", **block_pin_golden(ref, fmt, a.threads))
            print(f"block_pin_{fmt}.npz written", flush=True)
        return
    np.savez_compressed(HERE / "mha_d32.npz", **mha_golden(ref))
    np.savez_compressed(HERE / "mha_d32_decoder.npz", **decoder_golden(ref))
    print("mha_d32.npz, mha_d32_decoder.npz written")
    if a.mha_only:
        return
    (HERE / "preprocess.json").write_text(json.dumps(preprocess_golden(ref), indent=1))
    print("preprocess.json written")
    if a.preprocess_only:
        return
    np.savez_compressed(HERE / "ops.npz", **op_vectors(ref))
    print("ops.npz written")
    if a.ops_only:
        return
    meta = {}
    for fmt in a.formats.split(","):
        g = trunk_golden(ref, fmt, a.threads)
        g.update(isa_spread(fmt, a.threads, g))
        np.savez_compressed(HERE / f"trunk_{fmt}_img0.npz", **g)
        meta[fmt] = {k: float(v) for k, v in g.items() if k != "sample"}
        print(fmt, meta[fmt], flush=True)
    (HERE / "trunk_meta.json").write_text(json.dumps({"reference": str(ref.path.name), **meta}, indent=2))


if __name__ == "__main__":
    main()
